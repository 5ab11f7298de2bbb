// The full-attention word step: the gated attention layers (one in four) of the Qwen3-Next /
// Qwen3.5 / Qwen3.6 stacks, for one word of each of n_seq sequences, between the projections.
//
// Follows FullAttn::forward for one word (crates/engine/src/model_next.rs:666-720, rope :653-664,
// the KV cache KvBuf::append :74-130 without its roll): q = q_norm(q part of the wq output),
// gate = its second half, k = k_norm(wk output), rope on the first `rot` values of q and k at
// the word's position (non-interleaved halves, inverse frequencies base^(-2i/rot) in f64 rounded
// to f32), k and v appended to the sequence's cache at row len, then for every query head the
// softmax of q.K^T / sqrt(hd) over rows 0 .. len of its kv head (head h reads kv head
// h / (n_head / n_kv)) times V, times sigmoid(gate).
//
// Layout of the work (split-K decoding), three launches:
//   k_attn_prep: one warp per query head (normalised, rotated into the workspace) and per kv head
//     (the new k, normalised and rotated, and v written to the caches at row len);
//   k_attn_part: a CTA takes rpc cache rows of one kv head of one sequence (32 to 256: more when the
//     grid is many waves deep; grid = ceil(cap / rpc) x n_kv x n_seq; CTAs past the sequence's
//     length return at once), 32 rows at a time: one thread starts bulk copies (cp.async.bulk) into
//     shared memory of the chunk's K rows, its V rows and (first) the kv head's prepared query heads;
//     the CTA scores the rows for all query heads at once (each warp 4 rows, each lane hd / 32 values
//     of a row, the (head, row) sums finished by a reduce-scatter butterfly), updates the online
//     softmax (running max and total, earlier sums rescaled) and adds the probabilities times V;
//   k_attn_combine: per query head the chunks merged in parallel (max-rescaled) and the gate.
// The rows of K and V are read once: HBM-bound at long caches.
#include <math.h>

#include "cwx_common.cuh"

namespace cwx {

namespace att {
constexpr int W = 8;
constexpr int T = W * 32;
constexpr int CHUNK = 32;   // cache rows per step of a chunk CTA, 4 per warp
constexpr int MAX_G = 16;   // query heads per kv head
constexpr int MAX_HD = 256;
constexpr int HG = 4;       // query heads per scoring pass (4 heads x 4 rows: one sum per half-warp lane)
}  // namespace att

struct AttnArgs {
    int n_head, n_kv, hd, rot, n_split, cap;
    int rpc;  // cache rows per k_attn_part CTA (a multiple of CHUNK)
    float eps, scale;
    double freq_base;
    const float* qg;
    const float* k_new;
    const float* v_new;
    float* k_cache;
    float* v_cache;
    const int32_t* len;
    const int32_t* pos;
    const float* q_norm_w;
    const float* k_norm_w;
    float* qn;    // workspace: the normalised, rotated query heads (n_seq, n_head, hd)
    float* part;  // workspace: per chunk and query head the hd weighted sums (n_seq, n_kv, n_split, g, hd)
    float* ml;    // workspace: per chunk and query head the chunk's max and exp total (.., g, 2)
    float* out;
    int* err;
};

__device__ __forceinline__ float att_warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float att_warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// One level of the reduce-scatter butterfly over N values per lane: the lanes with bit N/2 set
// keep the upper half, the others the lower half, each adding its partner's copy.
template <int N>
__device__ __forceinline__ void rs_level(float* v, int lane) {
    constexpr int H = N / 2;
    const bool up = (lane & H) != 0;
#pragma unroll
    for (int i = 0; i < H; ++i) {
        const float send = up ? v[i] : v[i + H];
        const float keep = up ? v[i + H] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, H);
    }
}

// Rope on the first rot values of y (shared memory) at position p, by one warp.
__device__ void rope_row(float* y, int hd, int rot, double base, int p, int lane) {
    const int half = rot / 2;
    for (int i = lane; i < half; i += 32) {
        const float inv = (float)(1.0 / pow(base, (2.0 * i) / (double)rot));
        const float f = (float)p * inv;
        const float c = cosf(f), s = sinf(f);
        const float a = y[i], b = y[i + half];
        y[i] = a * c - b * s;
        y[i + half] = a * s + b * c;
    }
    __syncwarp();
}

// This lane's DPL values of a row (hd = 32 DPL floats at `row`): 16-byte pieces lane, lane + 32
// (DPL 8), so a warp's loads cover consecutive 512-byte spans (no shared-memory bank conflicts);
// q and k use the same mapping, which is all a dot product needs.
template <int DPL>
__device__ __forceinline__ void load_row(const float* row, int lane, float* k) {
    if (DPL == 8) {
        const float4 a = reinterpret_cast<const float4*>(row)[lane], b = reinterpret_cast<const float4*>(row)[lane + 32];
        k[0] = a.x; k[1] = a.y; k[2] = a.z; k[3] = a.w;
        k[4] = b.x; k[5] = b.y; k[6] = b.z; k[7] = b.w;
    } else if (DPL == 4) {
        const float4 a = reinterpret_cast<const float4*>(row)[lane];
        k[0] = a.x; k[1] = a.y; k[2] = a.z; k[3] = a.w;
    } else {
        const float2 a = reinterpret_cast<const float2*>(row)[lane];
        k[0] = a.x; k[1] = a.y;
    }
}

// Value j of this lane's DPL values under load_row's mapping.
template <int DPL>
__device__ __forceinline__ int dim_of(int lane, int j) {
    return DPL == 8 ? (j < 4 ? 4 * lane + j : 128 + 4 * lane + j - 4) : DPL * lane + j;
}

// Query head blockIdx.x < n_head of sequence blockIdx.y: normalised (candle's RmsNorm:
// x / sqrt(mean(x^2) + eps) * w, the squares summed per lane then by a butterfly) and rotated into
// the workspace;
// blockIdx.x = n_head + j: kv head j's new k (normalised, rotated) and v into the caches at row len.
// One warp each.
__global__ void __launch_bounds__(32) k_attn_prep(AttnArgs p) {
    __shared__ float y[att::MAX_HD];
    const int lane = threadIdx.x, seq = blockIdx.y, hd = p.hd;
    pdl_wait();
    // the length, the position, the head's row and its norm weights all requested at once (the row
    // does not depend on the length; a length out of range still leaves before any write)
    const bool qhead = (int)blockIdx.x < p.n_head;
    const int kvh = qhead ? 0 : blockIdx.x - p.n_head;
    const int64_t h = (int64_t)seq * p.n_head + (qhead ? blockIdx.x : 0);
    const int64_t nr = ((int64_t)seq * p.n_kv + kvh) * hd;
    const float* x = qhead ? p.qg + h * 2 * hd : p.k_new + nr;
    const float* w = qhead ? p.q_norm_w : p.k_norm_w;
    float xv[att::MAX_HD / 32], wv[att::MAX_HD / 32];
#pragma unroll
    for (int i = 0; i < att::MAX_HD / 32; ++i) {
        const int d = lane + 32 * i;
        xv[i] = d < hd ? x[d] : 0.f;
        wv[i] = d < hd ? w[d] : 0.f;
    }
    const int L = p.len[seq];
    const int P = p.pos[seq];
    if (L < 0 || L >= p.cap) {
        if (lane == 0 && blockIdx.x == 0) dev_error(p.err, DE_SHAPE);
        return;
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < att::MAX_HD / 32; ++i) ss += xv[i] * xv[i];
    ss = att_warp_sum(ss);
    const float r = sqrtf(ss / (float)hd + p.eps);
#pragma unroll
    for (int i = 0; i < att::MAX_HD / 32; ++i)
        if (lane + 32 * i < hd) y[lane + 32 * i] = xv[i] / r * wv[i];
    __syncwarp();
    rope_row(y, hd, p.rot, p.freq_base, P, lane);
    if (qhead) {
        for (int d = lane; d < hd; d += 32) p.qn[h * hd + d] = y[d];
    } else {
        const int64_t row = (((int64_t)seq * p.n_kv + kvh) * p.cap + L) * hd;
        for (int d = lane; d < hd; d += 32) {
            p.k_cache[row + d] = y[d];
            p.v_cache[row + d] = p.v_new[nr + d];
        }
    }
}

// Rows rpc blockIdx.x .. of kv head blockIdx.y of sequence blockIdx.z, 32 at a time; DPL = hd / 32.
// Dynamic shared memory: a chunk's K rows, its V rows (32 hd floats each) and the kv head's g
// prepared query heads (g hd), brought by bulk copies; the softmax runs online over the chunks
// (running max and total per query head, earlier sums rescaled), one partial result per CTA.
// G: the query heads per kv head (EXACT) or a bound on them (g <= G, checked at run time).
template <int DPL, int G, bool EXACT>
__global__ void __launch_bounds__(att::T, 2) k_attn_part(AttnArgs p) {
    using namespace att;
    extern __shared__ __align__(16) float kv_sm[];
    __shared__ float pr[CHUNK][G + 1];          // scores (stride G + 1: the softmax reads a column)
    __shared__ __align__(16) float pw[CHUNK][G < 4 ? 4 : G];  // exp(s - m), per row (16-byte rows)
    __shared__ float mh[G], lh[G];
    __shared__ __align__(16) float sc[G < 4 ? 4 : G];  // rescale of the earlier chunks' sums, per head
    __shared__ __align__(8) uint64_t bar[2];  // K rows (and the query heads), V rows
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
    constexpr int hd = 32 * DPL;
    const int g = EXACT ? G : p.n_head / p.n_kv;
    float* Ks = kv_sm;
    float* Vs = kv_sm + CHUNK * hd;
    float* Qs = kv_sm + 2 * CHUNK * hd;

    pdl_wait();  // (the prep kernel's query heads and new cache row)
    const int L = p.len[seq];
    if (L < 0 || L >= p.cap) return;  // (recorded by k_attn_prep)
    const int p0 = r * p.rpc;
    if (p0 > L) return;
    const int pend = min(p0 + p.rpc, L + 1);
    const int64_t kvrow0 = ((int64_t)seq * p.n_kv + kvh) * p.cap;  // first cache row of this kv head
    auto issue_k = [&](int c, bool with_q) {  // (thread 0) chunk c's K rows, and the query heads
        const int m = min(CHUNK, pend - c);
        const uint32_t bytes = (uint32_t)(m * hd * 4), qb = with_q ? (uint32_t)(g * hd * 4) : 0u;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // (earlier reads of the buffer first)
        mbar_expect_tx(&bar[0], bytes + qb);
        bulk_g2s(Ks, p.k_cache + (kvrow0 + c) * hd, bytes, &bar[0]);
        if (with_q) bulk_g2s(Qs, p.qn + ((int64_t)seq * p.n_head + kvh * g) * hd, qb, &bar[0]);
    };
    auto issue_v = [&](int c) {  // (thread 0) chunk c's V rows
        const uint32_t bytes = (uint32_t)(min(CHUNK, pend - c) * hd * 4);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(&bar[1], bytes);
        bulk_g2s(Vs, p.v_cache + (kvrow0 + c) * hd, bytes, &bar[1]);
    };
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
        issue_k(p0, true);
        issue_v(p0);
    }
    if (tid < G) {
        mh[tid] = -INFINITY;  // running max and exp total of each query head over the CTA's chunks
        lh[tid] = 0.f;
    }
    constexpr int G4 = G < 4 ? 4 : G;
    // the weighted sum of V: thread t takes DPT values d0 .. of the rows of its row group (all
    // threads busy at every head dim; the groups' sums are added once, after the last chunk)
    constexpr int DPT = DPL == 8 ? 2 : 1;      // values per thread
    constexpr int TPR = 32 * DPL / DPT;        // threads per row group (hd / DPT)
    constexpr int NRG = T / TPR;               // row groups: 2 (hd 256, 128) or 4 (hd 64)
    constexpr int RG = CHUNK / NRG;            // rows per group
    const int rg = tid / TPR, d0 = (tid % TPR) * DPT;
    float acc[G4][DPT];  // the running weighted sums of its values, per query head
#pragma unroll
    for (int hh = 0; hh < G4; ++hh)
#pragma unroll
        for (int k = 0; k < DPT; ++k) acc[hh][k] = 0.f;
    __syncthreads();  // (the barrier's init is visible to every waiting thread)

    // chunk i: wait for its K rows, score them, start chunk i+1's K rows; softmax; wait for its V
    // rows, weight them, start chunk i+1's V rows. A bounded wait that gives up in any thread makes
    // the whole CTA wait once more for what it has in flight and leave.
    uint32_t ph = 0;
    for (int c0 = p0; c0 < pend; c0 += CHUNK, ph ^= 1) {
        const int n = min(CHUNK, pend - c0);
        const int c1 = c0 + CHUNK;
        if (!__syncthreads_and(mbar_wait(&bar[0], ph, p.err))) {
            mbar_wait(&bar[0], ph, p.err);
            mbar_wait(&bar[1], ph, p.err);
            return;
        }

        // scores: warp rows 4 warp .. + 3 of the chunk, HG query heads per pass; 4 x 4 (head, row)
        // sums per lane, finished by a reduce-scatter over 16 lanes and one exchange across the halves
        constexpr int RW = CHUNK / W;  // rows per warp (4)
#pragma unroll
        for (int hg = 0; hg < G; hg += HG) {
            if (!EXACT && hg >= g) break;
            float q[HG][DPL];
#pragma unroll
            for (int hh = 0; hh < HG; ++hh) {
                if (hg + hh < g) {
                    load_row<DPL>(Qs + (hg + hh) * hd, lane, q[hh]);
                } else {
#pragma unroll
                    for (int j = 0; j < DPL; ++j) q[hh][j] = 0.f;
                }
            }
            float v[HG * RW];
#pragma unroll
            for (int jp = 0; jp < RW; ++jp) {
                float k[DPL];
                load_row<DPL>(Ks + (warp * RW + jp) * hd, lane, k);  // (rows past n hold stale data: masked)
#pragma unroll
                for (int hh = 0; hh < HG; ++hh) {
                    float s = 0.f;
#pragma unroll
                    for (int j = 0; j < DPL; ++j) s += q[hh][j] * k[j];
                    v[hh * RW + jp] = s;
                }
            }
            rs_level<16>(v, lane);
            rs_level<8>(v, lane);
            rs_level<4>(v, lane);
            rs_level<2>(v, lane);
            const float sum = v[0] + __shfl_xor_sync(0xffffffffu, v[0], 16);
            const int hh = (lane & 15) >> 2, jp = lane & 3;  // the (head, row) whose sum this lane holds
            const int row = warp * RW + jp;
            if (lane < 16 && hg + hh < g) pr[row][hg + hh] = row < n ? sum * p.scale : -INFINITY;
        }
        __syncthreads();
        if (tid == 0 && c1 < pend) issue_k(c1, false);  // (the K buffer is free: scores are done)

        // the softmax so far per query head (lane = row): the new running max, the chunk's exp
        // weights against it, the earlier sums' rescale factor
        for (int hh = warp; hh < g; hh += W) {
            const float a = pr[lane][hh];
            const float m_old = mh[hh];
            const float m = fmaxf(m_old, att_warp_max(a));
            const float ea = expf(a - m);
            const float l = att_warp_sum(ea);
            pw[lane][hh] = ea;
            __syncwarp();
            if (lane == 0) {
                const float so = expf(m_old - m);  // (0 for the first chunk)
                sc[hh] = so;
                mh[hh] = m;
                lh[hh] = lh[hh] * so + l;
            }
        }
        __syncthreads();

        // exp-weighted sum of the V rows: thread d holds value d for every query head
        if (!__syncthreads_and(mbar_wait(&bar[1], ph, p.err))) {
            mbar_wait(&bar[1], ph, p.err);
            if (c1 < pend) mbar_wait(&bar[0], ph ^ 1, p.err);
            return;
        }
        {
            const float4* s4 = reinterpret_cast<const float4*>(sc);
#pragma unroll
            for (int q4 = 0; q4 < G4 / 4; ++q4) {
                const float4 f = s4[q4];
#pragma unroll
                for (int k = 0; k < DPT; ++k) {
                    acc[4 * q4 + 0][k] *= f.x;
                    acc[4 * q4 + 1][k] *= f.y;
                    acc[4 * q4 + 2][k] *= f.z;
                    acc[4 * q4 + 3][k] *= f.w;
                }
            }
            const int row1 = min(n, (rg + 1) * RG);
            for (int row = rg * RG; row < row1; ++row) {
                float vv[DPT];
                if (DPT == 2) {
                    const float2 t2 = *reinterpret_cast<const float2*>(Vs + row * hd + d0);
                    vv[0] = t2.x;
                    vv[DPT - 1] = t2.y;
                } else {
                    vv[0] = Vs[row * hd + d0];
                }
                const float4* w4 = reinterpret_cast<const float4*>(pw[row]);
#pragma unroll
                for (int q4 = 0; q4 < G4 / 4; ++q4) {  // (columns past g hold stale values: never stored)
                    const float4 w = w4[q4];
#pragma unroll
                    for (int k = 0; k < DPT; ++k) {
                        acc[4 * q4 + 0][k] += w.x * vv[k];
                        acc[4 * q4 + 1][k] += w.y * vv[k];
                        acc[4 * q4 + 2][k] += w.z * vv[k];
                        acc[4 * q4 + 3][k] += w.w * vv[k];
                    }
                }
            }
        }
        __syncthreads();  // (the V buffer, pw and sc are reused by the next chunk)
        if (tid == 0 && c1 < pend) issue_v(c1);
    }

    // the row groups' sums, added in group order (the K and V buffers, contiguous, are free: no copy
    // is in flight)
    static_assert((NRG - 1) * G <= 2 * CHUNK, "row-group sums fit in the K and V buffers");
    float* red = Ks;
    if (rg > 0) {
#pragma unroll
        for (int hh = 0; hh < G; ++hh)
#pragma unroll
            for (int k = 0; k < DPT; ++k) red[((rg - 1) * G + hh) * hd + d0 + k] = acc[hh][k];
    }
    __syncthreads();
    const int64_t part_i = ((int64_t)seq * p.n_kv + kvh) * p.n_split + r;
    if (rg == 0) {
        float* part = p.part + part_i * g * hd;
#pragma unroll
        for (int hh = 0; hh < G; ++hh) {
            if (!EXACT && hh >= g) break;
#pragma unroll
            for (int k = 0; k < DPT; ++k) {
                float v = acc[hh][k];
                for (int r2 = 1; r2 < NRG; ++r2) v += red[((r2 - 1) * G + hh) * hd + d0 + k];
                part[hh * hd + d0 + k] = v;
            }
        }
    }
    if (tid < g) {
        p.ml[(part_i * g + tid) * 2] = mh[tid];
        p.ml[(part_i * g + tid) * 2 + 1] = lh[tid];
    }
}

// Query head blockIdx.x of sequence blockIdx.y: the chunks merged (warp w of CW takes chunks w,
// w + CW, ..; the warps' sums then added in warp order), each rescaled by exp(m_chunk - M), divided by the
// softmax total, times sigmoid(gate).
template <int DPL, int CW>
__global__ void __launch_bounds__(CW * 32) k_attn_combine(AttnArgs p) {
    using namespace att;
    constexpr int CT = CW * 32;
    __shared__ float red[CW][MAX_HD + 1];
    __shared__ float dred[CW], mx[CW];
    const int h = blockIdx.x, seq = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int hd = 32 * DPL;
    pdl_wait();
    // (the gate value of this thread's output, requested with the length)
    const float gt = tid < hd ? p.qg[((int64_t)seq * p.n_head + h) * 2 * hd + hd + tid] : 0.f;
    const int L = p.len[seq];
    if (L < 0 || L >= p.cap) return;  // (recorded by k_attn_prep)
    const int g = p.n_head / p.n_kv, kvh = h / g, hh = h % g;
    const int n_act = L / p.rpc + 1;
    const int64_t c0 = ((int64_t)seq * p.n_kv + kvh) * p.n_split;  // first chunk of this kv head
    const float* ml = p.ml + (c0 * g + hh) * 2;                     // chunk r at ml[2 g r]
    const float* sums = p.part + (c0 * g + hh) * hd;                // chunk r at sums[g hd r]
    float m = -INFINITY;
    for (int r = tid; r < n_act; r += CT) m = fmaxf(m, ml[(int64_t)r * 2 * g]);
    m = att_warp_max(m);
    if (lane == 0) mx[warp] = m;
    __syncthreads();
    float M = mx[0];
#pragma unroll
    for (int w = 1; w < CW; ++w) M = fmaxf(M, mx[w]);
    float num[DPL], den = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) num[j] = 0.f;
#pragma unroll 4
    for (int r = warp; r < n_act; r += CW) {  // (unrolled: several chunks' loads in flight)
        const float e = expf(ml[(int64_t)r * 2 * g] - M);
        den += e * ml[(int64_t)r * 2 * g + 1];
        float v[DPL];
        load_row<DPL>(sums + (int64_t)r * g * hd, lane, v);
#pragma unroll
        for (int j = 0; j < DPL; ++j) num[j] += e * v[j];
    }
#pragma unroll
    for (int j = 0; j < DPL; ++j) red[warp][dim_of<DPL>(lane, j)] = num[j];
    if (lane == 0) dred[warp] = den;
    __syncthreads();
    if (tid < hd) {
        float o = 0.f, D = 0.f;
#pragma unroll
        for (int w = 0; w < CW; ++w) {
            o += red[w][tid];
            D += dred[w];
        }
        p.out[((int64_t)seq * p.n_head + h) * hd + tid] = (o / D) * (1.0f / (1.0f + expf(-gt)));
    }
}

template <int DPL, int G, bool EXACT>
static cudaError_t launch_part(dim3 grid, size_t smem, cudaStream_t st, const AttnArgs& a) {
    static bool attr = false;  // (the dynamic shared memory limit, once per instantiation)
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(k_attn_part<DPL, G, EXACT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (2 * att::CHUNK + G) * 32 * DPL * (int)sizeof(float));
        if (e != cudaSuccess) return e;
        attr = true;
    }
    return launch_pdl(k_attn_part<DPL, G, EXACT>, grid, dim3(att::T), smem, st, a);
}

template <int DPL>
static cudaError_t launch_attn(dim3 grid, size_t smem, cudaStream_t st, const AttnArgs& a) {
    cudaError_t e = launch_pdl(k_attn_prep, dim3(a.n_head + a.n_kv, grid.z), dim3(32), 0, st, a);
    if (e != cudaSuccess) return e;
    switch (a.n_head / a.n_kv) {  // the query heads per kv head: exact variants, else a bound of 16
        case 1: e = launch_part<DPL, 1, true>(grid, smem, st, a); break;
        case 2: e = launch_part<DPL, 2, true>(grid, smem, st, a); break;
        case 4: e = launch_part<DPL, 4, true>(grid, smem, st, a); break;
        case 8: e = launch_part<DPL, 8, true>(grid, smem, st, a); break;
        case 16: e = launch_part<DPL, 16, true>(grid, smem, st, a); break;
        default: e = launch_part<DPL, 16, false>(grid, smem, st, a); break;
    }
    if (e != cudaSuccess) return e;
    // the merge: 32 warps when a head has many chunk results (their loads in flight together), else 8
    if (a.n_split >= 64) return launch_pdl(k_attn_combine<DPL, 32>, dim3(a.n_head, grid.z), dim3(32 * 32), 0, st, a);
    return launch_pdl(k_attn_combine<DPL, 8>, dim3(a.n_head, grid.z), dim3(8 * 32), 0, st, a);
}

}  // namespace cwx

using namespace cwx;

extern "C" int cwx_attn_word(cwx_ctx* c, const cwx_attn_layer* L, int32_t n_seq, int32_t cap, const float* qg,
                             const float* k_new, const float* v_new, float* k_cache, float* v_cache,
                             const int32_t* len, const int32_t* pos, float* out, void* stream) {
    if (!L) return fail(CWX_EINVAL, "cwx_attn_word: null layer");
    if (L->n_head < 1 || L->n_kv < 1 || L->n_head % L->n_kv != 0 || L->n_kv > 65535)
        return fail(CWX_EINVAL, "cwx_attn_word: %d query heads over %d kv heads", L->n_head, L->n_kv);
    if (L->n_head / L->n_kv > att::MAX_G)
        return fail(CWX_EUNSUPPORTED, "cwx_attn_word: %d query heads per kv head (at most %d)", L->n_head / L->n_kv,
                    att::MAX_G);
    if (L->hd != 64 && L->hd != 128 && L->hd != 256)
        return fail(CWX_EUNSUPPORTED, "cwx_attn_word: head dim %d (64, 128 or 256)", L->hd);
    if (L->rot < 0 || L->rot > L->hd || L->rot % 2 != 0)
        return fail(CWX_EINVAL, "cwx_attn_word: rotary dims %d for head dim %d", L->rot, L->hd);
    if (!(L->eps >= 0.f) || !(L->freq_base > 0.0))
        return fail(CWX_EINVAL, "cwx_attn_word: eps %g, freq_base %g", (double)L->eps, L->freq_base);
    if (n_seq < 0 || n_seq > 65535 || cap < 1) return fail(CWX_EINVAL, "cwx_attn_word: n_seq %d, cap %d", n_seq, cap);
    if (!L->q_norm_w || !L->k_norm_w) return fail(CWX_EINVAL, "cwx_attn_word: null norm weights");
    if (!c) return fail(CWX_EINVAL, "cwx_attn_word: null context");
    if (n_seq == 0) return CWX_OK;
    if (!qg || !k_new || !v_new || !k_cache || !v_cache || !len || !pos || !out)
        return fail(CWX_EINVAL, "cwx_attn_word: null argument");
    if ((((uintptr_t)k_cache | (uintptr_t)v_cache) & 15) != 0)
        return fail(CWX_EINVAL, "cwx_attn_word: the caches must be 16-byte aligned");
    CWX_CUDA(cudaSetDevice(c->device));
    const cudaStream_t st = (cudaStream_t)stream;
    const int g = L->n_head / L->n_kv;
    // rows per chunk CTA: 32, or more when the grid would otherwise run more than 4 waves of 2
    // CTAs per SM (fewer partial results to write and merge), at most 256
    const int64_t chunks = (int64_t)n_seq * L->n_kv * ((cap + att::CHUNK - 1) / att::CHUNK);
    int nch = (int)(chunks / (8 * (int64_t)c->sm_count));
    nch = nch < 1 ? 1 : nch > 8 ? 8 : nch;
    const int rpc = att::CHUNK * nch;
    const int n_split = (cap + rpc - 1) / rpc;
    const size_t f4 = sizeof(float);
    const size_t qn_b = (((size_t)n_seq * L->n_head * L->hd * f4) + 255) & ~(size_t)255;
    const size_t part_b = (((size_t)n_seq * L->n_kv * n_split * g * L->hd * f4) + 255) & ~(size_t)255;
    const size_t ml_b = (size_t)n_seq * L->n_kv * n_split * g * 2 * f4;
    int rc = ensure_ws(c, qn_b + part_b + ml_b, st);
    if (rc) return rc;
    float* ws = reinterpret_cast<float*>(c->ws);
    AttnArgs a{L->n_head, L->n_kv, L->hd, L->rot, n_split, cap, rpc, L->eps, (float)(1.0 / sqrt((double)L->hd)),
               L->freq_base, qg, k_new, v_new, k_cache, v_cache, len, pos, L->q_norm_w, L->k_norm_w,
               ws, ws + qn_b / f4, ws + (qn_b + part_b) / f4, out, c->d_err};
    const dim3 grid(n_split, L->n_kv, n_seq);
    const size_t smem = (2 * att::CHUNK + g) * L->hd * f4;
    cudaError_t e;
    switch (L->hd) {
        case 64: e = launch_attn<2>(grid, smem, st, a); break;
        case 128: e = launch_attn<4>(grid, smem, st, a); break;
        default: e = launch_attn<8>(grid, smem, st, a); break;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cwx_attn_word launch");
    c->launches += 3;
    return CWX_OK;
}
