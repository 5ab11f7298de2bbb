// The Gated DeltaNet word step: the linear-attention mixer that runs before the MoE block in the
// Qwen3-Next / Qwen3.5 / Qwen3.6 layers, for one word of each of n_seq sequences.
//
// cwx_gdn_word follows the reference's one-kernel word step (crates/engine/src/attn_kernel.rs:24-143,
// dispatched by gdn_word, attn_kernel.rs:880-895, from LinearAttn::forward, model_next.rs:470-580):
// causal depthwise conv over the last `taps` inputs + SiLU, L2 norms of q and k, the query scale
// 1/sqrt(dk), the gates beta = sigmoid(b) and g = exp(softplus(alpha + dt_bias) * A), the delta
// rule on each value head's dk x dv memory (sk = k . S, d = (v - g sk) beta, S' = g S + k d^T,
// o = q . S'), then the output RMS norm times norm_w and the SiLU gate of z.
// cwx_delta_word is the delta rule alone on prepared q, k, v, beta and decay
// (crates/engine/src/delta_kernel.rs:20-50, the one-word case of delta_steps, model_next.rs:17-38).
//
// Layout of the work: one value head's memory is dk rows x dv columns of f32, read once and
// written once (HBM-bound at batch: 2 dk dv 4 bytes per head and word). Heads of up to 128 x 128
// (dv a multiple of 4) take k_gdn_head, one CTA per head and word. Other shapes take k_gdn_word:
// every column is independent in the delta rule, so a head is split over ceil(dv / 32) CTAs of 32
// columns (one per lane), each CTA's 8 warps taking dk / 8 rows of its columns; the only coupling
// across a head's columns, the output RMS norm, is summed over the head's CTAs through distributed
// shared memory (the CTAs of a head form one thread-block cluster, at most 8: dv <= 256).
#include <cooperative_groups.h>

#include "cwx_common.cuh"

namespace cwx {

namespace cg = cooperative_groups;

namespace gdn {
constexpr int W = 8;         // warps per CTA (each a band of rows)
constexpr int T = W * 32;    // threads per CTA
constexpr int COLS = 32;     // memory columns per CTA, one per lane
constexpr int MAX_SPLIT = 8;  // CTAs per head (a portable cluster)
}  // namespace gdn

struct GdnArgs {
    int n_k, n_v, dk, dv, taps, cycle;
    float eps;
    const float* qkv;
    const float* z;
    const float* ba;
    const float* conv_state;
    const float* conv_w;
    const float* dt_bias;
    const float* a;
    const float* norm_w;
    const float* s;
    float* o;
    float* s_out;
    float* conv_out;
};

__device__ __forceinline__ float gdn_silu(float x) { return x / (1.0f + expf(-x)); }

// Sum of v over the warp, in a fixed butterfly order (the same bits in every lane).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One word of one value head (blockIdx.y) of one sequence (blockIdx.z), columns 32 blockIdx.x ..
// of its memory; RPW rows per warp (dk <= 8 RPW).
template <int RPW>
__global__ void __launch_bounds__(gdn::T, RPW <= 16 ? 3 : RPW <= 32 ? 2 : 1) k_gdn_word(GdnArgs p) {
    using namespace gdn;
    __shared__ float q_sh[W * RPW], k_sh[W * RPW];
    __shared__ float part[W][COLS];
    __shared__ float v_sh[COLS];
    __shared__ float red[2 * W];
    __shared__ float ssq;  // this CTA's sum of o^2 over its columns (read by the head's other CTAs)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y, seq = blockIdx.z;
    const int dk = p.dk, dv = p.dv, taps = p.taps;
    const int channels = 2 * p.n_k * dk + p.n_v * dv;
    const int per_group = p.n_v / p.n_k;
    const int kh = p.cycle ? h % p.n_k : h / per_group;
    const int j = blockIdx.x * COLS + lane;
    const bool jok = j < dv;
    const int r0 = warp * RPW;
    const int64_t head = (int64_t)seq * p.n_v + h;
    const float* S = p.s + head * dk * dv;
    float* SO = p.s_out + head * dk * dv;
    const float* X = p.qkv + (int64_t)seq * channels;
    const float* CS = p.conv_state + (int64_t)seq * (taps - 1) * channels;
    float* CO = p.conv_out + (int64_t)seq * (taps - 1) * channels;
    const float* cw = p.conv_w;

    pdl_wait();
    // the memory column first: its loads are the long pole and depend on nothing else
    float col[RPW];
#pragma unroll
    for (int ii = 0; ii < RPW; ++ii) {
        const int i = r0 + ii;
        col[ii] = (jok && i < dk) ? S[(int64_t)i * dv + j] : 0.f;
    }

    // q and k of key head kh: conv over the window + SiLU; the head's first value head (and its
    // first CTA) moves their window one word on
    const bool qk_writer = blockIdx.x == 0 && (p.cycle ? h < p.n_k : h % per_group == 0);
    for (int i = tid; i < W * RPW; i += T) {
        float qv = 0.f, kv = 0.f;
        if (i < dk) {
            const int cq = kh * dk + i, ck = p.n_k * dk + kh * dk + i;
            float xq = 0.f, xk = 0.f;
            for (int t = 0; t + 1 < taps; ++t) {
                xq += cw[(int64_t)cq * taps + t] * CS[(int64_t)t * channels + cq];
                xk += cw[(int64_t)ck * taps + t] * CS[(int64_t)t * channels + ck];
            }
            xq += cw[(int64_t)cq * taps + taps - 1] * X[cq];
            xk += cw[(int64_t)ck * taps + taps - 1] * X[ck];
            qv = gdn_silu(xq);
            kv = gdn_silu(xk);
            if (qk_writer) {
                for (int t = 0; t + 2 < taps; ++t) {
                    CO[(int64_t)t * channels + cq] = CS[(int64_t)(t + 1) * channels + cq];
                    CO[(int64_t)t * channels + ck] = CS[(int64_t)(t + 1) * channels + ck];
                }
                CO[(int64_t)(taps - 2) * channels + cq] = X[cq];
                CO[(int64_t)(taps - 2) * channels + ck] = X[ck];
            }
        }
        q_sh[i] = qv;
        k_sh[i] = kv;
    }
    // v of this CTA's columns (each column's window is moved by the CTA that owns it)
    if (warp == 0 && jok) {
        const int cv = 2 * p.n_k * dk + h * dv + j;
        float xv = 0.f;
        for (int t = 0; t + 1 < taps; ++t) xv += cw[(int64_t)cv * taps + t] * CS[(int64_t)t * channels + cv];
        xv += cw[(int64_t)cv * taps + taps - 1] * X[cv];
        v_sh[lane] = gdn_silu(xv);
        for (int t = 0; t + 2 < taps; ++t) CO[(int64_t)t * channels + cv] = CS[(int64_t)(t + 1) * channels + cv];
        CO[(int64_t)(taps - 2) * channels + cv] = X[cv];
    }
    __syncthreads();

    // L2 norms of q and k (per-warp butterflies, then the warps in order)
    {
        float sq = 0.f, sk = 0.f;
        for (int i = tid; i < dk; i += T) {
            sq += q_sh[i] * q_sh[i];
            sk += k_sh[i] * k_sh[i];
        }
        sq = warp_sum(sq);
        sk = warp_sum(sk);
        if (lane == 0) {
            red[warp] = sq;
            red[W + warp] = sk;
        }
    }
    __syncthreads();
    float tq = 0.f, tk = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
        tq += red[w];
        tk += red[W + w];
    }
    const float qscale = 1.0f / (sqrtf(tq + p.eps) * sqrtf((float)dk));
    const float kscale = 1.0f / sqrtf(tk + p.eps);

    // gates of this head and word
    const float* ba = p.ba + (int64_t)seq * 2 * p.n_v;
    const float beta = 1.0f / (1.0f + expf(-ba[h]));
    const float g = expf(logf(expf(ba[p.n_v + h] + p.dt_bias[h]) + 1.0f) * p.a[h]);

    // sk = k . S (this warp's rows, then the warps in order)
    float skp = 0.f;
#pragma unroll
    for (int ii = 0; ii < RPW; ++ii) skp += (k_sh[r0 + ii] * kscale) * col[ii];
    part[warp][lane] = skp;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) tot += part[w][lane];
    const float d = (v_sh[lane] - tot * g) * beta;
    __syncthreads();  // (part is reused)

    // S' = g S + k d, o = q . S'
    float acc = 0.f;
#pragma unroll
    for (int ii = 0; ii < RPW; ++ii) {
        const int i = r0 + ii;
        const float ns = g * col[ii] + (k_sh[i] * kscale) * d;
        if (jok && i < dk) SO[(int64_t)i * dv + j] = ns;
        acc += (q_sh[i] * qscale) * ns;
    }
    part[warp][lane] = acc;
    __syncthreads();
    float o = 0.f;
    if (warp == 0) {
#pragma unroll
        for (int w = 0; w < W; ++w) o += part[w][lane];
        const float sq = warp_sum(jok ? o * o : 0.f);
        if (lane == 0) ssq = sq;
    }
    // the RMS norm over the head's dv columns: the CTAs of the head (one cluster) add their sums
    // in rank order, so every CTA gets the same total
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    float total = 0.f;
    if (warp == 0) {
        const int n = (int)cluster.num_blocks();
        for (int r = 0; r < n; ++r) total += *cluster.map_shared_rank(&ssq, r);
    }
    cluster.sync();  // no CTA leaves while another reads its sum
    if (warp == 0 && jok) {
        const float rms = 1.0f / sqrtf(total / (float)dv + p.eps);
        const int64_t oi = head * dv + j;
        const float x = o * rms * p.norm_w[j];
        p.o[oi] = x * gdn_silu(p.z[oi]);
    }
}

// The same word step with one CTA per head, for dk <= 128 and dv <= 128 with dv % 4 == 0 (the
// models' 128 x 128 heads): the head's memory (64 KB) comes into shared memory by one bulk copy
// started at the kernel's start, under the conv pass; lane l owns memory columns 4l .. 4l+3
// (16-byte shared-memory reads and global stores, a warp covers a 512-byte row), warp w rows
// 16w .. 16w+15; the conv of the head's q, k and v channels is one pass over all threads; the
// column sums and the RMS norm stay inside the CTA. Three CTAs per SM: 192 KB of memory in flight.
namespace gdnh {
constexpr int RPW = 16;                // rows per warp
constexpr int MAX_DK = gdn::W * RPW;   // 128
constexpr int MAX_DV = 128;
}  // namespace gdnh

__global__ void __launch_bounds__(gdn::T, 3) k_gdn_head(GdnArgs p) {
    using namespace gdn;
    using gdnh::RPW;
    extern __shared__ __align__(16) float st_sm[];  // the head's memory, dk x dv, by one bulk copy
    __shared__ __align__(8) uint64_t sbar;
    __shared__ float xc[2 * gdnh::MAX_DK + gdnh::MAX_DV];  // silu(conv): q | k | v of this head
    __shared__ __align__(16) float part[W][gdnh::MAX_DV];
    __shared__ __align__(16) float d_sh[gdnh::MAX_DV];
    __shared__ float red[2 * W];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.x, seq = blockIdx.y;
    const int dk = p.dk, dv = p.dv, taps = p.taps;
    const int channels = 2 * p.n_k * dk + p.n_v * dv;
    const int per_group = p.n_v / p.n_k;
    const int kh = p.cycle ? h % p.n_k : h / per_group;
    const int j0 = 4 * lane;
    const bool jok = j0 < dv;
    const int r0 = warp * RPW;
    const int64_t head = (int64_t)seq * p.n_v + h;
    const float* S = p.s + head * dk * dv;
    float* SO = p.s_out + head * dk * dv;
    const float* X = p.qkv + (int64_t)seq * channels;
    const float* CS = p.conv_state + (int64_t)seq * (taps - 1) * channels;
    float* CO = p.conv_out + (int64_t)seq * (taps - 1) * channels;

    pdl_wait();
    if (tid == 0) {  // the memory first: its copy is the long pole and runs under the conv pass
        mbar_init(&sbar, 1);
        fence_mbar_init();
        mbar_expect_tx(&sbar, (uint32_t)(dk * dv * 4));
        bulk_g2s(st_sm, S, (uint32_t)(dk * dv * 4), &sbar);
    }
    // the head's gate inputs and this thread's output-gate values, requested now so that they
    // arrive under the conv pass
    const float* ba = p.ba + (int64_t)seq * 2 * p.n_v;
    const float b_raw = ba[h], a_raw = ba[p.n_v + h], dtb = p.dt_bias[h], a_h = p.a[h];
    const float zv = tid < dv ? p.z[head * dv + tid] : 0.f, nw = tid < dv ? p.norm_w[tid] : 0.f;

    // conv + SiLU of q, k (key head kh) and v (this head) in one pass; the window moves one word
    // on (q, k by the key head's first value head)
    const bool qk_writer = p.cycle ? h < p.n_k : h % per_group == 0;
    // (at most 384 channels over 256 threads: a thread's two channels load together, then compute,
    // then move their windows, so that no load waits behind a store it might alias)
    const int nc = 2 * dk + dv;
    auto chan = [&](int c) {
        return c < dk ? kh * dk + c : c < 2 * dk ? p.n_k * dk + kh * dk + (c - dk) : 2 * p.n_k * dk + h * dv + (c - 2 * dk);
    };
    const int ca = tid, cb = tid + T;
    const bool ha = ca < nc, hb = cb < nc;
    const int cha = ha ? chan(ca) : 0, chb = hb ? chan(cb) : 0;
    const float* wa = p.conv_w + (int64_t)cha * taps;
    const float* wb = p.conv_w + (int64_t)chb * taps;
    float xa = 0.f, xb = 0.f;
    for (int t = 0; t + 1 < taps; ++t) {
        if (ha) xa += wa[t] * CS[t * channels + cha];
        if (hb) xb += wb[t] * CS[t * channels + chb];
    }
    const float na = ha ? X[cha] : 0.f, nb = hb ? X[chb] : 0.f;
    if (ha) {
        xa += wa[taps - 1] * na;
        xc[ca] = gdn_silu(xa);
    }
    if (hb) {
        xb += wb[taps - 1] * nb;
        xc[cb] = gdn_silu(xb);
    }
    if (ha && (ca >= 2 * dk || qk_writer)) {
        for (int t = 0; t + 2 < taps; ++t) CO[t * channels + cha] = CS[(t + 1) * channels + cha];
        CO[(taps - 2) * channels + cha] = na;
    }
    if (hb && (cb >= 2 * dk || qk_writer)) {
        for (int t = 0; t + 2 < taps; ++t) CO[t * channels + chb] = CS[(t + 1) * channels + chb];
        CO[(taps - 2) * channels + chb] = nb;
    }
    __syncthreads();
    {
        float sq = 0.f, sk = 0.f;
        for (int i = tid; i < dk; i += T) {
            sq += xc[i] * xc[i];
            sk += xc[dk + i] * xc[dk + i];
        }
        sq = warp_sum(sq);
        sk = warp_sum(sk);
        if (lane == 0) {
            red[warp] = sq;
            red[W + warp] = sk;
        }
    }
    __syncthreads();
    float tq = 0.f, tk = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
        tq += red[w];
        tk += red[W + w];
    }
    const float qscale = 1.0f / (sqrtf(tq + p.eps) * sqrtf((float)dk));
    const float kscale = 1.0f / sqrtf(tk + p.eps);
    const float beta = 1.0f / (1.0f + expf(-b_raw));
    const float g = expf(logf(expf(a_raw + dtb) + 1.0f) * a_h);

    // sk = k . S over this warp's rows, then over the warps in order (a copy that did not arrive
    // in time, in any thread: the CTA waits once more, bounded, writes NaN for the head's read-out,
    // so that the failure shows, and leaves; this entry point has no context to record it in)
    if (!__syncthreads_and(mbar_wait(&sbar, 0, nullptr))) {
        mbar_wait(&sbar, 0, nullptr);
        if (tid < dv) p.o[head * dv + tid] = __int_as_float(0x7fc00000);
        return;
    }
    auto col = [&](int ii) {  // this thread's 4 columns of row r0 + ii
        const int i = r0 + ii;
        return (jok && i < dk) ? *reinterpret_cast<const float4*>(st_sm + i * dv + j0) : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    float4 sp = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int ii = 0; ii < RPW; ++ii) {
        const float kv = (r0 + ii < dk ? xc[dk + r0 + ii] : 0.f) * kscale;
        const float4 c = col(ii);
        sp.x += kv * c.x;
        sp.y += kv * c.y;
        sp.z += kv * c.z;
        sp.w += kv * c.w;
    }
    if (jok) *reinterpret_cast<float4*>(&part[warp][j0]) = sp;
    __syncthreads();
    if (tid < dv) {
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < W; ++w) tot += part[w][tid];
        d_sh[tid] = (xc[2 * dk + tid] - tot * g) * beta;
    }
    __syncthreads();
    const float4 d = jok ? *reinterpret_cast<const float4*>(&d_sh[j0]) : make_float4(0.f, 0.f, 0.f, 0.f);

    // S' = g S + k d, o = q . S'
    float4 ac = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int ii = 0; ii < RPW; ++ii) {
        const int i = r0 + ii;
        const bool iok = i < dk;
        const float kv = (iok ? xc[dk + i] : 0.f) * kscale;
        const float qv = (iok ? xc[i] : 0.f) * qscale;
        const float4 c = col(ii);
        float4 ns;
        ns.x = g * c.x + kv * d.x;
        ns.y = g * c.y + kv * d.y;
        ns.z = g * c.z + kv * d.z;
        ns.w = g * c.w + kv * d.w;
        if (jok && iok) *reinterpret_cast<float4*>(SO + i * dv + j0) = ns;
        ac.x += qv * ns.x;
        ac.y += qv * ns.y;
        ac.z += qv * ns.z;
        ac.w += qv * ns.w;
    }
    if (jok) *reinterpret_cast<float4*>(&part[warp][j0]) = ac;  // (the sums of sk were read before d_sh's barrier)
    __syncthreads();
    float o = 0.f;
    if (tid < dv) {
#pragma unroll
        for (int w = 0; w < W; ++w) o += part[w][tid];
    }
    // RMS norm over the head's dv values (dv <= 128: warps 0-3)
    const float sq = warp_sum(tid < dv ? o * o : 0.f);
    if (lane == 0 && warp < 4) red[warp] = sq;
    __syncthreads();
    if (tid < dv) {
        const float total = ((red[0] + red[1]) + red[2]) + red[3];
        const float rms = 1.0f / sqrtf(total / (float)dv + p.eps);
        const float x = o * rms * nw;
        p.o[head * dv + tid] = x * gdn_silu(zv);
    }
}

// The delta rule for one word of prepared inputs, the reference's packed layout: qk (heads, 2 dk)
// q then k; vbd (heads, dv + 2) v, beta, decay; s (heads, dk, dv); out (heads, dk dv + dv) the new
// memory then the read-out.
template <int RPW>
__global__ void __launch_bounds__(gdn::T) k_delta_word(const float* qk, const float* vbd, const float* s, float* out,
                                                       int dk, int dv) {
    using namespace gdn;
    __shared__ float q_sh[W * RPW], k_sh[W * RPW];
    __shared__ float part[W][COLS];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t h = blockIdx.y;
    const int j = blockIdx.x * COLS + lane;
    const bool jok = j < dv;
    const int r0 = warp * RPW;
    const float* q = qk + h * 2 * dk;
    const float* k = q + dk;
    const float* v = vbd + h * (dv + 2);
    const float* S = s + h * dk * dv;
    float* SO = out + h * ((int64_t)dk * dv + dv);
    pdl_wait();
    float col[RPW];
#pragma unroll
    for (int ii = 0; ii < RPW; ++ii) {
        const int i = r0 + ii;
        col[ii] = (jok && i < dk) ? S[(int64_t)i * dv + j] : 0.f;
    }
    for (int i = tid; i < W * RPW; i += T) {
        q_sh[i] = i < dk ? q[i] : 0.f;
        k_sh[i] = i < dk ? k[i] : 0.f;
    }
    const float beta = v[dv], g = v[dv + 1];
    const float vj = jok ? v[j] : 0.f;
    __syncthreads();
    float skp = 0.f;
#pragma unroll
    for (int ii = 0; ii < RPW; ++ii) skp += k_sh[r0 + ii] * col[ii];
    part[warp][lane] = skp;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < W; ++w) tot += part[w][lane];
    const float d = (vj - tot * g) * beta;
    __syncthreads();
    float acc = 0.f;
#pragma unroll
    for (int ii = 0; ii < RPW; ++ii) {
        const int i = r0 + ii;
        const float ns = g * col[ii] + k_sh[i] * d;
        if (jok && i < dk) SO[(int64_t)i * dv + j] = ns;
        acc += q_sh[i] * ns;
    }
    part[warp][lane] = acc;
    __syncthreads();
    if (warp == 0 && jok) {
        float o = 0.f;
#pragma unroll
        for (int w = 0; w < W; ++w) o += part[w][lane];
        SO[(int64_t)dk * dv + j] = o;
    }
}

template <int RPW>
static cudaError_t launch_gdn(const GdnArgs& p, int n_seq, cudaStream_t st) {
    const int nsplit = (p.dv + gdn::COLS - 1) / gdn::COLS;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nsplit, p.n_v, n_seq);
    cfg.blockDim = dim3(gdn::T);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = nsplit;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, k_gdn_word<RPW>, p);
}

static int rows_per_warp(int dk) { return dk <= 128 ? 16 : dk <= 256 ? 32 : 64; }

}  // namespace cwx

using namespace cwx;

extern "C" int cwx_gdn_word(const cwx_gdn_layer* L, int32_t n_seq, const float* qkv, const float* z, const float* ba,
                            const float* conv_state, const float* s, float* o, float* s_out, float* conv_out,
                            void* stream) {
    if (!L) return fail(CWX_EINVAL, "cwx_gdn_word: null layer");
    if (n_seq < 0 || n_seq > 65535) return fail(CWX_EINVAL, "cwx_gdn_word: n_seq %d outside 0 .. 65535", n_seq);
    if (L->n_k < 1 || L->n_v < 1 || L->n_v % L->n_k != 0 || L->n_v > 65535)
        return fail(CWX_EINVAL, "cwx_gdn_word: %d value heads over %d key heads", L->n_v, L->n_k);
    if (L->dk < 1 || L->dv < 1 || L->taps < 2)
        return fail(CWX_EINVAL, "cwx_gdn_word: dk %d, dv %d, taps %d", L->dk, L->dv, L->taps);
    if (L->dk > 512 || L->dv > gdn::COLS * gdn::MAX_SPLIT)
        return fail(CWX_EUNSUPPORTED, "cwx_gdn_word: dk %d > 512 or dv %d > 256", L->dk, L->dv);
    if (!(L->eps >= 0.f)) return fail(CWX_EINVAL, "cwx_gdn_word: eps %g", (double)L->eps);
    if (!L->conv_w || !L->dt_bias || !L->a || !L->norm_w)
        return fail(CWX_EINVAL, "cwx_gdn_word: null layer tensor");
    if (n_seq == 0) return CWX_OK;
    if (!qkv || !z || !ba || !conv_state || !s || !o || !s_out || !conv_out)
        return fail(CWX_EINVAL, "cwx_gdn_word: null argument");
    if (conv_out == conv_state) return fail(CWX_EINVAL, "cwx_gdn_word: conv_out must be a buffer of its own");
    GdnArgs p{L->n_k, L->n_v, L->dk, L->dv, L->taps, L->cycle ? 1 : 0, L->eps, qkv, z, ba, conv_state,
              L->conv_w, L->dt_bias, L->a, L->norm_w, s, o, s_out, conv_out};
    const cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    if (L->dk <= gdnh::MAX_DK && L->dv <= gdnh::MAX_DV && L->dv % 4 == 0 && ((uintptr_t)s & 15) == 0 &&
        ((uintptr_t)s_out & 15) == 0) {
        static bool attr = false;  // (the dynamic shared memory limit, once)
        if (!attr) {
            e = cudaFuncSetAttribute(k_gdn_head, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     gdnh::MAX_DK * gdnh::MAX_DV * (int)sizeof(float));
            if (e != cudaSuccess) return cuda_fail(e, "cwx_gdn_word attribute");
            attr = true;
        }
        e = launch_pdl(k_gdn_head, dim3(L->n_v, n_seq), dim3(gdn::T), (size_t)L->dk * L->dv * sizeof(float), st, p);
        return e == cudaSuccess ? CWX_OK : cuda_fail(e, "cwx_gdn_word launch");
    }
    switch (rows_per_warp(L->dk)) {
        case 16: e = launch_gdn<16>(p, n_seq, st); break;
        case 32: e = launch_gdn<32>(p, n_seq, st); break;
        default: e = launch_gdn<64>(p, n_seq, st); break;
    }
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "cwx_gdn_word launch");
}

extern "C" int cwx_delta_word(int32_t heads, int32_t dk, int32_t dv, const float* qk, const float* vbd, const float* s,
                              float* out, void* stream) {
    if (heads < 0 || heads > 65535 || dk < 1 || dv < 1)
        return fail(CWX_EINVAL, "cwx_delta_word: heads %d, dk %d, dv %d", heads, dk, dv);
    if (dk > 512) return fail(CWX_EUNSUPPORTED, "cwx_delta_word: dk %d > 512", dk);
    if (heads == 0) return CWX_OK;
    if (!qk || !vbd || !s || !out) return fail(CWX_EINVAL, "cwx_delta_word: null argument");
    if (out == s) return fail(CWX_EINVAL, "cwx_delta_word: out must be a buffer of its own");
    const dim3 grid((dv + gdn::COLS - 1) / gdn::COLS, heads);
    const cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    switch (rows_per_warp(dk)) {
        case 16: e = launch_pdl(k_delta_word<16>, grid, dim3(gdn::T), 0, st, qk, vbd, s, out, dk, dv); break;
        case 32: e = launch_pdl(k_delta_word<32>, grid, dim3(gdn::T), 0, st, qk, vbd, s, out, dk, dv); break;
        default: e = launch_pdl(k_delta_word<64>, grid, dim3(gdn::T), 0, st, qk, vbd, s, out, dk, dv); break;
    }
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "cwx_delta_word launch");
}
