// Router logits, route() and the expert piles.
//
//   router logits  candle-nn Linear (x . W^T + b), called at crates/engine/src/experts.rs:2577;
//                  gpt-oss bias crates/engine/src/model_gptoss.rs:168-175
//   route          crates/engine/src/experts.rs:2364-2372; fused Metal form
//                  crates/engine/src/fuse_kernel.rs:20-75 (same pick order: probability, then
//                  lowest index)
//   piles          cw_pile crates/engine/src/fuse_kernel.rs:180-202 and the CPU sort of group2
//                  experts.rs:2243-2267: picks grouped by expert, stable in pick order
//   shared gate    SharedExpert::forward model_next.rs:738 (sum_keepdim of x * gate_inp)
//
// Arithmetic chosen so the results are those of the candle CPU path bit for bit where that is
// defined: softmax sums in candle's x86 AVX order (vendor/candle-core/src/cpu/avx.rs:243-257,
// lanes reduced as in vec_reduce 51-66), exp correctly rounded to f32 (f64 exp rounded once;
// glibc's expf, which Rust's f32::exp calls, misrounds a few inputs next to a rounding midpoint),
// the pick order of a stable descending sort. Router logits
// accumulate exact f32 products in f64 and round once (a decode form for small batches and a
// tiled form with operand reuse for prefill-sized batches).
#include "cwx_common.cuh"
#include "kernels.cuh"
#include "products.cuh"

namespace cwx {

constexpr int SGATE_SMEM = 4096;  // hidden sizes up to this stage the shared gate's products

// Router logits on the FP64 tensor cores: block = 8 warps on a tile of 8 experts x 8 tokens,
// warp w taking the w-th eighth of K; each warp accumulates its slice with mma m8n8k4 f64 (the
// products of f32 inputs are exact in f64), the eight slices are added in warp order and the sum is
// rounded once to f32 (+ the bias).
__device__ __forceinline__ void dmma_8x8x4(double* c, double a, double b) {
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};"
                 : "+d"(c[0]), "+d"(c[1])
                 : "d"(a), "d"(b));
}

__global__ void __launch_bounds__(256) k_router(const float* __restrict__ x, const float* __restrict__ w,
                                                const float* __restrict__ bias, int T, int H, int E,
                                                float* __restrict__ logits) {
    __shared__ double red[8][64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e0 = blockIdx.x * 8, t0 = blockIdx.y * 8;
    {
        // the router rows of this block's experts are weights no kernel writes: the first token
        // tile asks L2 for them (one 128-byte line per request) before waiting for the kernel
        // before, so the loop below finds them there
        const char* wb = reinterpret_cast<const char*>(w + (int64_t)e0 * H);
        const int64_t bytes = blockIdx.y == 0 ? (int64_t)min(8, E - e0) * H * 4 : 0;
        for (int64_t o = (int64_t)threadIdx.x * 128; o < bytes; o += 256 * 128)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(wb + o));
    }
    pdl_wait();
    const int r = lane >> 2, kq = lane & 3;
    const int ks = (H + 7) / 8, k0 = warp * ks, k1 = min(H, k0 + ks);
    // A[r][k] = w[e0 + r][k], B[k][n] = x[t0 + n][k]: each lane reads row r at k = 4j + kq
    const bool ea = e0 + r < E, tb = t0 + r < T;
    const float* wr = w + (int64_t)(ea ? e0 + r : 0) * H;
    const float* xr = x + (int64_t)(tb ? t0 + r : 0) * H;
    double c[2] = {0.0, 0.0};
    int k = k0;
    // 16-column chunks with the reduction index permuted inside a chunk (the same way for both
    // operands): step i of chunk c takes columns k0 + 16c + 4q + i (q = 0..3), so lane (r, q)
    // holds its four steps' values as one float4 of each operand; PF chunks are in flight ahead
    // of the multiplies
    if ((k0 & 3) == 0 && (H & 3) == 0 && (((uintptr_t)w | (uintptr_t)x) & 15) == 0) {
        constexpr int PF = 4;
        const int nch = (k1 - k0) >> 4;
        const float4* w4 = reinterpret_cast<const float4*>(wr + k0) + kq;
        const float4* x4 = reinterpret_cast<const float4*>(xr + k0) + kq;
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        float4 aw[PF], bx[PF];
#pragma unroll
        for (int j = 0; j < PF; ++j) {
            aw[j] = j < nch && ea ? __ldg(w4 + 4 * j) : z;
            bx[j] = j < nch && tb ? __ldg(x4 + 4 * j) : z;
        }
        for (int c0 = 0; c0 < nch; c0 += PF) {
#pragma unroll
            for (int j = 0; j < PF; ++j) {
                const int ch = c0 + j;
                if (ch < nch) {
                    const float4 a = aw[j], b = bx[j];
                    if (ch + PF < nch) {
                        aw[j] = ea ? __ldg(w4 + 4 * (ch + PF)) : z;
                        bx[j] = tb ? __ldg(x4 + 4 * (ch + PF)) : z;
                    }
                    dmma_8x8x4(c, (double)a.x, (double)b.x);
                    dmma_8x8x4(c, (double)a.y, (double)b.y);
                    dmma_8x8x4(c, (double)a.z, (double)b.z);
                    dmma_8x8x4(c, (double)a.w, (double)b.w);
                }
            }
        }
        k = k0 + 16 * nch;
    }
    for (; k < k1; k += 4) {
        const bool in = k + kq < k1;
        const float av = ea && in ? __ldg(wr + k + kq) : 0.f, bv = tb && in ? __ldg(xr + k + kq) : 0.f;
        dmma_8x8x4(c, (double)av, (double)bv);
    }
    // C[r][2kq], C[r][2kq+1]
    red[warp][r * 8 + 2 * kq] = c[0];
    red[warp][r * 8 + 2 * kq + 1] = c[1];
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int idx = lane * 2 + h, er = idx >> 3, tn = idx & 7;
            double v = red[0][idx];
            for (int q = 1; q < 8; ++q) v += red[q][idx];
            const int e = e0 + er, t = t0 + tn;
            if (e < E && t < T) {
                float l = (float)v;
                if (bias) l = __fadd_rn(l, bias[e]);
                logits[(int64_t)t * E + e] = l;
            }
        }
    }
}

// One block (8 warps) per token: softmax over E (<= 1024, up to 4 experts per thread), K picks
// (<= 16) best first with ties to the lowest id, weights renormalised over the picks when norm.
// The softmax denominator keeps candle's AVX order: lane L of one warp sums elements 32i + L over
// the whole 32-element steps in order, the lanes are reduced in the AVX tree, and a tail is added
// element by element. Top-k: each warp selects the best K of its experts, warp 0 merges the 8
// candidate lists. Optionally (warp 1, meanwhile) the shared-expert gate
// sigmoid(sum_keepdim(x * gate_inp)) in the same AVX summation order.
__global__ void __launch_bounds__(256) k_route(const float* __restrict__ logits, int T, int E, int K, int norm,
                                               uint32_t* __restrict__ ids, float* __restrict__ wout,
                                               const float* __restrict__ x, const float* __restrict__ g_inp,
                                               int H, float* __restrict__ sgate) {
    pdl_wait();
    __shared__ float pv[1024];
    __shared__ float wred[8];
    __shared__ float s_sum;
    __shared__ float cv[8][16];
    __shared__ int ci[8][16];
    __shared__ float sp[SGATE_SMEM];  // x * gate_inp for the shared gate, staged by every thread
    const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool sp_smem = sgate && H <= SGATE_SMEM;
    if (sp_smem)
        for (int h = tid; h < H; h += 256) sp[h] = __fmul_rn(__ldg(x + (int64_t)t * H + h), __ldg(g_inp + h));
    float v[4];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int e = tid + 256 * j;
        v[j] = e < E ? logits[(int64_t)t * E + e] : -INFINITY;
        if (e < E) mx = fmaxf(mx, v[j]);
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) wred[warp] = mx;
    __syncthreads();
    mx = wred[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, wred[w]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int e = tid + 256 * j;
        if (e < E) {
            v[j] = exp_cr(__fsub_rn(v[j], mx));
            pv[e] = v[j];
        }
    }
    __syncthreads();
    if (warp == 0) {
        const int whole = E / 32;  // whole 32-element steps
        float acc = 0.f;
        for (int i = 0; i < whole; ++i) acc = __fadd_rn(acc, pv[32 * i + lane]);
        float sum = avx_lane_tree(acc);
        for (int j = whole * 32; j < E; ++j) sum = __fadd_rn(sum, pv[j]);  // tail in order
        if (lane == 0) s_sum = sum;
    }
    __syncthreads();
    const float ssum = s_sum;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int e = tid + 256 * j;
        v[j] = e < E ? __fdiv_rn(v[j], ssum) : -1.0f;  // probabilities; -1 marks padding
    }
    // this warp's best K of its experts (ascending id within a thread: the first wins ties)
    for (int r = 0; r < K; ++r) {
        float bv = -2.0f;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (v[j] > bv) {
                bv = v[j];
                bi = tid + 256 * j;
            }
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            cv[warp][r] = bv;
            ci[warp][r] = bi;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (tid + 256 * j == bi) v[j] = -3.0f;  // taken
    }
    __syncthreads();
    if (warp == 0) {
        // merge: lane l holds candidates l, l + 32, ... of the 8 x K list
        const int nc = 8 * K;
        float mv[4];
        int mi[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c = lane + 32 * j;
            mv[j] = c < nc ? cv[c / K][c % K] : -2.0f;
            mi[j] = c < nc ? ci[c / K][c % K] : 0x7fffffff;
        }
        float tot = 0.f;
        for (int r = 0; r < K; ++r) {
            float bv = -2.0f;
            int bi = 0x7fffffff, bj = -1;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (mv[j] > bv || (mv[j] == bv && mi[j] < bi)) {
                    bv = mv[j];
                    bi = mi[j];
                    bj = j;
                }
            int owner = lane;
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                const int oo = __shfl_xor_sync(0xffffffffu, owner, o);
                if (ov > bv || (ov == bv && oi < bi)) {
                    bv = ov;
                    bi = oi;
                    owner = oo;
                }
            }
            if (owner == lane && bj >= 0) mv[bj] = -3.0f;  // taken
            if (bi >= E) bi = E - 1;  // only when every candidate is NaN: keep ids in range
            if (lane == 0) {
                ids[(int64_t)t * K + r] = (uint32_t)bi;
                wout[(int64_t)t * K + r] = bv;
                if (norm) tot = __fadd_rn(tot, bv);
            }
        }
        if (lane == 0 && norm)
            for (int r = 0; r < K; ++r) wout[(int64_t)t * K + r] = __fdiv_rn(wout[(int64_t)t * K + r], tot);
    } else if (warp == 1 && sp_smem) {
        // candle's sum_keepdim order over the staged products (staged before the first barrier)
        const int wholeh = H / 32;
        float a = 0.f;
        for (int i = 0; i < wholeh; ++i) a = __fadd_rn(a, sp[32 * i + lane]);
        float sum = avx_lane_tree(a);
        for (int j = wholeh * 32; j < H; ++j) sum = __fadd_rn(sum, sp[j]);
        if (lane == 0) sgate[t] = __fdiv_rn(1.0f, __fadd_rn(exp_cr(-sum), 1.0f));
    } else if (warp == 1 && sgate) {
        const float* xr = x + (int64_t)t * H;
        const int wholeh = H / 32;
        float a = 0.f;
        // loads issued 16 at a time ahead of the in-order sum (the sum's order is fixed)
        for (int i0 = 0; i0 < wholeh; i0 += 16) {
            float pr[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                pr[j] = i0 + j < wholeh ? __fmul_rn(__ldg(xr + 32 * (i0 + j) + lane), __ldg(g_inp + 32 * (i0 + j) + lane)) : 0.f;
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (i0 + j < wholeh) a = __fadd_rn(a, pr[j]);
        }
        float sum = avx_lane_tree(a);
        for (int j = wholeh * 32; j < H; ++j) sum = __fadd_rn(sum, __fmul_rn(xr[j], g_inp[j]));
        if (lane == 0) sgate[t] = __fdiv_rn(1.0f, __fadd_rn(exp_cr(-sum), 1.0f));
    }
}

// ---------------------------------------------------------------- piles
constexpr int PERM_TILE = 1024;

// n_dev (optional): the picks are the first *n_dev of the n slots (a count another kernel wrote)
__device__ __forceinline__ int64_t picks_of(int64_t n, const int32_t* n_dev) {
    if (!n_dev) return n;
    const int64_t d = *n_dev;
    return d < n ? (d > 0 ? d : 0) : n;
}

__global__ void __launch_bounds__(1024) k_perm_count(const uint32_t* __restrict__ ids, int64_t n, int E,
                                                     uint32_t* __restrict__ tile_counts, int* err,
                                                     const int32_t* n_dev) {
    pdl_wait();
    n = picks_of(n, n_dev);
    extern __shared__ uint32_t hist[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    int64_t i = (int64_t)blockIdx.x * PERM_TILE + threadIdx.x;
    if (i < n) {
        uint32_t id = ids[i];
        if (id < (uint32_t)E) atomicAdd(&hist[id], 1u);
        else dev_error(err, DE_BAD_ID);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) tile_counts[(int64_t)blockIdx.x * E + e] = hist[e];
}

// One block: per expert, prefix over tiles; exclusive scan over experts; heads; used list.
// tile_counts becomes the absolute start of each (tile, expert) run.
__global__ void __launch_bounds__(1024) k_perm_scan(uint32_t* __restrict__ tile_counts, int ntiles, int E,
                                                    uint32_t* __restrict__ heads, uint32_t* __restrict__ used3,
                                                    uint32_t* __restrict__ n_used) {
    pdl_wait();
    extern __shared__ uint32_t sm[];
    uint32_t* cnt = sm;       // E
    uint32_t* first = sm + E; // E
    __shared__ uint32_t carry, ucarry;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        uint32_t run = 0;
        for (int t = 0; t < ntiles; ++t) {
            uint32_t c = tile_counts[(int64_t)t * E + e];
            tile_counts[(int64_t)t * E + e] = run;
            run += c;
        }
        cnt[e] = run;
    }
    if (threadIdx.x == 0) {
        carry = 0;
        ucarry = 0;
    }
    __syncthreads();
    // exclusive scans of counts and of the used flags, E in chunks of blockDim
    __shared__ uint32_t wsum[32], wusum[32];
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int base = 0; base < E; base += blockDim.x) {
        int e = base + threadIdx.x;
        uint32_t c = e < E ? cnt[e] : 0;
        uint32_t u = c > 0 ? 1 : 0;
        uint32_t ic = c, iu = u;
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t a = __shfl_up_sync(0xffffffffu, ic, o), b = __shfl_up_sync(0xffffffffu, iu, o);
            if (lane >= o) {
                ic += a;
                iu += b;
            }
        }
        if (lane == 31) {
            wsum[warp] = ic;
            wusum[warp] = iu;
        }
        __syncthreads();
        if (warp == 0) {
            uint32_t a = lane < nw ? wsum[lane] : 0, b = lane < nw ? wusum[lane] : 0;
            for (int o = 1; o < 32; o <<= 1) {
                uint32_t x = __shfl_up_sync(0xffffffffu, a, o), y = __shfl_up_sync(0xffffffffu, b, o);
                if (lane >= o) {
                    a += x;
                    b += y;
                }
            }
            if (lane < nw) {
                wsum[lane] = a;
                wusum[lane] = b;
            }
        }
        __syncthreads();
        uint32_t pre = (warp ? wsum[warp - 1] : 0) + ic - c + carry;
        uint32_t upre = (warp ? wusum[warp - 1] : 0) + iu - u + ucarry;
        if (e < E) {
            first[e] = pre;
            heads[3 * e] = (uint32_t)e;
            heads[3 * e + 1] = pre;
            heads[3 * e + 2] = c;
            if (u) {
                used3[3 * upre] = (uint32_t)e;
                used3[3 * upre + 1] = pre;
                used3[3 * upre + 2] = c;
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            carry += wsum[nw - 1];
            ucarry += wusum[nw - 1];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) *n_used = ucarry;
    for (int e = threadIdx.x; e < E; e += blockDim.x)
        for (int t = 0; t < ntiles; ++t) tile_counts[(int64_t)t * E + e] += first[e];
}

// Stable scatter: warps of a tile take their 32 picks in order; within a warp, peers with the
// same expert are ranked by lane.
__global__ void __launch_bounds__(1024) k_perm_scatter(const uint32_t* __restrict__ ids, int64_t n, int E,
                                                       const uint32_t* __restrict__ tile_base,
                                                       uint32_t* __restrict__ pairs, const int32_t* n_dev) {
    pdl_wait();
    n = picks_of(n, n_dev);
    extern __shared__ uint32_t base[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) base[e] = tile_base[(int64_t)blockIdx.x * E + e];
    __syncthreads();
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int64_t i = (int64_t)blockIdx.x * PERM_TILE + threadIdx.x;
    bool valid = i < n;
    uint32_t id = valid ? ids[i] : 0xffffffffu;
    if (id >= (uint32_t)E) valid = false;
    for (int w = 0; w < 32; ++w) {
        if (warp == w) {
            uint32_t key = valid ? id : 0xffffffffu;
            uint32_t peers = __match_any_sync(0xffffffffu, key);
            uint32_t rank = __popc(peers & ((1u << lane) - 1u));
            if (valid) {
                pairs[base[id] + rank] = (uint32_t)i;
            }
            __syncwarp();
            if (valid && rank == 0) base[id] += __popc(peers);
        }
        __syncthreads();
    }
}

// Small piles in one block (n <= 2048 picks, E <= 1024 experts): counts, the exclusive scan,
// heads and the used list, then one thread per expert writes its own picks in pick order (stable
// by construction). Replaces the three launches of the general path for decode-sized batches.
constexpr int PERM_SMALL_N = 2048;
__global__ void __launch_bounds__(1024) k_perm_small(const uint32_t* __restrict__ ids, int n, int E,
                                                     uint32_t* __restrict__ pairs, uint32_t* __restrict__ heads,
                                                     uint32_t* __restrict__ used3, uint32_t* __restrict__ n_used,
                                                     int* err, const int32_t* n_dev) {
    pdl_wait();
    n = (int)picks_of(n, n_dev);
    __shared__ uint32_t sid[PERM_SMALL_N];
    __shared__ uint32_t cnt[1024];
    __shared__ uint32_t wsum[32], wusum[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    cnt[tid] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += 1024) {
        const uint32_t id = ids[i];
        sid[i] = id;
        if (id < (uint32_t)E) atomicAdd(&cnt[id], 1u);
        else dev_error(err, DE_BAD_ID);
    }
    __syncthreads();
    const uint32_t c = tid < E ? cnt[tid] : 0u, u = c > 0u ? 1u : 0u;
    uint32_t ic = c, iu = u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t a = __shfl_up_sync(0xffffffffu, ic, o), b = __shfl_up_sync(0xffffffffu, iu, o);
        if (lane >= o) {
            ic += a;
            iu += b;
        }
    }
    if (lane == 31) {
        wsum[warp] = ic;
        wusum[warp] = iu;
    }
    __syncthreads();
    if (warp == 0) {
        uint32_t a = wsum[lane], b = wusum[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t x = __shfl_up_sync(0xffffffffu, a, o), y = __shfl_up_sync(0xffffffffu, b, o);
            if (lane >= o) {
                a += x;
                b += y;
            }
        }
        wsum[lane] = a;
        wusum[lane] = b;
    }
    __syncthreads();
    const uint32_t first = (warp ? wsum[warp - 1] : 0u) + ic - c;
    const uint32_t uf = (warp ? wusum[warp - 1] : 0u) + iu - u;
    if (tid == 0) *n_used = wusum[31];
    if (tid < E) {
        heads[3 * tid] = (uint32_t)tid;
        heads[3 * tid + 1] = first;
        heads[3 * tid + 2] = c;
        if (u) {
            used3[3 * uf] = (uint32_t)tid;
            used3[3 * uf + 1] = first;
            used3[3 * uf + 2] = c;
        }
        cnt[tid] = first;  // running write position of this expert's pile
    }
    __syncthreads();
    // stable scatter: warp 0 takes the picks 32 at a time, in order; lanes with the same expert are
    // ranked by lane, and the expert's position advances by their number
    if (warp == 0)
        for (int i0 = 0; i0 < n; i0 += 32) {
            const int i = i0 + lane;
            const uint32_t id = i < n ? sid[i] : 0xffffffffu;
            const bool valid = id < (uint32_t)E;
            const uint32_t peers = __match_any_sync(0xffffffffu, valid ? id : 0xffffffffu);
            const uint32_t rank = __popc(peers & ((1u << lane) - 1u));
            if (valid) pairs[cnt[id] + rank] = (uint32_t)i;
            __syncwarp();
            if (valid && rank == 0) cnt[id] += __popc(peers);
            __syncwarp();
        }
}

// ---------------------------------------------------------------- host launchers
// Tiled router for large batches: a block computes 64 experts x 64 tokens; K runs in chunks of
// 32 columns staged in shared memory by cp.async (double-buffered, rows padded to 36 floats so
// the fragment loads of a warp hit 32 different banks). Warp w holds experts 16 (w % 4) .. +15
// and tokens 32 (w / 4) .. +31 as 2 x 4 m8n8k4 f64 tiles; each logit's exact products are summed
// in f64 in K order and rounded once.
constexpr int RT = 64, RK = 32, RPAD = 36;

__device__ __forceinline__ void cp16_zfill(void* dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}

__global__ void __launch_bounds__(256) k_router_tiled(const float* __restrict__ x, const float* __restrict__ w,
                                                      const float* __restrict__ bias, int T, int H, int E,
                                                      float* __restrict__ logits) {
    pdl_wait();
    __shared__ __align__(16) float ws[2][RT][RPAD];
    __shared__ __align__(16) float xs[2][RT][RPAD];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int e0 = blockIdx.x * RT, t0 = blockIdx.y * RT;
    const int eg = warp & 3, tg = warp >> 2;
    const int r = lane >> 2, kq = lane & 3;
    // staging: 64 rows x 8 pieces of 16 bytes per operand per chunk, two per thread
    auto stage = [&](int buf, int k0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int i = tid + 256 * h, row = i >> 3, pc = i & 7;
            const int kc = k0 + 4 * pc;
            const int kb = H - kc > 4 ? 16 : (H - kc > 0 ? 4 * (H - kc) : 0);
            const int e = e0 + row, t = t0 + row;
            const bool ein = e < E, tin = t < T;
            cp16_zfill(&ws[buf][row][4 * pc], w + (int64_t)(ein ? e : 0) * H + (kb ? kc : 0), ein ? kb : 0);
            cp16_zfill(&xs[buf][row][4 * pc], x + (int64_t)(tin ? t : 0) * H + (kb ? kc : 0), tin ? kb : 0);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    double c[2][4][2];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) c[i][j][0] = c[i][j][1] = 0.0;
    const int nch = (H + RK - 1) / RK;
    stage(0, 0);
    for (int ch = 0; ch < nch; ++ch) {
        const int buf = ch & 1;
        if (ch + 1 < nch) {
            stage(buf ^ 1, (ch + 1) * RK);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
#pragma unroll
        for (int k4 = 0; k4 < RK / 4; ++k4) {
            double a[2], b[4];
#pragma unroll
            for (int i = 0; i < 2; ++i) a[i] = (double)ws[buf][eg * 16 + 8 * i + r][4 * k4 + kq];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = (double)xs[buf][tg * 32 + 8 * j + r][4 * k4 + kq];
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) dmma_8x8x4(c[i][j], a[i], b[j]);
        }
        __syncthreads();  // the buffer is restaged two chunks later
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int e = e0 + eg * 16 + 8 * i + r, t = t0 + tg * 32 + 8 * j + 2 * kq + h;
                if (e < E && t < T) {
                    float l = (float)c[i][j][h];
                    if (bias) l = __fadd_rn(l, bias[e]);
                    logits[(int64_t)t * E + e] = l;
                }
            }
}

int launch_router(const float* x, const float* w, const float* b, int T, int H, int E, float* logits,
                  cudaStream_t st) {
    if (T == 0) return CWX_OK;
    if (T >= 1024 && H % 4 == 0) {
        cudaError_t e = launch_pdl(k_router_tiled, dim3((E + RT - 1) / RT, (T + RT - 1) / RT), dim3(256), 0, st, x, w,
                                   b, T, H, E, logits);
        return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_router_tiled");
    }
    cudaError_t e = launch_pdl(k_router, dim3((E + 7) / 8, (T + 7) / 8), dim3(256), 0, st, x, w, b, T, H, E, logits);
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_router");
}

int launch_route(const float* logits, int T, int E, int K, int norm, uint32_t* ids, float* w, const float* x,
                 const float* g_inp, int H, float* sgate, cudaStream_t st) {
    if (T == 0) return CWX_OK;
    cudaError_t e = launch_pdl(k_route, dim3(T), dim3(256), 0, st, logits, T, E, K, norm, ids, w, x, g_inp, H, sgate);
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_route");
}

int perm_launches(int64_t n, int E) { return n <= PERM_SMALL_N && E <= 1024 ? 1 : 3; }

size_t perm_scratch_bytes(int64_t n, int E) {
    int64_t ntiles = (n + PERM_TILE - 1) / PERM_TILE;
    return (size_t)(ntiles > 0 ? ntiles : 1) * E * 4;
}

int launch_permute(const uint32_t* ids, int64_t n, int E, uint32_t* pairs, uint32_t* heads, uint32_t* used3,
                   uint32_t* n_used, uint32_t* scratch, int* err, cudaStream_t st, const int32_t* n_dev) {
    if (n <= PERM_SMALL_N && E <= 1024) {
        cudaError_t e = launch_pdl(k_perm_small, dim3(1), dim3(1024), 0, st, ids, (int)n, E, pairs, heads, used3, n_used,
                                   err, n_dev);
        return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_perm_small");
    }
    int ntiles = (int)((n + PERM_TILE - 1) / PERM_TILE);
    if (ntiles == 0) ntiles = 1;
    size_t sh = (size_t)E * 4;
    // the scan keeps two words per expert: above 48 KB (more than 6,144 experts) the kernel must
    // be opted in to the larger dynamic shared memory (per device; repeated calls are cheap)
    if (2 * sh > 48 * 1024) {
        cudaError_t a = cudaFuncSetAttribute(k_perm_scan, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(2 * sh));
        if (a != cudaSuccess) return cuda_fail(a, "cudaFuncSetAttribute(k_perm_scan)");
    }
    cudaError_t e = launch_pdl(k_perm_count, dim3(ntiles), dim3(1024), sh, st, ids, n, E, scratch, err, n_dev);
    if (e == cudaSuccess)
        e = launch_pdl(k_perm_scan, dim3(1), dim3(1024), 2 * sh, st, scratch, ntiles, E, heads, used3, n_used);
    if (e == cudaSuccess)
        e = launch_pdl(k_perm_scatter, dim3(ntiles), dim3(1024), sh, st, ids, n, E, scratch, pairs, n_dev);
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "permute kernels");
}

}  // namespace cwx
