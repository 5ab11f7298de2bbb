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
// lanes reduced as in vec_reduce 51-66), exp correctly rounded to f32 (what glibc's expf, which
// Rust's f32::exp calls, returns), the pick order of a stable descending sort. Router logits
// accumulate exact f32 products in f64 (T <= 64) and round once.
#include "cwx_common.cuh"
#include "kernels.cuh"

namespace cwx {

__device__ __forceinline__ float exp_cr(float x) { return (float)exp((double)x); }

// candle's AVX order for a sum whose 32-element steps live one per lane: lane L holds the sum of
// elements 32*s + L over the whole steps, in step order. Returns the reduced value in all lanes.
__device__ __forceinline__ float avx_lane_tree(float acc) {
    float b = __shfl_down_sync(0xffffffffu, acc, 8);
    float c = __shfl_down_sync(0xffffffffu, acc, 16);
    float d = __shfl_down_sync(0xffffffffu, acc, 24);
    float X = __fadd_rn(__fadd_rn(acc, b), __fadd_rn(c, d));  // valid in lanes 0..7
    float X4 = __shfl_down_sync(0xffffffffu, X, 4);
    float t0 = __fadd_rn(X, X4);  // valid in lanes 0..3
    float t1 = __shfl_down_sync(0xffffffffu, t0, 1);
    float t2 = __shfl_down_sync(0xffffffffu, t0, 2);
    float t3 = __shfl_down_sync(0xffffffffu, t0, 3);
    float r = __fadd_rn(__fadd_rn(t0, t1), __fadd_rn(t2, t3));
    return __shfl_sync(0xffffffffu, r, 0);
}

// logits (T, E): one warp per (expert, K quarter), 8 tokens per block row (blockIdx.y), f64
// partial sums reduced in a fixed order. Block = 8 warps = 2 experts.
__global__ void __launch_bounds__(256) k_router(const float* __restrict__ x, const float* __restrict__ w,
                                                const float* __restrict__ bias, int T, int H, int E,
                                                float* __restrict__ logits) {
    __shared__ double part[8][8];
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int e = blockIdx.x * 2 + (warp >> 2);
    int q = warp & 3;
    int kq = (H + 3) / 4;
    int k0 = q * kq, k1 = min(H, k0 + kq);
    const float* wr = w + (int64_t)(e < E ? e : 0) * H;
    for (int t0 = 8 * blockIdx.y; t0 < T; t0 += 8 * gridDim.y) {
        double acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.0;
        if (e < E) {
            for (int k = k0 + lane; k < k1; k += 32) {
                double wv = (double)__ldg(wr + k);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (t0 + j < T) acc[j] = fma(wv, (double)__ldg(x + (int64_t)(t0 + j) * H + k), acc[j]);
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            double v = acc[j];
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            acc[j] = v;
        }
        if (lane < 8) {
            double v = acc[0];
#pragma unroll
            for (int j = 1; j < 8; ++j)
                if (lane == j) v = acc[j];
            part[warp][lane] = v;
        }
        __syncthreads();
        if ((warp & 3) == 0 && lane < 8 && e < E && t0 + lane < T) {
            double s = ((part[warp][lane] + part[warp + 1][lane]) + part[warp + 2][lane]) + part[warp + 3][lane];
            float l = (float)s;
            if (bias) l = __fadd_rn(l, bias[e]);
            logits[(int64_t)(t0 + lane) * E + e] = l;
        }
        __syncthreads();
    }
}

// One warp per token: softmax over E (<= 1024), k picks (<= 32) best first with ties to the
// lowest id, weights renormalised over the picks when norm. Optionally the shared-expert gate
// sigmoid(sum_keepdim(x * gate_inp)) in candle's AVX summation order.
__global__ void __launch_bounds__(256) k_route(const float* __restrict__ logits, int T, int E, int K, int norm,
                                               uint32_t* __restrict__ ids, float* __restrict__ wout,
                                               const float* __restrict__ x, const float* __restrict__ g_inp,
                                               int H, float* __restrict__ sgate) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const float* l = logits + (int64_t)warp * E;
    const int NV = 32;  // up to 1024 experts
    float v[NV];
    int nv = (E + 31) / 32;
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        int e = 32 * i + lane;
        v[i] = (i < nv && e < E) ? l[e] : -INFINITY;
        if (i < nv && e < E) mx = fmaxf(mx, v[i]);
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    int whole = E / 32;  // whole 32-element steps
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        int e = 32 * i + lane;
        if (i < nv && e < E) v[i] = exp_cr(__fsub_rn(v[i], mx));
        if (i < whole) acc = __fadd_rn(acc, v[i]);
    }
    float s = avx_lane_tree(acc);
    if (E % 32) {  // tail elements added one by one, in order
        float tail = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i)
            if (i == whole) tail = v[i];
        for (int j = 0; j < E % 32; ++j) s = __fadd_rn(s, __shfl_sync(0xffffffffu, tail, j));
    }
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        int e = 32 * i + lane;
        v[i] = (i < nv && e < E) ? __fdiv_rn(v[i], s) : -1.0f;  // probabilities; -1 marks padding
    }
    float pw[32];
    uint32_t pid[32];
    for (int j = 0; j < K; ++j) {
        float bv = -2.0f;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            int e = 32 * i + lane;
            if (i < nv && e < E && v[i] > bv) {  // ascending e within a lane: first wins ties
                bv = v[i];
                bi = e;
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (bi >= E) bi = E - 1;  // only when every candidate is NaN: keep ids in range
        pw[j] = bv;
        pid[j] = (uint32_t)bi;
#pragma unroll
        for (int i = 0; i < NV; ++i)
            if (32 * i + lane == bi) v[i] = -3.0f;  // taken
    }
    if (lane == 0) {
        float tot = 0.f;
        if (norm)
            for (int j = 0; j < K; ++j) tot = __fadd_rn(tot, pw[j]);
        for (int j = 0; j < K; ++j) {
            ids[(int64_t)warp * K + j] = pid[j];
            wout[(int64_t)warp * K + j] = norm ? __fdiv_rn(pw[j], tot) : pw[j];
        }
    }
    if (sgate) {
        const float* xr = x + (int64_t)warp * H;
        int wholeh = H / 32;
        float a = 0.f;
        for (int i = 0; i < wholeh; ++i) a = __fadd_rn(a, __fmul_rn(xr[32 * i + lane], g_inp[32 * i + lane]));
        float sum = avx_lane_tree(a);
        for (int j = wholeh * 32; j < H; ++j) sum = __fadd_rn(sum, __fmul_rn(xr[j], g_inp[j]));
        if (lane == 0) sgate[warp] = __fdiv_rn(1.0f, __fadd_rn(exp_cr(-sum), 1.0f));
    }
}

// ---------------------------------------------------------------- piles
constexpr int PERM_TILE = 1024;

__global__ void __launch_bounds__(1024) k_perm_count(const uint32_t* __restrict__ ids, int64_t n, int E,
                                                     uint32_t* __restrict__ tile_counts, int* err) {
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
                                                       uint32_t* __restrict__ pairs) {
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

// ---------------------------------------------------------------- host launchers
int launch_router(const float* x, const float* w, const float* b, int T, int H, int E, float* logits,
                  cudaStream_t st) {
    if (T == 0) return CWX_OK;
    int ty = (T + 7) / 8;
    if (ty > 64) ty = 64;
    k_router<<<dim3((E + 1) / 2, ty), 256, 0, st>>>(x, w, b, T, H, E, logits);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_router");
}

int launch_route(const float* logits, int T, int E, int K, int norm, uint32_t* ids, float* w, const float* x,
                 const float* g_inp, int H, float* sgate, cudaStream_t st) {
    if (T == 0) return CWX_OK;
    int warps_per_block = 8;
    k_route<<<(T + warps_per_block - 1) / warps_per_block, 32 * warps_per_block, 0, st>>>(logits, T, E, K, norm, ids,
                                                                                          w, x, g_inp, H, sgate);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_route");
}

size_t perm_scratch_bytes(int64_t n, int E) {
    int64_t ntiles = (n + PERM_TILE - 1) / PERM_TILE;
    return (size_t)(ntiles > 0 ? ntiles : 1) * E * 4;
}

int launch_permute(const uint32_t* ids, int64_t n, int E, uint32_t* pairs, uint32_t* heads, uint32_t* used3,
                   uint32_t* n_used, uint32_t* scratch, int* err, cudaStream_t st) {
    int ntiles = (int)((n + PERM_TILE - 1) / PERM_TILE);
    if (ntiles == 0) ntiles = 1;
    size_t sh = (size_t)E * 4;
    k_perm_count<<<ntiles, 1024, sh, st>>>(ids, n, E, scratch, err);
    k_perm_scan<<<1, 1024, 2 * sh, st>>>(scratch, ntiles, E, heads, used3, n_used);
    k_perm_scatter<<<ntiles, 1024, sh, st>>>(ids, n, E, scratch, pairs);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "permute kernels");
}

}  // namespace cwx
