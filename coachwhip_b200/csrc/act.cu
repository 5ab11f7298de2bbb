// Activation preparation for the expert products, and the weighted combine.
//
//   activation       ExpertAct::hidden crates/engine/src/experts.rs:2389-2406 (SiLU; gpt-oss clamped
//                    SwiGLU with per-expert biases), cw_silu_mul crates/engine/src/fuse_kernel.rs:77-96
//   Q8 activations   BlockQ8K::from_float vendor/candle-core/src/quantized/k_quants.rs:2495-2534,
//                    BlockQ8_0::from_float k_quants.rs:784-820 (the VecDotType quantisation candle's
//                    CPU QMatMul applies to its left-hand side, k_quants.rs:2595-2603)
//   combine          cw_weighted_sum fuse_kernel.rs:277-291 (pick order) + shared expert
//                    crates/engine/src/model_next.rs:731-741 + residual model_next.rs:1437
//
// Packed activation rows: per 256-column piece, 1024 bytes: first the 32 hi chunks, then the 32 lo
// chunks, each chunk 8 f16 values; chunk (ss*2 + q)*4 + c of a half holds columns
// 64c + 16ss + 8q + 0..7. This is the order in which the grouped products' threads read them
// (gemv.cu), and a product that needs only the hi parts copies the first 528 bytes of a piece.
// Q8_K rows (one Q8_K block per piece) hold the block's codes as exact f16 integers in the hi
// chunks and the block scale d as an f32 at byte 512 (the rest of the lo half is zero): the
// products sum code x weight per piece and scale the sum by d once.
#include "cwx_common.cuh"
#include "kernels.cuh"
#include "products.cuh"

namespace cwx {

// One warp per (row, 256 columns); lane l takes columns 8l..8l+7 of the block. Up to two
// independent preparations per launch (blockIdx.y picks one).
struct PrepPair {
    PrepArgs p[2];
};
__global__ void __launch_bounds__(256) k_prep(PrepPair pp) {
    pdl_wait();
    const PrepArgs& p = pp.p[blockIdx.y];
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t nb = (p.K + 255) / 256;
    if (w >= p.R * nb) return;
    const int64_t r = w / nb, b = w % nb;
    const int64_t c0 = b * 256;
    const int len = (int)(p.K - c0 < 256 ? p.K - c0 : 256);
    const int k0 = 8 * lane;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (k0 + j < len) ? p.src[r * p.K + c0 + k0 + j] : 0.f;
    if (p.up) {
        if (p.act == CWX_ACT_SILU) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (k0 + j < len) v[j] = __fmul_rn(silu_f(v[j]), p.up[r * p.K + c0 + k0 + j]);
        } else {
            const int64_t e = p.ids ? (int64_t)p.ids[r] : 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (k0 + j >= len) continue;
                const int64_t col = c0 + k0 + j;
                float gv = v[j], uv = p.up[r * p.K + col];
                if (p.gate_b) gv = __fadd_rn(gv, p.gate_b[e * p.K + col]);
                gv = fminf(gv, p.limit);
                if (p.up_b) uv = __fadd_rn(uv, p.up_b[e * p.K + col]);
                uv = fminf(fmaxf(uv, -p.limit), p.limit);
                const float z = __fmul_rn(gv, p.alpha);
                const float sg = __fdiv_rn(1.0f, __fadd_rn(expf(-z), 1.0f));
                v[j] = __fmul_rn(__fadd_rn(uv, 1.0f), __fmul_rn(gv, sg));
            }
        }
    }
    pack_piece(p.mode, v, p.out + r * packed_row_bytes(p.K) + b * 1024, lane);
}

// acc + sum_j w[t][j] * rows[pick j][c .. c+3] in pick order; the rows of up to 8 picks are
// loaded before the first add, so their loads are in flight together.
__device__ __forceinline__ float4 sum_picks4(const float* __restrict__ rows, const uint32_t* __restrict__ idx,
                                             const float* __restrict__ w, int64_t t, int K, int H, int64_t c,
                                             float4 acc) {
    for (int j0 = 0; j0 < K; j0 += 8) {
        float4 v[8];
        float wj[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (j0 + u < K) {
                const int64_t p = t * K + j0 + u, r = idx ? (int64_t)idx[p] : p;
                v[u] = *reinterpret_cast<const float4*>(rows + r * H + c);
                wj[u] = w[p];
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (j0 + u < K) {
                acc.x = __fadd_rn(acc.x, __fmul_rn(v[u].x, wj[u]));
                acc.y = __fadd_rn(acc.y, __fmul_rn(v[u].y, wj[u]));
                acc.z = __fadd_rn(acc.z, __fmul_rn(v[u].z, wj[u]));
                acc.w = __fadd_rn(acc.w, __fmul_rn(v[u].w, wj[u]));
            }
        }
    }
    return acc;
}

// out[t] = sum_j w[t][j] * rows[t*K + j] (pick order, from 0) + sgate[t] * shared[t] + residual[t]
// rows are indexed by pick (t*K + j), or through idx (row of pick p = idx[p]) when idx is set.
__global__ void __launch_bounds__(256) k_combine(const float* __restrict__ rows, const uint32_t* __restrict__ idx,
                                                 const float* __restrict__ w, int T, int K, int H,
                                                 const float* __restrict__ shared, const float* __restrict__ sgate,
                                                 const float* __restrict__ residual, float* __restrict__ out) {
    pdl_wait();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * H) return;
    const int64_t t = i / H, c = i % H;
    float acc = 0.f;
    for (int j = 0; j < K; ++j) {
        const int64_t p = t * K + j, r = idx ? (int64_t)idx[p] : p;
        acc = __fadd_rn(acc, __fmul_rn(rows[r * H + c], w[p]));
    }
    if (shared) acc = __fadd_rn(acc, __fmul_rn(shared[t * H + c], sgate[t]));
    if (residual) acc = __fadd_rn(acc, residual[i]);
    out[i] = acc;
}

// The same sum four columns at a time (H a multiple of 4): one block row of float4 per token.
__global__ void __launch_bounds__(256) k_combine4(const float* __restrict__ rows, const uint32_t* __restrict__ idx,
                                                  const float* __restrict__ w, int T, int K, int H,
                                                  const float* __restrict__ shared, const float* __restrict__ sgate,
                                                  const float* __restrict__ residual, float* __restrict__ out) {
    pdl_wait();
    const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i >= (int64_t)T * H) return;
    const int64_t t = i / H, c = i % H;
    const float4 acc0 = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 acc = sum_picks4(rows, idx, w, t, K, H, c, acc0);
    if (shared) {
        const float4 v = *reinterpret_cast<const float4*>(shared + t * H + c);
        const float g = sgate[t];
        acc.x = __fadd_rn(acc.x, __fmul_rn(v.x, g));
        acc.y = __fadd_rn(acc.y, __fmul_rn(v.y, g));
        acc.z = __fadd_rn(acc.z, __fmul_rn(v.z, g));
        acc.w = __fadd_rn(acc.w, __fmul_rn(v.w, g));
    }
    if (residual) {
        const float4 v = *reinterpret_cast<const float4*>(residual + i);
        acc.x = __fadd_rn(acc.x, v.x);
        acc.y = __fadd_rn(acc.y, v.y);
        acc.z = __fadd_rn(acc.z, v.z);
        acc.w = __fadd_rn(acc.w, v.w);
    }
    *reinterpret_cast<float4*>(out + i) = acc;
}

// ---------------------------------------------------------------- residual add + RMSNorm
// add_norm (crates/engine/src/fuse_kernel.rs:433-471): sum = a + b (+ c), out = rms_norm(sum) *
// alpha, candle's RmsNorm v / sqrt(mean(v^2) + eps) * alpha. One block per row; thread t owns the
// quads (4 consecutive columns) t, t + 256, ... in both passes, whether the row is read as float4
// or as scalars, so the result does not depend on the pointers' alignment. The squares are exact
// in f64 and summed in f64 in a fixed order (the thread's quads in order, an xor-shuffle tree,
// the warps in order), then rounded once: at least as accurate as the reference's f32 sums (a
// left-to-right sum on the CPU, a tree in the Metal kernel), so the outputs agree with either to
// the rounding of the reference's own sum. sqrt and the divide are correctly rounded, as in Rust.
__global__ void __launch_bounds__(NORM_THREADS) k_add_norm(const float* a, const float* b, const float* c,
                                                          const float* __restrict__ alpha, float eps, int H, int vec,
                                                          float* sum, float* out) {
    pdl_wait();
    const int64_t o = (int64_t)blockIdx.x * H;
    const int nq = (H + 3) / 4;
    double ss = 0.0;
    for (int q = threadIdx.x; q < nq; q += NORM_THREADS) {
        const int64_t i = o + 4 * q;
        if (vec) {
            const float4 va = *reinterpret_cast<const float4*>(a + i), vb = *reinterpret_cast<const float4*>(b + i);
            float4 v = make_float4(__fadd_rn(va.x, vb.x), __fadd_rn(va.y, vb.y), __fadd_rn(va.z, vb.z), __fadd_rn(va.w, vb.w));
            if (c) {
                const float4 vc = *reinterpret_cast<const float4*>(c + i);
                v = make_float4(__fadd_rn(v.x, vc.x), __fadd_rn(v.y, vc.y), __fadd_rn(v.z, vc.z), __fadd_rn(v.w, vc.w));
            }
            *reinterpret_cast<float4*>(sum + i) = v;
            ss += sq4(v);
        } else {
            for (int j = 0; j < 4 && 4 * q + j < H; ++j) {
                float v = __fadd_rn(a[i + j], b[i + j]);
                if (c) v = __fadd_rn(v, c[i + j]);
                sum[i + j] = v;
                ss += (double)v * (double)v;
            }
        }
    }
    norm_row(ss, sum + o, alpha, eps, H, vec, out + o);
}

// The combine of k_combine / k_combine4 (the same operations in the same order, so `out` is the
// same bits) with the next layer's RMSNorm of the row fused after it: one block per token.
__global__ void __launch_bounds__(NORM_THREADS) k_combine_norm(const float* __restrict__ rows,
                                                              const uint32_t* __restrict__ idx,
                                                              const float* __restrict__ w, int K, int H,
                                                              const float* __restrict__ shared,
                                                              const float* __restrict__ sgate,
                                                              const float* __restrict__ residual,
                                                              const float* __restrict__ alpha, float eps, int vec,
                                                              float* out, float* __restrict__ norm_out) {
    pdl_wait();
    const int64_t t = blockIdx.x, o = t * H;
    const int nq = (H + 3) / 4;
    const float g = shared ? sgate[t] : 0.f;
    double ss = 0.0;
    for (int q = threadIdx.x; q < nq; q += NORM_THREADS) {
        const int c = 4 * q;
        if (vec) {
            float4 acc = sum_picks4(rows, idx, w, t, K, H, c, make_float4(0.f, 0.f, 0.f, 0.f));
            if (shared) {
                const float4 v = *reinterpret_cast<const float4*>(shared + o + c);
                acc.x = __fadd_rn(acc.x, __fmul_rn(v.x, g));
                acc.y = __fadd_rn(acc.y, __fmul_rn(v.y, g));
                acc.z = __fadd_rn(acc.z, __fmul_rn(v.z, g));
                acc.w = __fadd_rn(acc.w, __fmul_rn(v.w, g));
            }
            if (residual) {
                const float4 v = *reinterpret_cast<const float4*>(residual + o + c);
                acc.x = __fadd_rn(acc.x, v.x);
                acc.y = __fadd_rn(acc.y, v.y);
                acc.z = __fadd_rn(acc.z, v.z);
                acc.w = __fadd_rn(acc.w, v.w);
            }
            *reinterpret_cast<float4*>(out + o + c) = acc;
            ss += sq4(acc);
        } else {
            for (int jc = c; jc < c + 4 && jc < H; ++jc) {
                float acc = 0.f;
                for (int j = 0; j < K; ++j) {
                    const int64_t p = t * K + j, r = idx ? (int64_t)idx[p] : p;
                    acc = __fadd_rn(acc, __fmul_rn(rows[r * H + jc], w[p]));
                }
                if (shared) acc = __fadd_rn(acc, __fmul_rn(shared[o + jc], g));
                if (residual) acc = __fadd_rn(acc, residual[o + jc]);
                out[o + jc] = acc;
                ss += (double)acc * (double)acc;
            }
        }
    }
    norm_row(ss, out + o, alpha, eps, H, vec, norm_out + o);
}

static bool al16(const void* p) { return !((uintptr_t)p & 15); }

int launch_add_norm(const float* a, const float* b, const float* c, const float* alpha, float eps, int64_t rows,
                    int H, float* sum, float* out, cudaStream_t st) {
    if (rows == 0) return CWX_OK;
    const int vec = H % 4 == 0 && al16(a) && al16(b) && (!c || al16(c)) && al16(alpha) && al16(sum) && al16(out);
    cudaError_t e = launch_pdl(k_add_norm, dim3((unsigned)rows), dim3(NORM_THREADS), 0, st, a, b, c, alpha, eps, H, vec,
                               sum, out);
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_add_norm");
}

int launch_combine_norm(const float* rows, const float* w, int T, int K, int H, const float* shared,
                        const float* sgate, const float* residual, const float* alpha, float eps, float* out,
                        float* norm_out, cudaStream_t st, const uint32_t* idx) {
    if (T == 0) return CWX_OK;
    const int vec = H % 4 == 0 && al16(rows) && al16(out) && (!shared || al16(shared)) &&
                    (!residual || al16(residual)) && al16(alpha) && al16(norm_out);
    cudaError_t e = launch_pdl(k_combine_norm, dim3((unsigned)T), dim3(NORM_THREADS), 0, st, rows, idx, w, K, H, shared,
                               sgate, residual, alpha, eps, vec, out, norm_out);
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_combine_norm");
}

int launch_prep2(const PrepArgs* p, int njobs, cudaStream_t st) {
    PrepPair pp;
    int64_t warps = 0;
    int nj = 0;
    for (int j = 0; j < njobs; ++j) {
        if (p[j].R == 0) continue;
        pp.p[nj++] = p[j];
        const int64_t wj = p[j].R * ((p[j].K + 255) / 256);
        if (wj > warps) warps = wj;
    }
    if (nj == 0) return CWX_OK;
    cudaError_t e = launch_pdl(k_prep, dim3((unsigned)((warps * 32 + 255) / 256), nj), dim3(256), 0, st, pp);
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_prep");
}

int launch_prep(const PrepArgs& p, cudaStream_t st) { return launch_prep2(&p, 1, st); }

int launch_combine(const float* rows, const float* w, int T, int K, int H, const float* shared, const float* sgate,
                   const float* residual, float* out, cudaStream_t st, const uint32_t* idx) {
    if (T == 0) return CWX_OK;
    const int64_t n = (int64_t)T * H;
    const bool vec = H % 4 == 0 && !(((uintptr_t)rows | (uintptr_t)out | (uintptr_t)shared | (uintptr_t)residual) & 15);
    cudaError_t e = vec ? launch_pdl(k_combine4, dim3((unsigned)((n / 4 + 255) / 256)), dim3(256), 0, st, rows, idx, w, T,
                                     K, H, shared, sgate, residual, out)
                        : launch_pdl(k_combine, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, rows, idx, w, T, K, H,
                                     shared, sgate, residual, out);
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_combine");
}

}  // namespace cwx
