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

namespace cwx {

__device__ __forceinline__ float silu_f(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

// One warp per (row, 256 columns); lane l takes columns 8l..8l+7 of the block. Up to two
// independent preparations per launch (blockIdx.y picks one).
struct PrepPair {
    PrepArgs p[2];
};
__global__ void __launch_bounds__(256) k_prep(PrepPair pp) {
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
    if (p.mode == AM_Q8_K) {
        // max |x| with the lowest index among equals, and the signed value there
        float am = -1.f, mv = 0.f;
        int ai = 1 << 30;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float f = fabsf(v[j]);
            if (f > am) {
                am = f;
                ai = k0 + j;
                mv = v[j];
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float oa = __shfl_xor_sync(0xffffffffu, am, o);
            const int oi = __shfl_xor_sync(0xffffffffu, ai, o);
            const float ov = __shfl_xor_sync(0xffffffffu, mv, o);
            if (oa > am || (oa == am && oi < ai)) {
                am = oa;
                ai = oi;
                mv = ov;
            }
        }
        float d = 0.f;
        if (am == 0.f) {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = 0.f;
        } else {
            const float iscale = __fdiv_rn(-127.f, mv);
            d = __fdiv_rn(1.0f, iscale);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float qv = roundf(__fmul_rn(iscale, v[j]));
                v[j] = fminf(fmaxf(qv, -128.f), 127.f);
            }
        }
        uint32_t hi[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
            hi[j] = *reinterpret_cast<const uint32_t*>(&h);
        }
        const int c = k0 >> 6, ss = (k0 >> 4) & 3, q = (k0 >> 3) & 1;
        uint8_t* piece = p.out + r * packed_row_bytes(p.K) + b * 1024;
        const int ch = (ss * 2 + q) * 4 + c;
        *reinterpret_cast<uint4*>(piece + 16 * ch) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(piece + 512 + 16 * ch) = make_uint4(ch == 0 ? __float_as_uint(d) : 0u, 0u, 0u, 0u);
        return;
    } else if (p.mode == AM_Q8_0) {
        // 32-column blocks: lanes 4i..4i+3 hold block i
        float am = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) am = fmaxf(am, fabsf(v[j]));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
        const float d = __fdiv_rn(am, 127.f);
        const float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
        const float dh = __half2float(__float2half_rn(d));
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float qv = roundf(__fmul_rn(v[j], id));
            qv = fminf(fmaxf(qv, -128.f), 127.f);
            v[j] = __fmul_rn(qv, dh);
        }
    }
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
        const float2 hf = __half22float2(h);
        const __half2 l = __floats2half2_rn(__fsub_rn(v[2 * j], hf.x), __fsub_rn(v[2 * j + 1], hf.y));
        hi[j] = *reinterpret_cast<const uint32_t*>(&h);
        lo[j] = *reinterpret_cast<const uint32_t*>(&l);
    }
    const int c = k0 >> 6, ss = (k0 >> 4) & 3, q = (k0 >> 3) & 1;
    uint8_t* piece = p.out + r * packed_row_bytes(p.K) + b * 1024;
    *reinterpret_cast<uint4*>(piece + 16 * ((ss * 2 + q) * 4 + c)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(piece + 512 + 16 * ((ss * 2 + q) * 4 + c)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

// out[t] = sum_j w[t][j] * rows[t*K + j] (pick order, from 0) + sgate[t] * shared[t] + residual[t]
// rows are indexed by pick (t*K + j), or through idx (row of pick p = idx[p]) when idx is set.
__global__ void __launch_bounds__(256) k_combine(const float* __restrict__ rows, const uint32_t* __restrict__ idx,
                                                 const float* __restrict__ w, int T, int K, int H,
                                                 const float* __restrict__ shared, const float* __restrict__ sgate,
                                                 const float* __restrict__ residual, float* __restrict__ out) {
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
    const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i >= (int64_t)T * H) return;
    const int64_t t = i / H, c = i % H;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < K; ++j) {
        const int64_t p = t * K + j, r = idx ? (int64_t)idx[p] : p;
        const float4 v = *reinterpret_cast<const float4*>(rows + r * H + c);
        const float wj = w[p];
        acc.x = __fadd_rn(acc.x, __fmul_rn(v.x, wj));
        acc.y = __fadd_rn(acc.y, __fmul_rn(v.y, wj));
        acc.z = __fadd_rn(acc.z, __fmul_rn(v.z, wj));
        acc.w = __fadd_rn(acc.w, __fmul_rn(v.w, wj));
    }
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
    k_prep<<<dim3((unsigned)((warps * 32 + 255) / 256), nj), 256, 0, st>>>(pp);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_prep");
}

int launch_prep(const PrepArgs& p, cudaStream_t st) { return launch_prep2(&p, 1, st); }

int launch_combine(const float* rows, const float* w, int T, int K, int H, const float* shared, const float* sgate,
                   const float* residual, float* out, cudaStream_t st, const uint32_t* idx) {
    if (T == 0) return CWX_OK;
    const int64_t n = (int64_t)T * H;
    const bool vec = H % 4 == 0 && !(((uintptr_t)rows | (uintptr_t)out | (uintptr_t)shared | (uintptr_t)residual) & 15);
    if (vec)
        k_combine4<<<(unsigned)((n / 4 + 255) / 256), 256, 0, st>>>(rows, idx, w, T, K, H, shared, sgate, residual,
                                                                    out);
    else
        k_combine<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(rows, idx, w, T, K, H, shared, sgate, residual, out);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_combine");
}

}  // namespace cwx
