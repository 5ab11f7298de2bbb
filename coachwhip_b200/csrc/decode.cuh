// Device dequantisation of GGUF quant blocks.
//
// The exact routines reproduce the reference's to_float arithmetic operation for operation (the
// products and differences use the _rn intrinsics so no FMA contraction changes a rounding), so
// the f32 values are bit-identical to the CPU restatement:
//   Q4_K  vendor/candle-core/src/quantized/k_quants.rs:1821-1848
//   Q6_K  k_quants.rs:2420-2451          Q8_0 k_quants.rs:766-782
//   MXFP4 k_quants.rs:673-691 (+ e8m0_to_f32_half 642-649)
//   IQ3_S vendor/candle-metal-kernels/src/metal_src/quantized.metal:6892-6915
//   IQ2_S quantized.metal:6917-6934
//   IQ2_XXS quantized.metal:6819-6842   IQ3_XXS :6862-6890   IQ4_XS :6999-7018
// The fast IQ paths produce f16 pairs for the tensor cores: the codebook values are exact in f16,
// the per-16/32-column scale is rounded to f16 (about 2^-11 relative per weight).
//
// Row addressing (see the tiled layout in cwx_common.cuh): K-quants, Q8_0 and MXFP4 rows are
// whole (row r of a piece at r * piece_row_bytes); the IQ formats' pieces are 16-row groups stored
// field by field, addressed through IqRow.
#pragma once
#include "cwx_common.cuh"
#include "iq_grids.h"

namespace cwx {

// f16 codebooks and sign masks in shared memory (codebook values are small integers, exact in f16).
struct HTables {
    const uint4* g2;   // IQ2_S: 1024 entries x 8 halves
    const uint2* g3;   // IQ3_S: 512 entries x 4 halves
    const uint4* sgn;  // sign byte -> f16 sign bits of 8 values (4 words of 2 halves)
};
constexpr int HTABLES_BYTES = 16384 + 4096 + 4096;

__device__ __forceinline__ float half_at(const void* p, int j) {
    return __half2float(reinterpret_cast<const __half*>(p)[j]);
}
__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t ld_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

__device__ __forceinline__ void get_scale_min_k4(int j, const uint8_t* q, int* d, int* m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

__device__ __forceinline__ float e8m0_to_f32_half(uint8_t e) {
    uint32_t bits = e < 2 ? (0x00200000u << e) : ((uint32_t)(e - 1) << 23);
    return __uint_as_float(bits);
}

// One row of an IQ2_S / IQ3_S 16-row group (layout in cwx_common.cuh); byte b of its GGUF block.
struct IqRow {
    const uint8_t* grp;
    int rg;
};
__device__ __forceinline__ uint8_t iq_byte(int fmt, const IqRow& r, int b) { return r.grp[soa_offset(fmt, r.rg, b)]; }
// Row rr of a piece (or of rows staged from it, starting at a 16-row boundary), rows prb bytes.
__device__ __forceinline__ IqRow iq_row_in(const uint8_t* piece, int rr, int64_t prb) {
    return IqRow{piece + (int64_t)(rr >> 4) * 16 * prb, rr & 15};
}

// Codebook value j of grid entry idx: from the shared-memory f16 tables, or from the packed
// codebooks in global memory when no tables are staged.
static __device__ const uint16_t d_iq2s_codes[1024] = CWX_IQ2S_CODES;
static __device__ const uint16_t d_iq3s_codes[512] = CWX_IQ3S_CODES;
static __device__ const uint16_t d_iq2xxs_codes[256] = CWX_IQ2XXS_CODES;
static __device__ const uint16_t d_iq3xxs_codes[256] = CWX_IQ3XXS_CODES;
template <bool SMEM>
__device__ __forceinline__ float iq_grid(int fmt, const HTables& t, int idx, int j) {
    if (SMEM) return fmt == F_IQ2_S ? half_at(&t.g2[idx], j) : half_at(&t.g3[idx], j);
    if (fmt == F_IQ2_S) return (float)((cwx_iq2s_expand(d_iq2s_codes[idx]) >> (8 * j)) & 0xFF);
    return (float)((cwx_iq3s_expand(d_iq3s_codes[idx]) >> (8 * j)) & 0xFF);
}

// ---------------------------------------------------------------- exact 16-column runs
// 16 consecutive columns [kofs, kofs+16) of one row's 256-column piece, bit-exact f32.
__device__ __forceinline__ uint32_t iq_u32(int fmt, const IqRow& r, int b) {
    return (uint32_t)iq_byte(fmt, r, b) | ((uint32_t)iq_byte(fmt, r, b + 1) << 8) |
           ((uint32_t)iq_byte(fmt, r, b + 2) << 16) | ((uint32_t)iq_byte(fmt, r, b + 3) << 24);
}

template <bool SMEM>
__device__ __forceinline__ void dec16_iq_exact(int fmt, const IqRow& r, int kofs, float* v, const HTables& t) {
    const int ib = kofs >> 5;
    if (fmt == F_MXFP4) {  // GGUF block ib of the piece row: e at 17 ib, nibble bytes after it
        const float dm = e8m0_to_f32_half(iq_byte(fmt, r, 17 * ib));
        const int8_t kv[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
        const int sh = (kofs & 16) ? 4 : 0;
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = __fmul_rn((float)kv[(iq_byte(fmt, r, 17 * ib + 1 + i) >> sh) & 0xF], dm);
        return;
    }
    const float d = h2f_bits((uint16_t)(iq_byte(fmt, r, 0) | (iq_byte(fmt, r, 1) << 8)));
    if (fmt == F_IQ2_XXS) {  // 8 bytes per 32 columns: 4 grid entries, then signs and scale
        const uint32_t aux = iq_u32(fmt, r, 2 + 8 * ib + 4);
        const float dl = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(aux >> 28))), 0.25f);
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
            const int g = ((kofs & 16) >> 3) + gi;
            const uint64_t grid = cwx_iq2s_expand(d_iq2xxs_codes[iq_byte(fmt, r, 2 + 8 * ib + g)]);
            const uint32_t sg = cwx_ksigns((aux >> (7 * g)) & 127u);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float x = __fmul_rn(dl, (float)((grid >> (8 * j)) & 0xFF));
                v[8 * gi + j] = ((sg >> j) & 1) ? -x : x;
            }
        }
        return;
    }
    if (fmt == F_IQ3_XXS) {  // grid entries at 2 + 8 per 32 columns; signs and scale at 66 + 4 per 32
        const uint32_t aux = iq_u32(fmt, r, 66 + 4 * ib);
        const float dl = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(aux >> 28))), 0.5f);
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
            const int g = ((kofs & 16) >> 3) + gi;
            const uint32_t sg = cwx_ksigns((aux >> (7 * g)) & 127u);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t grid = cwx_iq3xxs_expand(d_iq3xxs_codes[iq_byte(fmt, r, 2 + 8 * ib + 2 * g + h)]);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float x = __fmul_rn(dl, (float)((grid >> (8 * j)) & 0xFF));
                    v[8 * gi + 4 * h + j] = ((sg >> (4 * h + j)) & 1) ? -x : x;
                }
            }
        }
        return;
    }
    if (fmt == F_IQ4_XS) {
        const uint32_t sh = (uint32_t)iq_byte(fmt, r, 2) | ((uint32_t)iq_byte(fmt, r, 3) << 8);
        const int ls = ((iq_byte(fmt, r, 4 + (ib >> 1)) >> (4 * (ib & 1))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4);
        const float dl = __fmul_rn(d, (float)(ls - 32));
        const int nsh = (kofs & 16) ? 4 : 0;
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = __fmul_rn(dl, (float)cwx_iq4nl((iq_byte(fmt, r, 8 + 16 * ib + i) >> nsh) & 0xF));
        return;
    }
    if (fmt == F_IQ2_S) {
        const uint8_t qh = iq_byte(fmt, r, 66 + ib);
        const int g0 = (kofs & 16) >> 3;  // 2 groups of 8
        const uint8_t sc = iq_byte(fmt, r, 74 + ib);
        const float dl = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)((sc >> (4 * (g0 >> 1))) & 0xF))), 0.25f);
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
            const int g = g0 + gi;
            const int idx = iq_byte(fmt, r, 2 + 4 * ib + g) | (((qh >> (2 * g)) & 3) << 8);
            const uint8_t sg = iq_byte(fmt, r, 34 + 4 * ib + g);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float x = __fmul_rn(dl, iq_grid<SMEM>(fmt, t, idx, j));
                v[8 * gi + j] = ((sg >> j) & 1) ? -x : x;
            }
        }
    } else {
        const uint8_t qh = iq_byte(fmt, r, 66 + ib);
        const int g0 = (kofs & 16) >> 2;  // 4 groups of 4
        const uint8_t sc = iq_byte(fmt, r, 106 + (ib >> 1));
        const float dl = __fmul_rn(d, (float)(1 + 2 * ((sc >> (4 * (ib & 1))) & 0xF)));
#pragma unroll
        for (int gi = 0; gi < 4; ++gi) {
            const int g = g0 + gi;
            const int idx = iq_byte(fmt, r, 2 + 8 * ib + g) | (((qh >> g) & 1) << 8);
            const uint8_t sg = iq_byte(fmt, r, 74 + 4 * ib + (g >> 1)) >> (4 * (g & 1));
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float x = __fmul_rn(dl, iq_grid<SMEM>(fmt, t, idx, j));
                v[4 * gi + j] = ((sg >> j) & 1) ? -x : x;
            }
        }
    }
}

// Whole-row formats: `b` is the row's bytes of its piece.
__device__ __forceinline__ void dec16_row_exact(int fmt, const uint8_t* b, int kofs, float* v) {
    switch (fmt) {
        case F_Q4_K: {
            const float d = h2f_bits(ld_u16(b)), mn = h2f_bits(ld_u16(b + 2));
            const int j = kofs >> 5, l0 = kofs & 16;
            int sc, m;
            get_scale_min_k4(j, b + 4, &sc, &m);
            const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(mn, (float)m);
            const uint8_t* q = b + 16 + 32 * (j >> 1) + l0;
            const int sh = (j & 1) * 4;
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __fsub_rn(__fmul_rn(d1, (float)((q[i] >> sh) & 0xF)), m1);
            break;
        }
        case F_Q6_K: {
            const int half = kofs >> 7, u = (kofs >> 5) & 3, l0 = kofs & 16;
            const uint8_t* ql = b + 64 * half;
            const uint8_t* qh = b + 128 + 32 * half;
            const int8_t* sc = (const int8_t*)(b + 192) + 8 * half;
            const float d = h2f_bits(ld_u16(b + 208));
            const float ds = __fmul_rn(d, (float)sc[(l0 >> 4) + 2 * u]);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int l = l0 + i;
                int q;
                if (u == 0) q = (ql[l] & 0xF) | ((qh[l] & 3) << 4);
                else if (u == 1) q = (ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4);
                else if (u == 2) q = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4);
                else q = (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4);
                v[i] = __fmul_rn(ds, (float)(q - 32));
            }
            break;
        }
        case F_Q8_0: {
            const uint8_t* blk = b + 34 * (kofs >> 5);
            const float d = h2f_bits(ld_u16(blk));
            const int8_t* qs = (const int8_t*)(blk + 2) + (kofs & 16);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __fmul_rn((float)qs[i], d);
            break;
        }
        case F_MXFP4: {
            const uint8_t* blk = b + 17 * (kofs >> 5);
            const float d = e8m0_to_f32_half(blk[0]);
            const int8_t kv[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
            const int sh = (kofs & 16) ? 4 : 0;
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __fmul_rn((float)kv[(blk[1 + i] >> sh) & 0xF], d);
            break;
        }
        default:
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
    }
}

// Any format: row rr of a piece whose rows are prb bytes. SMEM: IQ codebooks from the
// shared-memory tables (load_htables) rather than from global memory.
template <bool SMEM>
__device__ __forceinline__ void dec16_exact(int fmt, const uint8_t* piece, int rr, int64_t prb, int kofs, float* v,
                                            const HTables& t) {
    if (soa_piece(fmt, prb)) dec16_iq_exact<SMEM>(fmt, iq_row_in(piece, rr, prb), kofs, v, t);
    else dec16_row_exact(fmt, piece + (int64_t)rr * prb, kofs, v);
}

// ---------------------------------------------------------------- tables
// Expand the packed codebooks into f16 tables in shared memory (every thread of the CTA calls
// this; the caller synchronises before use).
__device__ __forceinline__ void load_htables(uint4* g2, uint2* g3, uint4* sgn) {
    for (int i = threadIdx.x; i < 1024; i += blockDim.x) {
        const uint64_t v = cwx_iq2s_expand(d_iq2s_codes[i]);
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            __half2 h = __floats2half2_rn((float)((v >> (16 * j)) & 0xFF), (float)((v >> (16 * j + 8)) & 0xFF));
            w[j] = *reinterpret_cast<uint32_t*>(&h);
        }
        g2[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    for (int i = threadIdx.x; i < 512; i += blockDim.x) {
        const uint32_t v = cwx_iq3s_expand(d_iq3s_codes[i]);
        __half2 a = __floats2half2_rn((float)(v & 0xFF), (float)((v >> 8) & 0xFF));
        __half2 b = __floats2half2_rn((float)((v >> 16) & 0xFF), (float)(v >> 24));
        g3[i] = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
    }
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            w[j] = (((i >> (2 * j)) & 1) ? 0x8000u : 0u) | (((i >> (2 * j + 1)) & 1) ? 0x80000000u : 0u);
        sgn[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

}  // namespace cwx
