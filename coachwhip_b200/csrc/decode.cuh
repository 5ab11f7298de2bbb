// Device dequantisation of GGUF quant blocks, 32 consecutive weights of one row at a time.
//
// Each routine reproduces the reference's to_float arithmetic operation for operation (the
// products and differences use the _rn intrinsics so no FMA contraction changes a rounding),
// so the f32 values are bit-identical to the CPU restatement:
//   Q4_K  vendor/candle-core/src/quantized/k_quants.rs:1821-1848
//   Q6_K  k_quants.rs:2420-2451          Q8_0 k_quants.rs:766-782
//   MXFP4 k_quants.rs:673-691 (+ e8m0_to_f32_half 642-649)
//   IQ3_S vendor/candle-metal-kernels/src/metal_src/quantized.metal:6892-6915
//   IQ2_S quantized.metal:6917-6934
// `row` points at one row's bytes of one 256-column K-piece (see the tiled layout in
// cwx_common.cuh); `u` is the 32-column unit inside the piece (0..7).
#pragma once
#include "cwx_common.cuh"
#include "iq_grids.h"

namespace cwx {

struct Tables {
    const uint64_t* iq2s;  // 1024 entries, 8 grid bytes each
    const uint32_t* iq3s;  // 512 entries, 4 grid bytes each
};

__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t ld_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

__device__ __forceinline__ void get_scale_min_k4(int j, const uint8_t* q, int* d, int* m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

__device__ __forceinline__ void dec_q4k(const uint8_t* b, int u, float* w) {
    float d = h2f_bits(ld_u16(b)), mn = h2f_bits(ld_u16(b + 2));
    const uint8_t* scales = b + 4;
    const uint8_t* q = b + 16 + 32 * (u >> 1);
    int sc, m;
    get_scale_min_k4(u, scales, &sc, &m);
    float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(mn, (float)m);
    int shift = (u & 1) * 4;
#pragma unroll
    for (int l = 0; l < 32; ++l) w[l] = __fsub_rn(__fmul_rn(d1, (float)((q[l] >> shift) & 0xF)), m1);
}

__device__ __forceinline__ void dec_q6k(const uint8_t* b, int u, float* w) {
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    float d = h2f_bits(ld_u16(b + 208));
    int half = u >> 2, v = u & 3;
    ql += 64 * half;
    qh += 32 * half;
    sc += 8 * half;
#pragma unroll
    for (int l = 0; l < 32; ++l) {
        int q;
        if (v == 0) q = (ql[l] & 0xF) | ((qh[l] & 3) << 4);
        else if (v == 1) q = (ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4);
        else if (v == 2) q = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4);
        else q = (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4);
        w[l] = __fmul_rn(__fmul_rn(d, (float)sc[l / 16 + 2 * v]), (float)(q - 32));
    }
}

__device__ __forceinline__ void dec_q8_0(const uint8_t* b, int u, float* w) {
    b += 34 * u;
    float d = h2f_bits(ld_u16(b));
    const int8_t* qs = (const int8_t*)(b + 2);
#pragma unroll
    for (int j = 0; j < 32; ++j) w[j] = __fmul_rn((float)qs[j], d);
}

__device__ __forceinline__ float e8m0_to_f32_half(uint8_t e) {
    uint32_t bits = e < 2 ? (0x00200000u << e) : ((uint32_t)(e - 1) << 23);
    return __uint_as_float(bits);
}

__device__ __forceinline__ void dec_mxfp4(const uint8_t* b, int u, float* w) {
    b += 17 * u;
    float d = e8m0_to_f32_half(b[0]);
    const int8_t kv[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        uint8_t q = b[1 + j];
        w[j] = __fmul_rn((float)kv[q & 0xF], d);
        w[j + 16] = __fmul_rn((float)kv[q >> 4], d);
    }
}

__device__ __forceinline__ void dec_iq3s(const uint8_t* b, int ib, float* w, const uint32_t* grid) {
    float d = h2f_bits(ld_u16(b));
    const uint8_t* qs = b + 2 + 8 * ib;
    uint8_t qh = b[66 + ib];
    const uint8_t* signs = b + 74 + 4 * ib;
    uint8_t scb = b[106 + ib / 2];
    float dl = __fmul_rn(d, (float)(1 + 2 * ((scb >> (4 * (ib & 1))) & 0xF)));
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        uint32_t gv = grid[qs[g] | (((qh >> g) & 1) << 8)];
        uint8_t s = signs[g >> 1] >> (4 * (g & 1));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float v = __fmul_rn(dl, (float)((gv >> (8 * j)) & 0xFF));
            w[4 * g + j] = ((s >> j) & 1) ? -v : v;
        }
    }
}

__device__ __forceinline__ void dec_iq2s(const uint8_t* b, int ib, float* w, const uint64_t* grid) {
    float d = h2f_bits(ld_u16(b));
    const uint8_t* qs = b + 2 + 4 * ib;
    const uint8_t* signs = b + 34 + 4 * ib;
    uint8_t qh = b[66 + ib];
    uint8_t scb = b[74 + ib];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        float dl = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)((scb >> (4 * (g >> 1))) & 0xF))), 0.25f);
        uint64_t gv = grid[qs[g] | (((qh >> (2 * g)) & 3) << 8)];
        uint8_t s = signs[g];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float v = __fmul_rn(dl, (float)((gv >> (8 * j)) & 0xFF));
            w[8 * g + j] = ((s >> j) & 1) ? -v : v;
        }
    }
}

// 32 weights of unit u of one row of a K-piece, bit-exact f32.
__device__ __forceinline__ void decode_unit(int fmt, const uint8_t* row, int u, float* w, const Tables& t) {
    switch (fmt) {
        case F_Q4_K: dec_q4k(row, u, w); break;
        case F_Q6_K: dec_q6k(row, u, w); break;
        case F_Q8_0: dec_q8_0(row, u, w); break;
        case F_MXFP4: dec_mxfp4(row, u, w); break;
        case F_IQ3_S: dec_iq3s(row, u, w, t.iq3s); break;
        case F_IQ2_S: dec_iq2s(row, u, w, t.iq2s); break;
        default:
#pragma unroll
            for (int j = 0; j < 32; ++j) w[j] = 0.f;
    }
}

static __device__ const uint16_t d_iq2s_codes[1024] = CWX_IQ2S_CODES;
static __device__ const uint16_t d_iq3s_codes[512] = CWX_IQ3S_CODES;

// Expand the packed codebooks into shared memory (called by every thread of a CTA; the caller
// synchronises before use).
__device__ __forceinline__ void load_tables(uint64_t* s_iq2s, uint32_t* s_iq3s) {
    for (int i = threadIdx.x; i < 1024; i += blockDim.x) s_iq2s[i] = cwx_iq2s_expand(d_iq2s_codes[i]);
    for (int i = threadIdx.x; i < 512; i += blockDim.x) s_iq3s[i] = cwx_iq3s_expand(d_iq3s_codes[i]);
}

}  // namespace cwx
