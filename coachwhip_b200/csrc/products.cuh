// The expert products' per-thread building blocks, shared by the grouped products (gemv.cu) and
// the fused decode layer (decode_layer.cu): replicated codebook tables in shared memory, the IQ /
// MXFP4 / IQ4_XS fast paths (a thread's two rows x 64 columns of a 256-column piece as exact f16
// MMA fragments, block scales applied to each piece's f32 partial sum), the Q4_K products (two exact
// integer products per piece) and the activation fragments of the packed rows (act.cu).
//
// The weight pointers these take address a 16-row group of a piece in the tiled bank layout
// (cwx_common.cuh): the layout in HBM and in a shared-memory slot copied from it are the same.
#pragma once
#include "cwx_common.cuh"
#include "decode.cuh"

namespace cwx {

// ---------------------------------------------------------------- activation and routing arithmetic
__device__ __forceinline__ float silu_f(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

// exp correctly rounded to f32: f64 exp rounded once.
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


template <int FMT>
struct Tbl {  // replicated codebook bytes in shared memory (128 bytes per entry)
    static constexpr int BYTES = FMT == F_IQ2_S ? 1024 * 128
                                 : FMT == F_IQ3_S ? 512 * 128
                                 : (FMT == F_IQ2_XXS || FMT == F_IQ3_XXS || FMT == F_IQ4_XS || FMT == F_MXFP4)
                                     ? 256 * 128
                                                                                               : 0;
};
// This lane's copy of the table: 8-value codebooks (IQ2_S, IQ2_XXS) keep 8 copies of 16 bytes per
// entry, 4-value ones (IQ3_S, IQ3_XXS) 16 copies of 8 bytes, the IQ4_XS nibble-pair table (256
// pairs of levels) 32 copies of 4 bytes.
__device__ __forceinline__ int tbl_lane(int fmt, int lane) {
    return (fmt == F_IQ2_S || fmt == F_IQ2_XXS)    ? (lane & 7) * 16
           : (fmt == F_IQ4_XS || fmt == F_MXFP4) ? (lane & 31) * 4
                                                 : (lane & 15) * 8;
}

// ---------------------------------------------------------------- fast IQ decode
__device__ __forceinline__ __half2 u2h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ uint32_t h22u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Sign bits q and q+1 of s8 onto the f16 sign bits (15, 31) of a value pair.
__device__ __forceinline__ uint32_t sign_pair(uint32_t s8, int q, uint32_t g) {
    const uint32_t m = s8 * ((1u << (15 - q)) + (1u << (30 - q)));
    return (m & 0x80008000u) ^ g;
}
// n in 0..15 -> (2n + 1, 2n + 1) in f16, exact (from the f16 bits of 1024 + 2n + 1).
__device__ __forceinline__ __half2 odd2(uint32_t n) {
    return __hsub2(u2h2(n * 0x00020002u + 0x64016401u), __floats2half2_rn(1024.f, 1024.f));
}

// IQ2_S: columns 16ss .. 16ss+15 of the thread's 64 (groups 2ss, 2ss+1) of one row as 8 f16
// pairs of exact integers g * sign * (2n + 1). Q = [qs 8 B | signs 8 B], H = [qh 2 B | scales 2 B]
// of the row's 64 columns; tl = this lane's copy of the table.
__device__ __forceinline__ void iq2s_pairs(const uint4& Q, uint32_t H, int ss, const uint8_t* tl, uint32_t* p) {
    const __half2 od = odd2((H >> (16 + 4 * ss)) & 0xFu);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int gi = 2 * ss + h;
        const uint32_t qw = gi < 4 ? Q.x : Q.y, sw = gi < 4 ? Q.z : Q.w;
        const uint32_t b = __byte_perm(qw, 0u, 0x4440 | (gi & 3));
        const uint32_t off = (b << 7) | (((H >> (2 * gi)) & 3u) << 15);
        const uint4 G = *reinterpret_cast<const uint4*>(tl + off);
        const uint32_t s8 = __byte_perm(sw, 0u, 0x4440 | (gi & 3));
        p[4 * h + 0] = h22u(__hmul2(u2h2(sign_pair(s8, 0, G.x)), od));
        p[4 * h + 1] = h22u(__hmul2(u2h2(sign_pair(s8, 2, G.y)), od));
        p[4 * h + 2] = h22u(__hmul2(u2h2(sign_pair(s8, 4, G.z)), od));
        p[4 * h + 3] = h22u(__hmul2(u2h2(sign_pair(s8, 6, G.w)), od));
    }
}

// IQ3_S: the same 16 columns (lookups 4ss .. 4ss+3 of 4 values). Qs = 16 index bytes, S = 64
// sign bits, qh = 16 high index bits, sc = two scale nibbles (per 32 columns).
__device__ __forceinline__ void iq3s_pairs(const uint4& Qs, const uint2& S, uint32_t qh, uint32_t sc, int ss,
                                           const uint8_t* tl, uint32_t* p) {
    const __half2 od = odd2((sc >> (4 * (ss >> 1))) & 0xFu);
#pragma unroll
    for (int h = 0; h < 4; ++h) {
        const int j = 4 * ss + h;
        const uint32_t qw = j < 4 ? Qs.x : j < 8 ? Qs.y : j < 12 ? Qs.z : Qs.w;
        const uint32_t b = __byte_perm(qw, 0u, 0x4440 | (j & 3));
        const uint32_t off = (b << 7) | (((qh >> j) & 1u) << 15);
        const uint2 G = *reinterpret_cast<const uint2*>(tl + off);
        const uint32_t s8 = __byte_perm(j < 8 ? S.x : S.y, 0u, 0x4440 | ((j >> 1) & 3));
        const int q = 4 * (j & 1);
        p[2 * h + 0] = h22u(__hmul2(u2h2(sign_pair(s8, q, G.x)), od));
        p[2 * h + 1] = h22u(__hmul2(u2h2(sign_pair(s8, q + 2, G.y)), od));
    }
}

// IQ2_XXS / IQ3_XXS sign byte from its 7 stored bits (the eighth makes the count even).
__device__ __forceinline__ uint32_t ksigns_d(uint32_t s7) { return s7 | ((__popc(s7) & 1u) << 7); }

// IQ2_XXS: columns 16ss .. 16ss+15 of the thread's 64 as 8 f16 pairs g * sign * (2s + 1). Q =
// [entries | signs/scale] of the 64 columns' two 32-column blocks.
__device__ __forceinline__ void iq2xxs_pairs(const uint4& Q, int ss, const uint8_t* tl, uint32_t* p) {
    const uint32_t qw = ss < 2 ? Q.x : Q.z, aux = ss < 2 ? Q.y : Q.w;
    const __half2 od = odd2(aux >> 28);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int l = 2 * (ss & 1) + h;
        const uint32_t b = __byte_perm(qw, 0u, 0x4440 | l);
        const uint4 G = *reinterpret_cast<const uint4*>(tl + (b << 7));
        const uint32_t s8 = ksigns_d((aux >> (7 * l)) & 127u);
        p[4 * h + 0] = h22u(__hmul2(u2h2(sign_pair(s8, 0, G.x)), od));
        p[4 * h + 1] = h22u(__hmul2(u2h2(sign_pair(s8, 2, G.y)), od));
        p[4 * h + 2] = h22u(__hmul2(u2h2(sign_pair(s8, 4, G.z)), od));
        p[4 * h + 3] = h22u(__hmul2(u2h2(sign_pair(s8, 6, G.w)), od));
    }
}

// IQ3_XXS: the same 16 columns. Q = the 16 grid-entry bytes of the two blocks, A = their
// signs/scale words.
__device__ __forceinline__ void iq3xxs_pairs(const uint4& Q, const uint2& A, int ss, const uint8_t* tl, uint32_t* p) {
    const uint32_t aux = ss < 2 ? A.x : A.y;
    const __half2 od = odd2(aux >> 28);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int l = 2 * (ss & 1) + h;
        const uint32_t w = ss < 2 ? (l < 2 ? Q.x : Q.y) : (l < 2 ? Q.z : Q.w);
        const uint32_t b0 = __byte_perm(w, 0u, 0x4440 | (2 * (l & 1)));
        const uint32_t b1 = __byte_perm(w, 0u, 0x4440 | (2 * (l & 1) + 1));
        const uint2 G0 = *reinterpret_cast<const uint2*>(tl + (b0 << 7));
        const uint2 G1 = *reinterpret_cast<const uint2*>(tl + (b1 << 7));
        const uint32_t s8 = ksigns_d((aux >> (7 * l)) & 127u);
        p[4 * h + 0] = h22u(__hmul2(u2h2(sign_pair(s8, 0, G0.x)), od));
        p[4 * h + 1] = h22u(__hmul2(u2h2(sign_pair(s8, 2, G0.y)), od));
        p[4 * h + 2] = h22u(__hmul2(u2h2(sign_pair(s8, 4, G1.x)), od));
        p[4 * h + 3] = h22u(__hmul2(u2h2(sign_pair(s8, 6, G1.y)), od));
    }
}

// Activation chunks of sub-step ss for this thread's token slot: hi columns 0-7 / 8-15 (and lo;
// a piece's 32 hi chunks come first, then its 32 lo chunks).
// Slots past the pass's tokens read whatever the slot holds: an MMA output column depends only on
// its own activation column, and those columns are never stored, so no branch or zeroing is needed
// (brow always points inside the activation slot).
__device__ __forceinline__ void load_b(const uint8_t* brow, int ss, bool lo, uint32_t* hb, uint32_t* lb) {
    const uint4 h0 = *reinterpret_cast<const uint4*>(brow + 128 * ss);
    const uint4 h1 = *reinterpret_cast<const uint4*>(brow + 128 * ss + 64);
    uint4 l0 = make_uint4(0, 0, 0, 0), l1 = l0;
    if (lo) {
        l0 = *reinterpret_cast<const uint4*>(brow + 512 + 128 * ss);
        l1 = *reinterpret_cast<const uint4*>(brow + 512 + 128 * ss + 64);
    }
    hb[0] = h0.x; hb[1] = h0.y; hb[2] = h0.z; hb[3] = h0.w;
    hb[4] = h1.x; hb[5] = h1.y; hb[6] = h1.z; hb[7] = h1.w;
    lb[0] = l0.x; lb[1] = l0.y; lb[2] = l0.z; lb[3] = l0.w;
    lb[4] = l1.x; lb[5] = l1.y; lb[6] = l1.z; lb[7] = l1.w;
}

// Fast-path inputs of one thread: the rows' index, sign and scale bytes and block scales, copied
// from the weight slot into registers (so, on the early-release path, the slot can go back to the
// producer before the decode and the MMAs run from these registers, the tables and the
// activation slot).
struct FastIn {
    uint4 QA, QB;     // IQ2_S: [qs | signs]; IQ3_S: qs; IQ2_XXS: [entries | signs/scale] x 2;
                      // IQ3_XXS: entries; IQ4_XS: the first 32-column block's nibble bytes
    uint4 QA2, QB2;   // IQ4_XS: the second block's nibble bytes
    uint2 SA, SB;     // IQ3_S: signs; IQ3_XXS: signs/scale words
    uint32_t HA, HB;  // IQ2_S: [qh | scales]; IQ3_S: qh | scales << 16; IQ4_XS: (ls - 32) of the two
                      // blocks as an f16 pair
    float dA, dB;     // block scales of the two rows (times 1/8 for IQ2_S and IQ2_XXS, 1/4 for IQ3_XXS)
};

// IQ4_XS scales (ls - 32) of blocks 2 c4 and 2 c4 + 1 as an f16 pair (exact), from the row's
// [d | scales_h] and scales_l words.
__device__ __forceinline__ uint32_t iq4xs_scales(uint2 m, int c4) {
    const uint32_t sh = m.x >> 16, sl = m.y;
    const int l0 = (int)(((sl >> (8 * c4)) & 15u) | (((sh >> (4 * c4)) & 3u) << 4));
    const int l1 = (int)(((sl >> (8 * c4 + 4)) & 15u) | (((sh >> (4 * c4 + 2)) & 3u) << 4));
    return h22u(__floats2half2_rn((float)(l0 - 32), (float)(l1 - 32)));
}

// IQ4_XS: columns 16ss .. 16ss+15 of the thread's 64 (the low (ss even) or high nibbles of block
// ss / 2's 16 bytes Q) as 8 f16 pairs level * (ls - 32): exact up to 2048 in magnitude (products of
// the largest levels and scales beyond it round to 11 bits). tl = this lane's copy of the pair
// table (nibble pair -> level pair).
__device__ __forceinline__ void iq4xs_pairs(const uint4& Q, __half2 sc, int nh, const uint8_t* tl, uint32_t* p) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint32_t x = w == 0 ? Q.x : w == 1 ? Q.y : w == 2 ? Q.z : Q.w;
        const uint32_t y = (nh ? x >> 4 : x) & 0x0F0F0F0Fu;
        const uint32_t z = y | (y >> 4);  // byte 0: nibbles 0, 1; byte 2: nibbles 2, 3
        const uint32_t v0 = *reinterpret_cast<const uint32_t*>(tl + ((z & 0xFFu) << 7));
        const uint32_t v1 = *reinterpret_cast<const uint32_t*>(tl + (((z >> 16) & 0xFFu) << 7));
        p[2 * w + 0] = h22u(__hmul2(u2h2(v0), sc));
        p[2 * w + 1] = h22u(__hmul2(u2h2(v1), sc));
    }
}

// MXFP4 scales of blocks 2 c4 and 2 c4 + 1 of a row (its 8 scale bytes e in the piece): the f16
// pair (2^(e0 - m), 2^(e1 - m)), m the largest of the 8, and the row's piece scale 2^(m - 128)
// (e8m0 halved, as the reference's e8m0_to_fp32_half). Code value x 2^(e - m) is exact in f16
// down to 2^-24 (codes are at most 12). A bank with a piece whose scales span more than 2^24 is
// marked at creation (cwx_bank::mx_wide) and its launches take the exact path instead.
__device__ __forceinline__ void mx_scales(uint2 e8, int c4, uint32_t* h, float* d) {
    uint32_t m = __vmaxu4(e8.x, e8.y);
    m = __vmaxu4(m, m >> 16);
    m = __vmaxu4(m, m >> 8);
    const int em = (int)(m & 0xFFu);
    const uint32_t w = (c4 < 2 ? e8.x : e8.y) >> (16 * (c4 & 1));
    uint32_t bits[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int k = (int)((w >> (8 * i)) & 0xFFu) - em;
        bits[i] = k >= -14 ? (uint32_t)(k + 15) << 10 : k >= -24 ? 1u << (k + 24) : 0u;
    }
    *h = bits[0] | (bits[1] << 16);
    *d = e8m0_to_f32_half((uint8_t)em);
}

// MXFP4 tail piece (a row's last 64 columns, two GGUF blocks of 17 bytes: e, then 16 nibble
// bytes), stored row after row (prb bytes a row): the fast path's inputs for rows 16 mt + g and
// + 8. The 64 columns are quarter 0; the other quarters' threads get zero weights (the packed
// activation rows hold zeros there too) but the same row scales, because every thread of a quad
// scales its own output columns (picks) of the rows' sums. The two blocks' scales enter as
// 2^(e - m), m the larger, exact in f16 while they are at most 24 apart (the bank is checked for
// it when it is made).
__device__ __forceinline__ void mx_tail_row(const uint8_t* p, uint4* q, uint4* q2, uint32_t* h, float* d) {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        w[i] = (uint32_t)p[1 + 4 * i] | ((uint32_t)p[2 + 4 * i] << 8) | ((uint32_t)p[3 + 4 * i] << 16) |
               ((uint32_t)p[4 + 4 * i] << 24);
        w[4 + i] = (uint32_t)p[18 + 4 * i] | ((uint32_t)p[19 + 4 * i] << 8) | ((uint32_t)p[20 + 4 * i] << 16) |
                   ((uint32_t)p[21 + 4 * i] << 24);
    }
    *q = make_uint4(w[0], w[1], w[2], w[3]);
    *q2 = make_uint4(w[4], w[5], w[6], w[7]);
    const int e0 = p[0], e1 = p[17], m = e0 > e1 ? e0 : e1;
    uint32_t bits[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int k = (i ? e1 : e0) - m;
        bits[i] = k >= -14 ? (uint32_t)(k + 15) << 10 : k >= -24 ? 1u << (k + 24) : 0u;
    }
    *h = bits[0] | (bits[1] << 16);
    *d = e8m0_to_f32_half((uint8_t)m);
}
__device__ __forceinline__ void fast_load_mx_tail(const uint8_t* wsl, int64_t prb, int mt, int g, int c4, FastIn& in) {
    mx_tail_row(wsl + (int64_t)(16 * mt + g) * prb, &in.QA, &in.QA2, &in.HA, &in.dA);
    mx_tail_row(wsl + (int64_t)(16 * mt + g + 8) * prb, &in.QB, &in.QB2, &in.HB, &in.dB);
    if (c4 != 0) in.QA = in.QA2 = in.QB = in.QB2 = make_uint4(0u, 0u, 0u, 0u);
}

template <int FMT>
__device__ __forceinline__ void fast_load(const uint8_t* wsl, int mt, int g, int c4, FastIn& in) {
    if (FMT == F_MXFP4) {
        const uint8_t* grp = wsl + mt * (16 * 136);
        in.QA = *reinterpret_cast<const uint4*>(grp + (g * 4 + c4) * 32);
        in.QA2 = *reinterpret_cast<const uint4*>(grp + (g * 4 + c4) * 32 + 16);
        in.QB = *reinterpret_cast<const uint4*>(grp + ((g + 8) * 4 + c4) * 32);
        in.QB2 = *reinterpret_cast<const uint4*>(grp + ((g + 8) * 4 + c4) * 32 + 16);
        mx_scales(*reinterpret_cast<const uint2*>(grp + 2048 + 8 * g), c4, &in.HA, &in.dA);
        mx_scales(*reinterpret_cast<const uint2*>(grp + 2048 + 8 * (g + 8)), c4, &in.HB, &in.dB);
    } else if (FMT == F_IQ4_XS) {
        const uint8_t* grp = wsl + mt * (16 * 136);
        in.QA = *reinterpret_cast<const uint4*>(grp + (g * 4 + c4) * 32);
        in.QA2 = *reinterpret_cast<const uint4*>(grp + (g * 4 + c4) * 32 + 16);
        in.QB = *reinterpret_cast<const uint4*>(grp + ((g + 8) * 4 + c4) * 32);
        in.QB2 = *reinterpret_cast<const uint4*>(grp + ((g + 8) * 4 + c4) * 32 + 16);
        const uint2 mA = *reinterpret_cast<const uint2*>(grp + 2048 + 8 * g);
        const uint2 mB = *reinterpret_cast<const uint2*>(grp + 2048 + 8 * (g + 8));
        in.HA = iq4xs_scales(mA, c4);
        in.HB = iq4xs_scales(mB, c4);
        in.dA = h2f_bits((uint16_t)(mA.x & 0xFFFFu));
        in.dB = h2f_bits((uint16_t)(mB.x & 0xFFFFu));
    } else if (FMT == F_IQ2_XXS) {
        const uint8_t* grp = wsl + mt * (16 * 66);
        in.QA = *reinterpret_cast<const uint4*>(grp + (g * 4 + c4) * 16);
        in.QB = *reinterpret_cast<const uint4*>(grp + ((g + 8) * 4 + c4) * 16);
        in.dA = __fmul_rn(h2f_bits(*reinterpret_cast<const uint16_t*>(grp + 1024 + 2 * g)), 0.125f);
        in.dB = __fmul_rn(h2f_bits(*reinterpret_cast<const uint16_t*>(grp + 1024 + 2 * (g + 8))), 0.125f);
    } else if (FMT == F_IQ3_XXS) {
        const uint8_t* grp = wsl + mt * (16 * 98);
        in.QA = *reinterpret_cast<const uint4*>(grp + (g * 4 + c4) * 16);
        in.QB = *reinterpret_cast<const uint4*>(grp + ((g + 8) * 4 + c4) * 16);
        in.SA = *reinterpret_cast<const uint2*>(grp + 1024 + (g * 4 + c4) * 8);
        in.SB = *reinterpret_cast<const uint2*>(grp + 1024 + ((g + 8) * 4 + c4) * 8);
        in.dA = __fmul_rn(h2f_bits(*reinterpret_cast<const uint16_t*>(grp + 1536 + 2 * g)), 0.25f);
        in.dB = __fmul_rn(h2f_bits(*reinterpret_cast<const uint16_t*>(grp + 1536 + 2 * (g + 8))), 0.25f);
    } else if (FMT == F_IQ2_S) {
        const uint8_t* grp = wsl + mt * (16 * 82);
        in.QA = *reinterpret_cast<const uint4*>(grp + (g * 4 + c4) * 16);
        in.QB = *reinterpret_cast<const uint4*>(grp + ((g + 8) * 4 + c4) * 16);
        in.HA = *reinterpret_cast<const uint32_t*>(grp + 1024 + (g * 4 + c4) * 4);
        in.HB = *reinterpret_cast<const uint32_t*>(grp + 1024 + ((g + 8) * 4 + c4) * 4);
        in.dA = __fmul_rn(h2f_bits(*reinterpret_cast<const uint16_t*>(grp + 1280 + 2 * g)), 0.125f);
        in.dB = __fmul_rn(h2f_bits(*reinterpret_cast<const uint16_t*>(grp + 1280 + 2 * (g + 8))), 0.125f);
    } else {
        const uint8_t* grp = wsl + mt * (16 * 110);
        in.QA = *reinterpret_cast<const uint4*>(grp + g * 64 + 16 * c4);
        in.QB = *reinterpret_cast<const uint4*>(grp + (g + 8) * 64 + 16 * c4);
        in.SA = *reinterpret_cast<const uint2*>(grp + 1024 + g * 32 + 8 * c4);
        in.SB = *reinterpret_cast<const uint2*>(grp + 1024 + (g + 8) * 32 + 8 * c4);
        in.HA = *reinterpret_cast<const uint16_t*>(grp + 1536 + g * 8 + 2 * c4) | ((uint32_t)grp[1664 + g * 4 + c4] << 16);
        in.HB = *reinterpret_cast<const uint16_t*>(grp + 1536 + (g + 8) * 8 + 2 * c4) |
                ((uint32_t)grp[1664 + (g + 8) * 4 + c4] << 16);
        in.dA = h2f_bits(*reinterpret_cast<const uint16_t*>(grp + 1728 + 2 * g));
        in.dB = h2f_bits(*reinterpret_cast<const uint16_t*>(grp + 1728 + 2 * (g + 8)));
    }
}

// A fast-path step from its inputs: this warp's 16 rows x 256 columns against NT n-tiles of 8
// activation rows (bnt bytes apart), hi activations plus the lo parts when `lo`; the piece's
// partial sums are scaled by the rows' block scales and added to acc[nt * 4 + i].
template <int FMT, int NT>
__device__ __forceinline__ void fast_compute(const FastIn& in, const uint8_t* tl, const uint8_t* brow, int bnt, bool lo,
                                             float* acc) {
    float t[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) t[nt][0] = t[nt][1] = t[nt][2] = t[nt][3] = 0.f;
#pragma unroll
    for (int ss = 0; ss < 4; ++ss) {
        uint32_t pa[8], pb[8];
        if (FMT == F_IQ4_XS || FMT == F_MXFP4) {
            const __half2 sa = ss < 2 ? __low2half2(u2h2(in.HA)) : __high2half2(u2h2(in.HA));
            const __half2 sb = ss < 2 ? __low2half2(u2h2(in.HB)) : __high2half2(u2h2(in.HB));
            iq4xs_pairs(ss < 2 ? in.QA : in.QA2, sa, ss & 1, tl, pa);
            iq4xs_pairs(ss < 2 ? in.QB : in.QB2, sb, ss & 1, tl, pb);
        } else if (FMT == F_IQ2_XXS) {
            iq2xxs_pairs(in.QA, ss, tl, pa);
            iq2xxs_pairs(in.QB, ss, tl, pb);
        } else if (FMT == F_IQ3_XXS) {
            iq3xxs_pairs(in.QA, in.SA, ss, tl, pa);
            iq3xxs_pairs(in.QB, in.SB, ss, tl, pb);
        } else if (FMT == F_IQ2_S) {
            iq2s_pairs(in.QA, in.HA, ss, tl, pa);
            iq2s_pairs(in.QB, in.HB, ss, tl, pb);
        } else {
            iq3s_pairs(in.QA, in.SA, in.HA & 0xFFFFu, in.HA >> 16, ss, tl, pa);
            iq3s_pairs(in.QB, in.SB, in.HB & 0xFFFFu, in.HB >> 16, ss, tl, pb);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            uint32_t hb[8], lb[8];
            load_b(brow + nt * bnt, ss, lo, hb, lb);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint32_t af[4] = {pa[2 * kk], pb[2 * kk], pa[2 * kk + 1], pb[2 * kk + 1]};
                mma_16816(t[nt], af, hb[2 * kk], hb[2 * kk + 1]);
                if (lo) mma_16816(t[nt], af, lb[2 * kk], lb[2 * kk + 1]);
            }
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        acc[nt * 4 + 0] = __fmaf_rn(t[nt][0], in.dA, acc[nt * 4 + 0]);
        acc[nt * 4 + 1] = __fmaf_rn(t[nt][1], in.dA, acc[nt * 4 + 1]);
        acc[nt * 4 + 2] = __fmaf_rn(t[nt][2], in.dB, acc[nt * 4 + 2]);
        acc[nt * 4 + 3] = __fmaf_rn(t[nt][3], in.dB, acc[nt * 4 + 3]);
    }
}

// Q4_K: y = d * sc * q - dmin * m per 32-column sub-block (sub-blocks 2c and 2c+1 are the low
// and high nibbles of the same 32 bytes of 64-column chunk c). Two exact-integer products on the
// tensor cores: A1 = sc * q (<= 945, exact in f16) and A2 = m (constant over a sub-block), both
// against the same activation fragments; per piece acc += d * t1 - dmin * t2 in f32.
struct Q4Row {
    uint4 qlo, qhi;  // the chunk's 32 quant bytes
    float d, dmin;
    uint32_t sc01;   // sc of sub-blocks 2c, 2c+1 as f16 pair halves (sc, sc) in two words
    __half2 s0, s1, m0, m1;
};

// The words of one Q4_K row a thread reads: the row's header (d, dmin, scales) and its chunk's
// 32 quant bytes (loaded ahead of the math by callers that pipeline their loads).
struct Q4Raw {
    uint4 h, qlo, qhi;
};
__device__ __forceinline__ Q4Raw q4_raw(const uint8_t* row, int c4) {
    return Q4Raw{*reinterpret_cast<const uint4*>(row), *reinterpret_cast<const uint4*>(row + 16 + 32 * c4),
                 *reinterpret_cast<const uint4*>(row + 32 + 32 * c4)};
}
__device__ __forceinline__ Q4Row q4_row_of(const Q4Raw& raw, int c4) {
    Q4Row r;
    const uint4 h = raw.h;  // d, dmin, scales[12]
    r.qlo = raw.qlo;
    r.qhi = raw.qhi;
    r.d = h2f_bits((uint16_t)(h.x & 0xFFFF));
    r.dmin = h2f_bits((uint16_t)(h.x >> 16));
    const uint32_t sw[3] = {h.y, h.z, h.w};  // scale bytes 0..11
    auto sb = [&](int i) -> uint32_t { return (sw[i >> 2] >> (8 * (i & 3))) & 0xFFu; };
    uint32_t sc[2], mn[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const int j = 2 * c4 + t;  // get_scale_min_k4 (vendor/candle-core/src/quantized/utils.rs:50)
        if (j < 4) {
            sc[t] = sb(j) & 63u;
            mn[t] = sb(j + 4) & 63u;
        } else {
            sc[t] = (sb(j + 4) & 0xFu) | ((sb(j - 4) >> 6) << 4);
            mn[t] = (sb(j + 4) >> 4) | ((sb(j) >> 6) << 4);
        }
    }
    r.s0 = __floats2half2_rn((float)sc[0], (float)sc[0]);
    r.s1 = __floats2half2_rn((float)sc[1], (float)sc[1]);
    r.m0 = __floats2half2_rn((float)mn[0], (float)mn[0]);
    r.m1 = __floats2half2_rn((float)mn[1], (float)mn[1]);
    return r;
}
__device__ __forceinline__ Q4Row q4_row(const uint8_t* row, int c4) { return q4_row_of(q4_raw(row, c4), c4); }

// Columns 16ss..16ss+15 of the thread's 64 as 8 f16 pairs sc * q.
__device__ __forceinline__ void q4_pairs(const Q4Row& r, int ss, uint32_t* p) {
    const uint4 q = (ss & 1) ? r.qhi : r.qlo;
    const __half2 sc = ss < 2 ? r.s0 : r.s1;
    const __half2 bias = __hmul2(sc, __floats2half2_rn(-1024.f, -1024.f));
    const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
        const uint32_t nib = (ss < 2 ? w4[wi] : (w4[wi] >> 4)) & 0x0F0F0F0Fu;
        // (1024 + q) as f16 from each nibble byte, then (1024 + q) * sc - 1024 * sc = q * sc exactly
        const uint32_t h0 = __byte_perm(nib, 0x64646464u, 0x4140), h1 = __byte_perm(nib, 0x64646464u, 0x4342);
        p[2 * wi] = h22u(__hfma2(u2h2(h0), sc, bias));
        p[2 * wi + 1] = h22u(__hfma2(u2h2(h1), sc, bias));
    }
}

// Activation scales of the thread's two output columns in each n-tile, for Q8_K rows (qi): the
// f32 at byte 512 of the piece in rows dx0 and dx1 (byte offsets from the slot's rows) and
// n-tile nt bnt bytes further.
struct DxAt {
    const uint8_t* p0;
    const uint8_t* p1;
};
__device__ __forceinline__ float dx_of(const DxAt& x, int nt, int bnt, int i) {
    return *reinterpret_cast<const float*>(((i & 1) ? x.p1 : x.p0) + nt * bnt);
}

template <int NT>
__device__ __forceinline__ void q4k_rows(const Q4Row& A, const Q4Row& Bq, const uint8_t* brow, int bnt, bool lo, bool qi,
                                         const DxAt& dx, float* acc);
template <int NT>
__device__ __forceinline__ void q4k_step(const uint8_t* wsl, int mt, int g, int c4, const uint8_t* brow, int bnt, bool lo,
                                         bool qi, const DxAt& dx, float* acc) {
    q4k_rows<NT>(q4_row(wsl + (16 * mt + g) * 144, c4), q4_row(wsl + (16 * mt + g + 8) * 144, c4), brow, bnt, lo,
                 qi, dx, acc);
}

// The two rows (g, g + 8) of a 16-row group of one piece against NT n-tiles of activation rows.
template <int NT>
__device__ __forceinline__ void q4k_rows(const Q4Row& A, const Q4Row& Bq, const uint8_t* brow, int bnt, bool lo, bool qi,
                                         const DxAt& dx, float* acc) {
    float t1[NT][4], t2[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) t1[nt][i] = t2[nt][i] = 0.f;
#pragma unroll
    for (int ss = 0; ss < 4; ++ss) {
        uint32_t pa[8], pb[8];
        q4_pairs(A, ss, pa);
        q4_pairs(Bq, ss, pb);
        const uint32_t ma = h22u(ss < 2 ? A.m0 : A.m1), mb = h22u(ss < 2 ? Bq.m0 : Bq.m1);
        const uint32_t am[4] = {ma, mb, ma, mb};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            uint32_t hb[8], lb[8];
            // Q8_K rows have no lo halves (and are copied without them)
            load_b(brow + nt * bnt, ss, lo && !qi, hb, lb);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint32_t af[4] = {pa[2 * kk], pb[2 * kk], pa[2 * kk + 1], pb[2 * kk + 1]};
                mma_16816(t1[nt], af, hb[2 * kk], hb[2 * kk + 1]);
                mma_16816(t2[nt], am, hb[2 * kk], hb[2 * kk + 1]);
                if (lo && !qi) {
                    mma_16816(t1[nt], af, lb[2 * kk], lb[2 * kk + 1]);
                    mma_16816(t2[nt], am, lb[2 * kk], lb[2 * kk + 1]);
                }
            }
        }
    }
    if (qi) {  // integer codes: the piece's sums times the rows' scales, then the code scale d
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const Q4Row& R = i < 2 ? A : Bq;
                const float r = __fmaf_rn(-t2[nt][i], R.dmin, __fmul_rn(t1[nt][i], R.d));
                acc[nt * 4 + i] = __fmaf_rn(r, dx_of(dx, nt, bnt, i), acc[nt * 4 + i]);
            }
    } else {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            acc[nt * 4 + 0] = __fmaf_rn(-t2[nt][0], A.dmin, __fmaf_rn(t1[nt][0], A.d, acc[nt * 4 + 0]));
            acc[nt * 4 + 1] = __fmaf_rn(-t2[nt][1], A.dmin, __fmaf_rn(t1[nt][1], A.d, acc[nt * 4 + 1]));
            acc[nt * 4 + 2] = __fmaf_rn(-t2[nt][2], Bq.dmin, __fmaf_rn(t1[nt][2], Bq.d, acc[nt * 4 + 2]));
            acc[nt * 4 + 3] = __fmaf_rn(-t2[nt][3], Bq.dmin, __fmaf_rn(t1[nt][3], Bq.d, acc[nt * 4 + 3]));
        }
    }
}

// The packed code words of a grid codebook (nibble-pair tables have none).
template <int FMT>
__device__ __forceinline__ const uint16_t* table_codes() {
    return FMT == F_IQ2_S     ? d_iq2s_codes
           : FMT == F_IQ2_XXS ? d_iq2xxs_codes
           : FMT == F_IQ3_S   ? d_iq3s_codes
           : FMT == F_IQ3_XXS ? d_iq3xxs_codes
                              : nullptr;
}

// One 16-byte chunk of a codebook entry's 128 replicated bytes: the entry's f16 values, repeated
// as often as they fit (8-value tables: once; 4-value tables: twice; nibble-pair tables: 4 times).
template <int FMT>
__device__ __forceinline__ uint4 table_chunk(int e, uint32_t code) {
    if (FMT == F_IQ2_S || FMT == F_IQ2_XXS) {
        const uint64_t v = cwx_iq2s_expand(code);
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            w[j] = h22u(__floats2half2_rn((float)((v >> (16 * j)) & 0xFF), (float)((v >> (16 * j + 8)) & 0xFF)));
        return make_uint4(w[0], w[1], w[2], w[3]);
    } else if (FMT == F_IQ3_S || FMT == F_IQ3_XXS) {
        const uint32_t v = FMT == F_IQ3_S ? cwx_iq3s_expand(code) : cwx_iq3xxs_expand(code);
        const uint32_t lo = h22u(__floats2half2_rn((float)(v & 0xFF), (float)((v >> 8) & 0xFF)));
        const uint32_t hi = h22u(__floats2half2_rn((float)((v >> 16) & 0xFF), (float)(v >> 24)));
        return make_uint4(lo, hi, lo, hi);
    } else {
        // nibble pair -> pair of levels: MXFP4's e2m1 codes times 2 (the reference's kvalues_mxfp4,
        // signed), IQ4_XS's IQ4_NL levels
        const int8_t kv[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
        const uint32_t q = FMT == F_MXFP4 ? h22u(__floats2half2_rn((float)kv[e & 15], (float)kv[e >> 4]))
                                          : h22u(__floats2half2_rn((float)cwx_iq4nl(e & 15), (float)cwx_iq4nl(e >> 4)));
        return make_uint4(q, q, q, q);
    }
}

// Replicated f16 codebooks (threads tid = 0 .. NTH-1 of the block; the caller synchronises them):
// entry e occupies bytes e * 128 .. e * 128 + 127 (see tbl_lane). Each group of 8 threads fills a
// run of consecutive entries: thread c of the group computes every eighth of them (their code
// words all loaded before the first store, one round trip to the code tables) and the group
// passes the chunks round with shuffles, so that thread c stores chunk c of each entry. Every
// store instruction of a warp then writes whole 128-byte lines of shared memory (no bank
// conflicts) and no chunk is computed twice.
template <int FMT, int NTH>
__device__ __forceinline__ void build_tables(uint8_t* tbl, int tid) {
    constexpr int NE = Tbl<FMT>::BYTES / 128, NG = NTH / 8, EPG = NE / NG;
    static_assert(NTH % 32 == 0 && NE % NG == 0, "table build: entries per thread group");
    const int e0 = (tid >> 3) * EPG, c = tid & 7;
    uint8_t* dst = tbl + (int64_t)e0 * 128 + 16 * c;
    constexpr bool grid = FMT == F_IQ2_S || FMT == F_IQ2_XXS || FMT == F_IQ3_S || FMT == F_IQ3_XXS;
    if constexpr (EPG == 0) {
        return;  // formats without a codebook
    } else if constexpr (EPG % 8 == 0) {
        constexpr int R = EPG / 8;  // entries this thread computes: e0 + 8 r + c
        uint32_t code[R];
#pragma unroll
        for (int r = 0; r < R; ++r) code[r] = grid ? table_codes<FMT>()[e0 + 8 * r + c] : 0u;
        const int base = (tid & 31) & ~7;  // the group's first lane
        // (a rolled loop: one copy of the expansion, which runs once per launch)
#pragma unroll 1
        for (int r = 0; r < R; ++r) {
            uint32_t cr = code[0];
#pragma unroll
            for (int q = 1; q < R; ++q) cr = r == q ? code[q] : cr;
            const uint4 v = table_chunk<FMT>(e0 + 8 * r + c, cr);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                uint4 q;
                q.x = __shfl_sync(0xffffffffu, v.x, base + k);
                q.y = __shfl_sync(0xffffffffu, v.y, base + k);
                q.z = __shfl_sync(0xffffffffu, v.z, base + k);
                q.w = __shfl_sync(0xffffffffu, v.w, base + k);
                *reinterpret_cast<uint4*>(dst + 128 * (8 * r + k)) = q;
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < EPG; ++j)
            *reinterpret_cast<uint4*>(dst + 128 * j) = table_chunk<FMT>(e0 + j, grid ? table_codes<FMT>()[e0 + j] : 0u);
    }
}

// One warp packs one 256-column piece of an activation row (act.cu's layout): lane l holds the
// values of columns 8l .. 8l+7 in v (zeros past the row's end); pack_words returns the lane's
// chunk index and its words. Q8_K: the block's codes as exact f16
// integers in the hi chunks and the scale d as an f32 at byte 512 (candle's BlockQ8K::from_float:
// the first of the largest |x|, iscale = -127 / x there, round half away from zero, clamp);
// Q8_0: values rounded through the 32-column blocks' codes (BlockQ8_0::from_float), then split
// like f32 rows; F32: f16 hi + lo parts.
__device__ __forceinline__ int pack_words(int mode, float* v, int lane, uint4* hiw, uint4* low, float* dq) {
    const int k0 = 8 * lane;
    if (mode == AM_Q8_K) {
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
        *hiw = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *low = make_uint4(0u, 0u, 0u, 0u);
        *dq = d;
        return (ss * 2 + q) * 4 + c;
    } else if (mode == AM_Q8_0) {
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
    *hiw = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *low = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *dq = 0.f;
    return (ss * 2 + q) * 4 + c;
}

// The piece's words stored in the packed layout: hi chunks, then lo chunks (Q8_K: the scale d as
// an f32 at byte 512, the rest of the lo half zero).
__device__ __forceinline__ void pack_piece(int mode, float* v, uint8_t* piece, int lane) {
    uint4 hi, lo;
    float d;
    const int ch = pack_words(mode, v, lane, &hi, &lo, &d);
    *reinterpret_cast<uint4*>(piece + 16 * ch) = hi;
    *reinterpret_cast<uint4*>(piece + 512 + 16 * ch) =
        mode == AM_Q8_K ? make_uint4(ch == 0 ? __float_as_uint(d) : 0u, 0u, 0u, 0u) : lo;
}

// ---------------------------------------------------------------- RMSNorm of a row (act.cu, decode_layer.cu)
constexpr int NORM_THREADS = 256;

// (NTH threads; a block larger than NORM_THREADS sums the same warp partials in the same order,
// the extra warps contributing zeros)
template <int NTH = NORM_THREADS>
__device__ __forceinline__ double norm_block_sum(double v, double* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    double s = red[0];
#pragma unroll
    for (int w = 1; w < NTH / 32; ++w) s += red[w];
    return s;
}

__device__ __forceinline__ double sq4(float4 v) {
    double s = (double)v.x * (double)v.x;
    s += (double)v.y * (double)v.y;
    s += (double)v.z * (double)v.z;
    s += (double)v.w * (double)v.w;
    return s;
}

// Second pass over a summed row: out = v / m * alpha (ss: this thread's share of the sum of squares).
template <int NTH = NORM_THREADS>
__device__ __forceinline__ void norm_row(double ss, const float* __restrict__ sum, const float* __restrict__ alpha,
                                         float eps, int H, bool vec, float* __restrict__ out) {
    __shared__ double red[NTH / 32];
    const double tot = norm_block_sum<NTH>(ss, red);
    const float m = __fsqrt_rn(__fadd_rn(__fdiv_rn((float)tot, (float)H), eps));
    const int nq = (H + 3) / 4;
    for (int q = threadIdx.x; q < nq; q += NTH) {
        if (vec) {
            const float4 v = *reinterpret_cast<const float4*>(sum + 4 * q);
            const float4 al = __ldg(reinterpret_cast<const float4*>(alpha) + q);
            float4 r;
            r.x = __fmul_rn(__fdiv_rn(v.x, m), al.x);
            r.y = __fmul_rn(__fdiv_rn(v.y, m), al.y);
            r.z = __fmul_rn(__fdiv_rn(v.z, m), al.z);
            r.w = __fmul_rn(__fdiv_rn(v.w, m), al.w);
            *reinterpret_cast<float4*>(out + 4 * q) = r;
        } else {
            for (int j = 0; j < 4 && 4 * q + j < H; ++j)
                out[4 * q + j] = __fmul_rn(__fdiv_rn(sum[4 * q + j], m), __ldg(alpha + 4 * q + j));
        }
    }
}

// (a, b or c may be the sum buffer itself: each element is read before the same thread writes it)

}  // namespace cwx
