// IQ block encoders for the synthetic banks (IQ2_S, IQ3_S, IQ2_XXS, IQ3_XXS, IQ4_XS), host and
// device.
//
// The reference ships no quantiser for these formats (its CPU code panics for IQ types and
// its GPU code only decodes them), so this encoder is this project's own: per sub-block scale
// from the absolute maximum, each value's magnitude rounded to the nearest codebook level,
// then the group of levels mapped to the nearest codebook entry (exact integer L2 distance in
// value space, lowest index on ties) through a precomputed map, signs stored bitwise. Only the
// validity of the bytes matters for parity: kernels and oracle decode the same bytes.
// IQ2_XXS / IQ3_XXS store 7 signs per 8 values (the eighth makes the count of negatives even):
// when a group's count is odd, the sign of its smallest magnitude (lowest index on ties) flips.
// IQ4_XS takes each value's nearest of the 16 IQ4_NL levels (lowest index on ties).
//
// Block layouts (GGUF, 256 weights):
//   IQ3_S (110 B): f16 d | qs[64] | qh[8] | signs[32] | scales[4]
//     element e = 32*ib + 4*g + j: entry = qs[8ib+g] | ((qh[ib] >> g) & 1) << 8,
//     value = d*(1+2*scale_ib) * grid[entry].byte[j] * (signs bit e ? -1 : 1)
//   IQ2_S (82 B): f16 d | qs[32] | signs[32] | qh[8] | scales[8]
//     element e = 32*ib + 8*g + j: entry = qs[4ib+g] | ((qh[ib] >> 2g) & 3) << 8,
//     value = d*(0.5+scale_{ib,g/2})*0.25 * grid[entry].byte[j] * (signs[4ib+g] bit j ? -1 : 1)
//   IQ2_XXS (66 B): f16 d | per ib (8 B): entries[4] | aux u32 (signs of group g at bits 7g..7g+6,
//     scale at bits 28..31); element e = 32*ib + 8*g + j:
//     value = d*(0.5+scale)*0.25 * grid[entries[g]].byte[j] * (ksigns(aux >> 7g & 127) bit j ? -1 : 1)
//   IQ3_XXS (98 B): f16 d | entries[64] | aux u32[8] (as IQ2_XXS); element e = 32*ib + 8*g + j:
//     value = d*(0.5+scale)*0.5 * grid[entries[8ib + 2g + j/4]].byte[j%4] * (ksigns bit j ? -1 : 1)
//   IQ4_XS (136 B): f16 d | scales_h u16 | scales_l[4] | qs[128]; ls_ib = 6 bits (low 4 in
//     scales_l[ib/2] nibble ib%2, high 2 at scales_h bits 2ib); element e = 32*ib + 16*h + m:
//     value = d*(ls_ib - 32) * levels[(qs[16ib + m] >> 4h) & 15]
#pragma once
#include <stdint.h>

#include "iq_grids.h"
#include "synth_math.h"

#define CWX_IQ3S_MAP_SIZE 4096  // 8 levels ^ 4 values
#define CWX_IQ2S_MAP_SIZE 6561  // 3 levels ^ 8 values
#define CWX_IQ3XXS_MAP_SIZE 4096
#define CWX_IQ2XXS_MAP_SIZE 6561

// Map from a group of per-value levels to the nearest IQ3_S codebook entry.
static inline void cwx_build_iq3s_map(uint16_t* map) {
    for (int c = 0; c < CWX_IQ3S_MAP_SIZE; ++c) {
        int want[4];
        for (int j = 0; j < 4; ++j) want[j] = 2 * ((c >> (3 * j)) & 7) + 1;
        int best = 0;
        long bestd = -1;
        for (int e = 0; e < 512; ++e) {
            uint32_t g = cwx_iq3s_expand(cwx_iq3s_codes[e]);
            long d = 0;
            for (int j = 0; j < 4; ++j) {
                long t = (long)((g >> (8 * j)) & 0xFF) - want[j];
                d += t * t;
            }
            if (bestd < 0 || d < bestd) {
                bestd = d;
                best = e;
            }
        }
        map[c] = (uint16_t)best;
    }
}

// Map from a group of per-value levels (base 3) to the nearest IQ2_S codebook entry.
static inline void cwx_build_iq2s_map(uint16_t* map) {
    static const int lv[3] = {0x08, 0x19, 0x2B};
    for (int c = 0; c < CWX_IQ2S_MAP_SIZE; ++c) {
        int want[8];
        int r = c;
        for (int j = 0; j < 8; ++j) {
            want[j] = lv[r % 3];
            r /= 3;
        }
        int best = 0;
        long bestd = -1;
        for (int e = 0; e < 1024; ++e) {
            uint64_t g = cwx_iq2s_expand(cwx_iq2s_codes[e]);
            long d = 0;
            for (int j = 0; j < 8; ++j) {
                long t = (long)((g >> (8 * j)) & 0xFF) - want[j];
                d += t * t;
            }
            if (bestd < 0 || d < bestd) {
                bestd = d;
                best = e;
            }
        }
        map[c] = (uint16_t)best;
    }
}

// Maps from groups of levels to the nearest IQ2_XXS (base 3, 8 values) and IQ3_XXS (base 8,
// 4 values; levels 4, 12, ..., 52, 62) codebook entries.
static inline void cwx_build_iq2xxs_map(uint16_t* map) {
    static const int lv[3] = {0x08, 0x19, 0x2B};
    for (int c = 0; c < CWX_IQ2XXS_MAP_SIZE; ++c) {
        int want[8];
        int r = c;
        for (int j = 0; j < 8; ++j) {
            want[j] = lv[r % 3];
            r /= 3;
        }
        int best = 0;
        long bestd = -1;
        for (int e = 0; e < 256; ++e) {
            uint64_t g = cwx_iq2s_expand(cwx_iq2xxs_codes[e]);
            long d = 0;
            for (int j = 0; j < 8; ++j) {
                long t = (long)((g >> (8 * j)) & 0xFF) - want[j];
                d += t * t;
            }
            if (bestd < 0 || d < bestd) {
                bestd = d;
                best = e;
            }
        }
        map[c] = (uint16_t)best;
    }
}

static inline void cwx_build_iq3xxs_map(uint16_t* map) {
    for (int c = 0; c < CWX_IQ3XXS_MAP_SIZE; ++c) {
        int want[4];
        for (int j = 0; j < 4; ++j) {
            const int l = (c >> (3 * j)) & 7;
            want[j] = l == 7 ? 62 : 8 * l + 4;
        }
        int best = 0;
        long bestd = -1;
        for (int e = 0; e < 256; ++e) {
            uint32_t g = cwx_iq3xxs_expand(cwx_iq3xxs_codes[e]);
            long d = 0;
            for (int j = 0; j < 4; ++j) {
                long t = (long)((g >> (8 * j)) & 0xFF) - want[j];
                d += t * t;
            }
            if (bestd < 0 || d < bestd) {
                bestd = d;
                best = e;
            }
        }
        map[c] = (uint16_t)best;
    }
}

CWX_SHD float cwx_absf(float x) { return cwx_u2f(cwx_f2u(x) & 0x7FFFFFFFu); }

// round half away from zero (Rust f32::round), as an int; x must be finite and small.
CWX_SHD int cwx_round_int(float x) {
    float a = cwx_absf(x);
    int i = (int)a;  // truncation
    if (CWX_FSUB(a, (float)i) >= 0.5f) i += 1;
    return x < 0.0f ? -i : i;
}

// One IQ3_S block from 256 floats.
CWX_SHD void cwx_encode_iq3s(const float* x, uint8_t* blk, const uint16_t* map) {
    float dli[8];
    float dmax = 0.0f;
    for (int ib = 0; ib < 8; ++ib) {
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) {
            float a = cwx_absf(x[32 * ib + i]);
            if (a > amax) amax = a;
        }
        dli[ib] = CWX_FDIV(amax, 15.0f);
        if (dli[ib] > dmax) dmax = dli[ib];
    }
    for (int i = 0; i < 110; ++i) blk[i] = 0;
    uint16_t dh = cwx_f32_to_f16_bits(CWX_FDIV(dmax, 31.0f));
    float d = cwx_f16_bits_to_f32(dh);
    blk[0] = (uint8_t)(dh & 0xFF);
    blk[1] = (uint8_t)(dh >> 8);
    if (!(d > 0.0f)) return;  // all-zero block: entry 0 with scale 0 is never read as nonzero
    uint8_t* qs = blk + 2;
    uint8_t* qh = blk + 66;
    uint8_t* signs = blk + 74;
    uint8_t* scales = blk + 106;
    for (int ib = 0; ib < 8; ++ib) {
        int s = cwx_round_int(CWX_FDIV(CWX_FSUB(CWX_FDIV(dli[ib], d), 1.0f), 2.0f));
        s = s < 0 ? 0 : (s > 15 ? 15 : s);
        scales[ib / 2] |= (uint8_t)(s << (4 * (ib % 2)));
        float dl = CWX_FMUL(d, (float)(1 + 2 * s));
        for (int g = 0; g < 8; ++g) {
            int code = 0;
            for (int j = 0; j < 4; ++j) {
                int e = 32 * ib + 4 * g + j;
                float v = x[e];
                int l = cwx_round_int(CWX_FDIV(CWX_FSUB(CWX_FDIV(cwx_absf(v), dl), 1.0f), 2.0f));
                l = l < 0 ? 0 : (l > 7 ? 7 : l);
                code |= l << (3 * j);
                if (v < 0.0f) signs[e / 8] |= (uint8_t)(1u << (e % 8));
            }
            int entry = map[code];
            qs[8 * ib + g] = (uint8_t)(entry & 0xFF);
            qh[ib] |= (uint8_t)(((entry >> 8) & 1) << g);
        }
    }
}

// One IQ2_S block from 256 floats.
CWX_SHD void cwx_encode_iq2s(const float* x, uint8_t* blk, const uint16_t* map) {
    float dli[16];
    float dmax = 0.0f;
    for (int h = 0; h < 16; ++h) {
        float amax = 0.0f;
        for (int i = 0; i < 16; ++i) {
            float a = cwx_absf(x[16 * h + i]);
            if (a > amax) amax = a;
        }
        dli[h] = CWX_FDIV(amax, 43.0f);
        if (dli[h] > dmax) dmax = dli[h];
    }
    for (int i = 0; i < 82; ++i) blk[i] = 0;
    uint16_t dh = cwx_f32_to_f16_bits(CWX_FDIV(dmax, 3.875f));
    float d = cwx_f16_bits_to_f32(dh);
    blk[0] = (uint8_t)(dh & 0xFF);
    blk[1] = (uint8_t)(dh >> 8);
    if (!(d > 0.0f)) return;
    uint8_t* qs = blk + 2;
    uint8_t* signs = blk + 34;
    uint8_t* qh = blk + 66;
    uint8_t* scales = blk + 74;
    float dq = CWX_FMUL(d, 0.25f);
    for (int h = 0; h < 16; ++h) {
        int ib = h / 2;
        int s = cwx_round_int(CWX_FSUB(CWX_FDIV(dli[h], dq), 0.5f));
        s = s < 0 ? 0 : (s > 15 ? 15 : s);
        scales[ib] |= (uint8_t)(s << (4 * (h % 2)));
        float dl = CWX_FMUL(CWX_FMUL(d, CWX_FADD(0.5f, (float)s)), 0.25f);
        for (int gg = 0; gg < 2; ++gg) {
            int g = 2 * (h % 2) + gg;
            int code = 0, mul = 1;
            uint8_t sb = 0;
            for (int j = 0; j < 8; ++j) {
                int e = 32 * ib + 8 * g + j;
                float v = x[e];
                float q = CWX_FDIV(cwx_absf(v), dl);
                int l = q < 16.5f ? 0 : (q < 34.0f ? 1 : 2);
                code += l * mul;
                mul *= 3;
                if (v < 0.0f) sb |= (uint8_t)(1u << j);
            }
            int entry = map[code];
            qs[4 * ib + g] = (uint8_t)(entry & 0xFF);
            qh[ib] |= (uint8_t)(((entry >> 8) & 3) << (2 * g));
            signs[4 * ib + g] = sb;
        }
    }
}

// Sign bits of 8 values with an even count of negatives: when odd, the smallest magnitude's flips.
CWX_SHD uint32_t cwx_even_signs(const float* v) {
    uint32_t sb = 0;
    int m = 0;
    float amin = cwx_absf(v[0]);
    for (int j = 0; j < 8; ++j) {
        if (v[j] < 0.0f) sb |= 1u << j;
        const float a = cwx_absf(v[j]);
        if (a < amin) {
            amin = a;
            m = j;
        }
    }
    if (cwx_ksigns(sb & 127u) != sb) sb ^= 1u << m;
    return sb;
}

// One IQ2_XXS block from 256 floats.
CWX_SHD void cwx_encode_iq2xxs(const float* x, uint8_t* blk, const uint16_t* map) {
    float dli[8];
    float dmax = 0.0f;
    for (int ib = 0; ib < 8; ++ib) {
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) {
            float a = cwx_absf(x[32 * ib + i]);
            if (a > amax) amax = a;
        }
        dli[ib] = CWX_FDIV(amax, 43.0f);
        if (dli[ib] > dmax) dmax = dli[ib];
    }
    for (int i = 0; i < 66; ++i) blk[i] = 0;
    uint16_t dh = cwx_f32_to_f16_bits(CWX_FDIV(dmax, 3.875f));
    float d = cwx_f16_bits_to_f32(dh);
    blk[0] = (uint8_t)(dh & 0xFF);
    blk[1] = (uint8_t)(dh >> 8);
    if (!(d > 0.0f)) return;
    float dq = CWX_FMUL(d, 0.25f);
    for (int ib = 0; ib < 8; ++ib) {
        int s = cwx_round_int(CWX_FSUB(CWX_FDIV(dli[ib], dq), 0.5f));
        s = s < 0 ? 0 : (s > 15 ? 15 : s);
        float dl = CWX_FMUL(CWX_FMUL(d, CWX_FADD(0.5f, (float)s)), 0.25f);
        uint32_t aux = (uint32_t)s << 28;
        uint8_t* q = blk + 2 + 8 * ib;
        for (int g = 0; g < 4; ++g) {
            const float* v = x + 32 * ib + 8 * g;
            int code = 0, mul = 1;
            for (int j = 0; j < 8; ++j) {
                float t = CWX_FDIV(cwx_absf(v[j]), dl);
                int l = t < 16.5f ? 0 : (t < 34.0f ? 1 : 2);
                code += l * mul;
                mul *= 3;
            }
            q[g] = (uint8_t)map[code];
            aux |= (cwx_even_signs(v) & 127u) << (7 * g);
        }
        for (int b = 0; b < 4; ++b) q[4 + b] = (uint8_t)(aux >> (8 * b));
    }
}

// One IQ3_XXS block from 256 floats.
CWX_SHD void cwx_encode_iq3xxs(const float* x, uint8_t* blk, const uint16_t* map) {
    float dli[8];
    float dmax = 0.0f;
    for (int ib = 0; ib < 8; ++ib) {
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) {
            float a = cwx_absf(x[32 * ib + i]);
            if (a > amax) amax = a;
        }
        dli[ib] = CWX_FDIV(amax, 62.0f);
        if (dli[ib] > dmax) dmax = dli[ib];
    }
    for (int i = 0; i < 98; ++i) blk[i] = 0;
    uint16_t dh = cwx_f32_to_f16_bits(CWX_FDIV(dmax, 7.75f));
    float d = cwx_f16_bits_to_f32(dh);
    blk[0] = (uint8_t)(dh & 0xFF);
    blk[1] = (uint8_t)(dh >> 8);
    if (!(d > 0.0f)) return;
    float dq = CWX_FMUL(d, 0.5f);
    for (int ib = 0; ib < 8; ++ib) {
        int s = cwx_round_int(CWX_FSUB(CWX_FDIV(dli[ib], dq), 0.5f));
        s = s < 0 ? 0 : (s > 15 ? 15 : s);
        float dl = CWX_FMUL(CWX_FMUL(d, CWX_FADD(0.5f, (float)s)), 0.5f);
        uint32_t aux = (uint32_t)s << 28;
        for (int g = 0; g < 4; ++g) {
            const float* v = x + 32 * ib + 8 * g;
            for (int h = 0; h < 2; ++h) {
                int code = 0;
                for (int j = 0; j < 4; ++j) {
                    int l = cwx_round_int(CWX_FDIV(CWX_FSUB(CWX_FDIV(cwx_absf(v[4 * h + j]), dl), 4.0f), 8.0f));
                    l = l < 0 ? 0 : (l > 7 ? 7 : l);
                    code |= l << (3 * j);
                }
                blk[2 + 8 * ib + 2 * g + h] = (uint8_t)map[code];
            }
            aux |= (cwx_even_signs(v) & 127u) << (7 * g);
        }
        for (int b = 0; b < 4; ++b) blk[66 + 4 * ib + b] = (uint8_t)(aux >> (8 * b));
    }
}

// One IQ4_XS block from 256 floats.
CWX_SHD void cwx_encode_iq4xs(const float* x, uint8_t* blk) {
    float dli[8];
    float dmax = 0.0f;
    for (int ib = 0; ib < 8; ++ib) {
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) {
            float a = cwx_absf(x[32 * ib + i]);
            if (a > amax) amax = a;
        }
        dli[ib] = CWX_FDIV(amax, 127.0f);
        if (dli[ib] > dmax) dmax = dli[ib];
    }
    for (int i = 0; i < 136; ++i) blk[i] = 0;
    uint16_t dh = cwx_f32_to_f16_bits(CWX_FDIV(dmax, 31.0f));
    float d = cwx_f16_bits_to_f32(dh);
    blk[0] = (uint8_t)(dh & 0xFF);
    blk[1] = (uint8_t)(dh >> 8);
    uint32_t sh = 0;
    for (int ib = 0; ib < 8; ++ib) {
        int s = d > 0.0f ? cwx_round_int(CWX_FDIV(dli[ib], d)) : 0;
        s = s < 0 ? 0 : (s > 31 ? 31 : s);
        const int ls = s + 32;
        blk[4 + ib / 2] |= (uint8_t)((ls & 15) << (4 * (ib % 2)));
        sh |= (uint32_t)(ls >> 4) << (2 * ib);
        const float dl = CWX_FMUL(d, (float)s);
        for (int i = 0; i < 32; ++i) {
            int best = 8;
            if (dl > 0.0f) {
                const float t = CWX_FDIV(x[32 * ib + i], dl);
                float bd = -1.0f;
                for (int q = 0; q < 16; ++q) {
                    const float e = cwx_absf(CWX_FSUB(t, (float)cwx_iq4nl(q)));
                    if (bd < 0.0f || e < bd) {
                        bd = e;
                        best = q;
                    }
                }
            }
            blk[8 + 16 * ib + (i & 15)] |= (uint8_t)(best << (4 * (i >> 4)));
        }
    }
    blk[2] = (uint8_t)(sh & 0xFF);
    blk[3] = (uint8_t)(sh >> 8);
}
