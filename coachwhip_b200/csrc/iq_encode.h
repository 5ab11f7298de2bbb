// IQ2_S / IQ3_S block encoders for the synthetic banks, host and device.
//
// The reference ships no quantiser for these formats (its CPU code panics for IQ types and
// its GPU code only decodes them), so this encoder is this project's own: per sub-block scale
// from the absolute maximum, each value's magnitude rounded to the nearest codebook level,
// then the group of levels mapped to the nearest codebook entry (exact integer L2 distance in
// value space, lowest index on ties) through a precomputed map, signs stored bitwise. Only the
// validity of the bytes matters for parity: kernels and oracle decode the same bytes.
//
// Block layouts (GGUF, 256 weights):
//   IQ3_S (110 B): f16 d | qs[64] | qh[8] | signs[32] | scales[4]
//     element e = 32*ib + 4*g + j: entry = qs[8ib+g] | ((qh[ib] >> g) & 1) << 8,
//     value = d*(1+2*scale_ib) * grid[entry].byte[j] * (signs bit e ? -1 : 1)
//   IQ2_S (82 B): f16 d | qs[32] | signs[32] | qh[8] | scales[8]
//     element e = 32*ib + 8*g + j: entry = qs[4ib+g] | ((qh[ib] >> 2g) & 3) << 8,
//     value = d*(0.5+scale_{ib,g/2})*0.25 * grid[entry].byte[j] * (signs[4ib+g] bit j ? -1 : 1)
#pragma once
#include <stdint.h>

#include "iq_grids.h"
#include "synth_math.h"

#define CWX_IQ3S_MAP_SIZE 4096  // 8 levels ^ 4 values
#define CWX_IQ2S_MAP_SIZE 6561  // 3 levels ^ 8 values

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
