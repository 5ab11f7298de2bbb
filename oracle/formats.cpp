// Oracle: GGUF block formats -- TEST INFRASTRUCTURE ONLY (see cw_oracle.h).
//
// Restates, operation for operation, the candle CPU code for each format:
//   Q4_K  to_float k_quants.rs:1821-1848, from_float 1694-1753, vec_dot_unopt 1612-1692
//   Q6_K  to_float k_quants.rs:2420-2451, from_float 2267-2337, vec_dot_unopt 2208-2265
//   Q8_0  to_float k_quants.rs:766-782,   from_float 784-820 (x86 path), vec_dot_unopt 855-873
//   Q8_K  from_float k_quants.rs:2495-2534, to_float 2536-2547
//   MXFP4 to_float k_quants.rs:673-691, from_float 694-731, vec_dot_unopt 738-758,
//         e8m0_to_f32_half 642-649, KVALUES_MXFP4 638
//   helpers utils.rs: nearest_int 1-3, get_scale_min_k4 50-60, make_qx_quants 62-218,
//         make_qkx1_quants 227-284
// and the Metal shader dequantisers for the IQ formats, which have no CPU code in the
// reference:
//   IQ3_S dequantize_iq3_s quantized.metal:6892-6915, IQ2_S dequantize_iq2_s :6917-6934,
//   IQ2_XXS :6819-6842, IQ3_XXS :6862-6890, IQ4_XS :6999-7018.
// Compiled with -ffp-contract=off so every f32 operation rounds where the Rust code does.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "cw_oracle.h"
#include "iq_encode.h"
#include "oracle_internal.h"

namespace cwo {

static const int8_t KVALUES_MXFP4[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

static inline float f16_to_f32(uint16_t h) { return cwx_f16_bits_to_f32(h); }
static inline uint16_t f32_to_f16(float f) { return cwx_f32_to_f16_bits(f); }
static inline int nearest_int(float v) { return (int)roundf(v); }  // f32::round: half away from zero

static inline void get_scale_min_k4(int j, const uint8_t* q, uint8_t* d, uint8_t* m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

static float e8m0_to_f32_half(uint8_t e) {
    uint32_t bits = e < 2 ? (0x00200000u << e) : ((uint32_t)(e - 1) << 23);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

// ---------------------------------------------------------------- Q8_K / Q8_0 (activations)

void q8k_from_float(const float* x, BQ8K* y) {
    float max = 0.f, amax = 0.f;
    for (int i = 0; i < 256; ++i) {
        float a = fabsf(x[i]);
        if (amax < a) {
            amax = a;
            max = x[i];
        }
    }
    if (amax == 0.f) {
        memset(y, 0, sizeof(*y));
        return;
    }
    float iscale = -127.f / max;
    for (int j = 0; j < 256; ++j) {
        float v = roundf(iscale * x[j]);
        v = v < -128.f ? -128.f : (v > 127.f ? 127.f : v);
        y->qs[j] = (int8_t)v;
    }
    for (int j = 0; j < 16; ++j) {
        int s = 0;
        for (int ii = 0; ii < 16; ++ii) s += y->qs[j * 16 + ii];
        y->bsums[j] = (int16_t)s;
    }
    y->d = 1.0f / iscale;
}

void q8_0_from_float(const float* x, BQ8_0* y) {
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    float d = amax / 127.f;
    float id = d != 0.f ? 1.f / d : 0.f;
    y->d = f32_to_f16(d);
    for (int i = 0; i < 32; ++i) {
        float v = roundf(x[i] * id);
        v = v < -128.f ? -128.f : (v > 127.f ? 127.f : v);  // `as i8` saturates
        y->qs[i] = (int8_t)v;
    }
}

// ---------------------------------------------------------------- Q4_K

static void make_qkx1_quants(int nmax, int ntry, const float* x, float* scale_out, float* min_out) {
    const int n = 32;
    uint8_t L[32] = {0};
    float mn = x[0], mx = x[0];
    for (int i = 1; i < n; ++i) {  // min_by / max_by with total_cmp: first minimum, last maximum
        if (x[i] < mn) mn = x[i];
        if (x[i] >= mx) mx = x[i];
    }
    if (mx == mn) {
        *scale_out = 0.f;
        *min_out = 0.f;
        return;
    }
    if (mn > 0.f) mn = 0.f;
    float iscale = (float)nmax / (mx - mn);
    float scale = 1.0f / iscale;
    for (int t = 0; t < ntry; ++t) {
        float sumlx = 0.f;
        int suml2 = 0;
        bool did_change = false;
        for (int i = 0; i < n; ++i) {
            int li = nearest_int(iscale * (x[i] - mn));
            li = li < 0 ? 0 : (li > nmax ? nmax : li);
            if ((uint8_t)li != L[i]) {
                L[i] = (uint8_t)li;
                did_change = true;
            }
            sumlx += (x[i] - mn) * (float)li;
            suml2 += li * li;
        }
        scale = sumlx / (float)suml2;
        float sum = 0.f;
        for (int i = 0; i < n; ++i) sum += x[i] - scale * (float)L[i];
        mn = sum / (float)n;
        if (mn > 0.f) mn = 0.f;
        iscale = 1.0f / scale;
        if (!did_change) break;
    }
    *scale_out = scale;
    *min_out = -mn;
}

void q4k_from_float(const float* x, BQ4K* b) {
    float mins[8], scales[8];
    for (int j = 0; j < 8; ++j) make_qkx1_quants(15, 5, x + 32 * j, &scales[j], &mins[j]);
    float max_scale = 0.f, max_min = 0.f;
    for (int j = 0; j < 8; ++j) {
        max_scale = fmaxf(scales[j], max_scale);
        max_min = fmaxf(mins[j], max_min);
    }
    float inv_scale = max_scale > 0.f ? 63.f / max_scale : 0.f;
    float inv_min = max_min > 0.f ? 63.f / max_min : 0.f;
    memset(b->scales, 0, 12);
    for (int j = 0; j < 8; ++j) {
        int lsi = nearest_int(inv_scale * scales[j]);
        int lmi = nearest_int(inv_min * mins[j]);
        uint8_t ls = (uint8_t)(lsi < 63 ? lsi : 63);
        uint8_t lm = (uint8_t)(lmi < 63 ? lmi : 63);
        if (j < 4) {
            b->scales[j] = ls;
            b->scales[j + 4] = lm;
        } else {
            b->scales[j + 4] = (uint8_t)((ls & 0xF) | ((lm & 0xF) << 4));
            b->scales[j - 4] |= (uint8_t)((ls >> 4) << 6);
            b->scales[j] |= (uint8_t)((lm >> 4) << 6);
        }
    }
    b->d = f32_to_f16(max_scale / 63.f);
    b->dmin = f32_to_f16(max_min / 63.f);
    uint8_t L[256] = {0};
    for (int j = 0; j < 8; ++j) {
        uint8_t sc, m;
        get_scale_min_k4(j, b->scales, &sc, &m);
        float d = f16_to_f32(b->d) * (float)sc;
        if (d != 0.f) {
            float dm = f16_to_f32(b->dmin) * (float)m;
            for (int ii = 0; ii < 32; ++ii) {
                int l = nearest_int((x[32 * j + ii] + dm) / d);
                L[32 * j + ii] = (uint8_t)(l < 0 ? 0 : (l > 15 ? 15 : l));
            }
        }
    }
    for (int j = 0; j < 256; j += 64)
        for (int l = 0; l < 32; ++l) b->qs[(j / 64) * 32 + l] = (uint8_t)(L[j + l] | (L[j + l + 32] << 4));
}

void q4k_to_float(const BQ4K* b, float* y) {
    float d = f16_to_f32(b->d), mn = f16_to_f32(b->dmin);
    int is = 0;
    for (int j = 0; j < 256; j += 64) {
        const uint8_t* q = b->qs + j / 2;
        uint8_t sc, m;
        get_scale_min_k4(is, b->scales, &sc, &m);
        float d1 = d * (float)sc, m1 = mn * (float)m;
        get_scale_min_k4(is + 1, b->scales, &sc, &m);
        float d2 = d * (float)sc, m2 = mn * (float)m;
        for (int l = 0; l < 32; ++l) *y++ = d1 * (float)(q[l] & 0xF) - m1;
        for (int l = 0; l < 32; ++l) *y++ = d2 * (float)(q[l] >> 4) - m2;
        is += 2;
    }
}

float q4k_vec_dot(int64_t n, const BQ4K* xs, const BQ8K* ys) {
    float sums[8] = {0};
    float sumf = 0.f;
    int8_t aux8[256];
    for (int64_t bi = 0; bi < n / 256; ++bi) {
        const BQ4K* x = xs + bi;
        const BQ8K* y = ys + bi;
        for (int c = 0; c < 4; ++c) {
            for (int l = 0; l < 32; ++l) aux8[64 * c + l] = (int8_t)(x->qs[32 * c + l] & 0xF);
            for (int l = 0; l < 32; ++l) aux8[64 * c + 32 + l] = (int8_t)(x->qs[32 * c + l] >> 4);
        }
        uint8_t scales[8], mins[8];
        for (int j = 0; j < 8; ++j) get_scale_min_k4(j, x->scales, &scales[j], &mins[j]);
        int sumi = 0;
        for (int j = 0; j < 16; ++j) sumi += (int)y->bsums[j] * (int)mins[j / 2];
        int32_t aux32[8] = {0};
        const int8_t* q8 = y->qs;
        const int8_t* a = aux8;
        for (int s = 0; s < 8; ++s) {
            int scale = scales[s];
            for (int r = 0; r < 4; ++r) {
                for (int l = 0; l < 8; ++l) aux32[l] += scale * (int)(int16_t)(q8[l] * a[l]);
                q8 += 8;
                a += 8;
            }
        }
        float d = f16_to_f32(x->d) * y->d;
        for (int l = 0; l < 8; ++l) sums[l] += d * (float)aux32[l];
        float dmin = f16_to_f32(x->dmin) * y->d;
        sumf -= dmin * (float)sumi;
    }
    float t = 0.f;
    for (int l = 0; l < 8; ++l) t += sums[l];
    return sumf + t;
}

// ---------------------------------------------------------------- Q6_K

static float make_qx_quants(int n, int nmax, const float* x, int8_t* ls, int rmse_type) {
    float max = 0.f, amax = 0.f;
    for (int i = 0; i < n; ++i) {
        float ax = fabsf(x[i]);
        if (ax > amax) {
            amax = ax;
            max = x[i];
        }
    }
    if (amax == 0.f) {
        for (int i = 0; i < n; ++i) ls[i] = 0;
        return 0.f;
    }
    float iscale = -(float)nmax / max;
    if (rmse_type == 0) {
        for (int i = 0; i < n; ++i) {
            int l = nearest_int(iscale * x[i]);
            l = l < -nmax ? -nmax : (l > nmax - 1 ? nmax - 1 : l);
            ls[i] = (int8_t)(nmax + l);
        }
        return 1.0f / iscale;
    }
    int weight_type = rmse_type % 2;
    float sumlx = 0.f, suml2 = 0.f;
    for (int i = 0; i < n; ++i) {
        int l = nearest_int(iscale * x[i]);
        l = l < -nmax ? -nmax : (l > nmax - 1 ? nmax - 1 : l);
        ls[i] = (int8_t)(l + nmax);
        float w = weight_type == 1 ? x[i] * x[i] : 1.0f;
        float lf = (float)l;
        sumlx += w * x[i] * lf;
        suml2 += w * lf * lf;
    }
    float scale = sumlx / suml2;
    float best = scale * sumlx;
    for (int itry = 0; itry < 3; ++itry) {
        float is = 1.0f / scale;
        float slx = 0.f, sl2 = 0.f;
        bool changed = false;
        for (int i = 0; i < n; ++i) {
            int l = nearest_int(is * x[i]);
            l = l < -nmax ? -nmax : (l > nmax - 1 ? nmax - 1 : l);
            if (l + nmax != (int)ls[i]) changed = true;
            float w = weight_type == 1 ? x[i] * x[i] : 1.0f;
            float lf = (float)l;
            slx += w * x[i] * lf;
            sl2 += w * lf * lf;
        }
        if (!changed || sl2 == 0.f || slx * slx <= best * sl2) break;
        for (int i = 0; i < n; ++i) {
            int l = nearest_int(is * x[i]);
            ls[i] = (int8_t)(nmax + (l < -nmax ? -nmax : (l > nmax - 1 ? nmax - 1 : l)));
        }
        sumlx = slx;
        suml2 = sl2;
        scale = sumlx / suml2;
        best = scale * sumlx;
    }
    for (int itry = 0; itry < 5; ++itry) {
        int n_changed = 0;
        for (int i = 0; i < n; ++i) {
            float w = weight_type == 1 ? x[i] * x[i] : 1.0f;
            int l = (int)ls[i] - nmax;
            float slx = sumlx - w * x[i] * (float)l;
            if (slx > 0.f) {
                float sl2 = suml2 - w * (float)l * (float)l;
                int new_l = nearest_int(x[i] * sl2 / slx);
                new_l = new_l < -nmax ? -nmax : (new_l > nmax - 1 ? nmax - 1 : new_l);
                if (new_l != l) {
                    slx += w * x[i] * (float)new_l;
                    sl2 += w * (float)new_l * (float)new_l;
                    if (sl2 > 0.f && slx * slx * suml2 > sumlx * sumlx * sl2) {
                        ls[i] = (int8_t)(nmax + new_l);
                        sumlx = slx;
                        suml2 = sl2;
                        scale = sumlx / suml2;
                        best = scale * sumlx;
                        n_changed++;
                    }
                }
            }
        }
        if (n_changed == 0) break;
    }
    (void)best;
    return scale;  // rmse_type < 3 for every caller here
}

void q6k_from_float(const float* x, BQ6K* y) {
    int8_t L[256];
    float scales[16];
    float max_scale = 0.f, max_abs_scale = 0.f;
    for (int ib = 0; ib < 16; ++ib) {
        float scale = make_qx_quants(16, 32, x + 16 * ib, L + 16 * ib, 1);
        scales[ib] = scale;
        float as = fabsf(scale);
        if (as > max_abs_scale) {
            max_abs_scale = as;
            max_scale = scale;
        }
    }
    float iscale = -128.f / max_scale;
    y->d = f32_to_f16(1.0f / iscale);
    for (int ib = 0; ib < 16; ++ib) {
        int v = nearest_int(iscale * scales[ib]);
        y->scales[ib] = (int8_t)(v < 127 ? v : 127);
    }
    for (int j = 0; j < 16; ++j) {
        float d = f16_to_f32(y->d) * (float)y->scales[j];
        if (d == 0.f) continue;
        for (int ii = 0; ii < 16; ++ii) {
            int ll = nearest_int(x[16 * j + ii] / d);
            ll = ll < -32 ? -32 : (ll > 31 ? 31 : ll);
            L[16 * j + ii] = (int8_t)(ll + 32);
        }
    }
    uint8_t* ql = y->ql;
    uint8_t* qh = y->qh;
    for (int j = 0; j < 256; j += 128) {
        for (int l = 0; l < 32; ++l) {
            uint8_t q1 = L[j + l] & 0xF, q2 = L[j + l + 32] & 0xF;
            uint8_t q3 = L[j + l + 64] & 0xF, q4 = L[j + l + 96] & 0xF;
            ql[l] = (uint8_t)(q1 | (q3 << 4));
            ql[l + 32] = (uint8_t)(q2 | (q4 << 4));
            qh[l] = (uint8_t)((L[j + l] >> 4) | ((L[j + l + 32] >> 4) << 2) | ((L[j + l + 64] >> 4) << 4) |
                              ((L[j + l + 96] >> 4) << 6));
        }
        ql += 64;
        qh += 32;
    }
}

void q6k_to_float(const BQ6K* x, float* ys) {
    float d = f16_to_f32(x->d);
    for (int n = 0; n < 256; n += 128) {
        int idx = n / 128;
        float* y = ys + n;
        const int8_t* sc = x->scales + 8 * idx;
        const uint8_t* ql = x->ql + 64 * idx;
        const uint8_t* qh = x->qh + 32 * idx;
        for (int l = 0; l < 32; ++l) {
            int is = l / 16;
            int8_t q1 = (int8_t)((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
            int8_t q2 = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
            int8_t q3 = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            int8_t q4 = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            y[l] = d * (float)sc[is] * (float)q1;
            y[l + 32] = d * (float)sc[is + 2] * (float)q2;
            y[l + 64] = d * (float)sc[is + 4] * (float)q3;
            y[l + 96] = d * (float)sc[is + 6] * (float)q4;
        }
    }
}

float q6k_vec_dot(int64_t n, const BQ6K* xs, const BQ8K* ys) {
    int8_t aux8[256];
    float sums[8] = {0};
    for (int64_t bi = 0; bi < n / 256; ++bi) {
        const BQ6K* x = xs + bi;
        const BQ8K* y = ys + bi;
        float aux32[8] = {0};
        for (int j = 0; j < 256; j += 128) {
            int8_t* a = aux8 + j;
            const uint8_t* q4 = x->ql + j / 2;
            const uint8_t* qh = x->qh + j / 4;
            for (int l = 0; l < 32; ++l) {
                a[l] = (int8_t)(((q4[l] & 0xF) | ((qh[l] & 3) << 4)) - 32);
                a[l + 32] = (int8_t)(((q4[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32);
                a[l + 64] = (int8_t)(((q4[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32);
                a[l + 96] = (int8_t)(((q4[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32);
            }
        }
        for (int j = 0; j < 16; ++j) {
            float scale = (float)x->scales[j];
            const int8_t* q8 = y->qs + 16 * j;
            const int8_t* a = aux8 + 16 * j;
            for (int h = 0; h < 2; ++h)
                for (int l = 0; l < 8; ++l) aux32[l] += scale * (float)(int16_t)(q8[8 * h + l] * a[8 * h + l]);
        }
        float d = f16_to_f32(x->d) * y->d;
        for (int l = 0; l < 8; ++l) sums[l] += aux32[l] * d;
    }
    float t = 0.f;
    for (int l = 0; l < 8; ++l) t += sums[l];
    return t;
}

// ---------------------------------------------------------------- Q8_0

void q8_0_to_float(const BQ8_0* x, float* y) {
    float d = f16_to_f32(x->d);
    for (int j = 0; j < 32; ++j) y[j] = (float)x->qs[j] * d;
}

float q8_0_vec_dot(int64_t n, const BQ8_0* xs, const BQ8_0* ys) {
    float sumf = 0.f;
    for (int64_t bi = 0; bi < n / 32; ++bi) {
        int s = 0;
        for (int j = 0; j < 32; ++j) s += (int)xs[bi].qs[j] * (int)ys[bi].qs[j];
        sumf += (float)s * f16_to_f32(xs[bi].d) * f16_to_f32(ys[bi].d);
    }
    return sumf;
}

// ---------------------------------------------------------------- MXFP4

static uint8_t best_index_mxfp4(float x, float e) {
    uint8_t best = 0;
    float best_err = fabsf((float)KVALUES_MXFP4[0] * e - x);
    for (int i = 1; i < 16; ++i) {
        float err = fabsf((float)KVALUES_MXFP4[i] * e - x);
        if (err < best_err) {
            best = (uint8_t)i;
            best_err = err;
        }
    }
    return best;
}

void mxfp4_from_float(const float* x, BMXFP4* y) {
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    uint8_t e = 0;
    if (amax > 0.f) {
        float v = floorf(log2f(amax)) - 2.0f + 127.0f;
        e = v <= 0.f ? 0 : (v >= 255.f ? 255 : (uint8_t)v);  // `as u8` saturates
    }
    y->e = e;
    float d = e8m0_to_f32_half(e);
    for (int j = 0; j < 16; ++j) {
        uint8_t x0 = best_index_mxfp4(x[j], d);
        uint8_t x1 = best_index_mxfp4(x[j + 16], d);
        y->qs[j] = (uint8_t)(x0 | (x1 << 4));
    }
}

void mxfp4_to_float(const BMXFP4* x, float* y) {
    float d = e8m0_to_f32_half(x->e);
    for (int j = 0; j < 16; ++j) {
        y[j] = (float)KVALUES_MXFP4[x->qs[j] & 0x0F] * d;
        y[j + 16] = (float)KVALUES_MXFP4[x->qs[j] >> 4] * d;
    }
}

float mxfp4_vec_dot(int64_t n, const BMXFP4* xs, const BQ8_0* ys) {
    float sumf = 0.f;
    for (int64_t bi = 0; bi < n / 32; ++bi) {
        float d = f16_to_f32(ys[bi].d) * e8m0_to_f32_half(xs[bi].e);
        int s1 = 0, s2 = 0;
        for (int j = 0; j < 16; ++j) {
            s1 += (int)ys[bi].qs[j] * (int)KVALUES_MXFP4[xs[bi].qs[j] & 0x0F];
            s2 += (int)ys[bi].qs[j + 16] * (int)KVALUES_MXFP4[xs[bi].qs[j] >> 4];
        }
        sumf += d * (float)(s1 + s2);
    }
    return sumf;
}

// ---------------------------------------------------------------- IQ3_S / IQ2_S (Metal semantics)

void iq3s_to_float(const uint8_t* b, float* y) {
    float d = f16_to_f32((uint16_t)(b[0] | (b[1] << 8)));
    const uint8_t* qs = b + 2;
    const uint8_t* qh = b + 66;
    const uint8_t* signs = b + 74;
    const uint8_t* scales = b + 106;
    for (int ib = 0; ib < 8; ++ib) {
        float dl = d * (float)(1 + 2 * ((scales[ib / 2] >> (4 * (ib % 2))) & 0xF));
        for (int g = 0; g < 8; ++g) {
            int entry = qs[8 * ib + g] | (((qh[ib] >> g) & 1) << 8);
            uint32_t grid = cwx_iq3s_expand(cwx_iq3s_codes[entry]);
            for (int j = 0; j < 4; ++j) {
                int e = 32 * ib + 4 * g + j;
                float s = (signs[e / 8] >> (e % 8)) & 1 ? -1.f : 1.f;
                y[e] = dl * (float)((grid >> (8 * j)) & 0xFF) * s;
            }
        }
    }
}

void iq2s_to_float(const uint8_t* b, float* y) {
    float d = f16_to_f32((uint16_t)(b[0] | (b[1] << 8)));
    const uint8_t* qs = b + 2;
    const uint8_t* signs = b + 34;
    const uint8_t* qh = b + 66;
    const uint8_t* scales = b + 74;
    for (int ib = 0; ib < 8; ++ib) {
        for (int g = 0; g < 4; ++g) {
            float dl = d * (0.5f + (float)((scales[ib] >> (4 * (g / 2))) & 0xF)) * 0.25f;
            int entry = qs[4 * ib + g] | (((qh[ib] >> (2 * g)) & 3) << 8);
            uint64_t grid = cwx_iq2s_expand(cwx_iq2s_codes[entry]);
            for (int j = 0; j < 8; ++j) {
                float s = (signs[4 * ib + g] >> j) & 1 ? -1.f : 1.f;
                y[32 * ib + 8 * g + j] = dl * (float)((grid >> (8 * j)) & 0xFF) * s;
            }
        }
    }
}

// ---------------------------------------------------------------- IQ2_XXS / IQ3_XXS / IQ4_XS
// Metal semantics: dequantize_iq2_xxs quantized.metal:6819-6842, dequantize_iq3_xxs :6862-6890,
// dequantize_iq4_xs :6999-7018 (the reference's CPU path has no dequantisation for them,
// k_quants.rs:2955-2993).

static inline uint32_t le32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

void iq2xxs_to_float(const uint8_t* b, float* y) {
    float d = f16_to_f32((uint16_t)(b[0] | (b[1] << 8)));
    for (int ib = 0; ib < 8; ++ib) {
        const uint8_t* q = b + 2 + 8 * ib;
        const uint32_t aux = le32(q + 4);
        float dl = d * (0.5f + (float)(aux >> 28)) * 0.25f;
        for (int g = 0; g < 4; ++g) {
            uint64_t grid = cwx_iq2s_expand(cwx_iq2xxs_codes[q[g]]);
            uint32_t signs = cwx_ksigns((aux >> (7 * g)) & 127u);
            for (int j = 0; j < 8; ++j)
                y[32 * ib + 8 * g + j] = dl * (float)((grid >> (8 * j)) & 0xFF) * ((signs >> j) & 1 ? -1.f : 1.f);
        }
    }
}

void iq3xxs_to_float(const uint8_t* b, float* y) {
    float d = f16_to_f32((uint16_t)(b[0] | (b[1] << 8)));
    for (int ib = 0; ib < 8; ++ib) {
        const uint8_t* q = b + 2 + 8 * ib;
        const uint32_t aux = le32(b + 66 + 4 * ib);
        float dl = d * (0.5f + (float)(aux >> 28)) * 0.5f;
        for (int g = 0; g < 4; ++g) {
            uint32_t signs = cwx_ksigns((aux >> (7 * g)) & 127u);
            for (int h = 0; h < 2; ++h) {
                uint32_t grid = cwx_iq3xxs_expand(cwx_iq3xxs_codes[q[2 * g + h]]);
                for (int j = 0; j < 4; ++j)
                    y[32 * ib + 8 * g + 4 * h + j] =
                        dl * (float)((grid >> (8 * j)) & 0xFF) * ((signs >> (4 * h + j)) & 1 ? -1.f : 1.f);
            }
        }
    }
}

void iq4xs_to_float(const uint8_t* b, float* y) {
    float d = f16_to_f32((uint16_t)(b[0] | (b[1] << 8)));
    const uint32_t sh = (uint32_t)(b[2] | (b[3] << 8));
    for (int ib = 0; ib < 8; ++ib) {
        const int ls = ((b[4 + ib / 2] >> (4 * (ib % 2))) & 0xF) | (((sh >> (2 * ib)) & 3) << 4);
        const float dl = d * (float)(ls - 32);
        const uint8_t* q = b + 8 + 16 * ib;
        for (int m = 0; m < 16; ++m) {
            y[32 * ib + m] = dl * (float)cwx_iq4nl(q[m] & 0xF);
            y[32 * ib + 16 + m] = dl * (float)cwx_iq4nl(q[m] >> 4);
        }
    }
}

// Built once, on first use; function-local statics initialise thread-safely.
const uint16_t* iq3s_map() {
    static const std::vector<uint16_t> m = [] {
        std::vector<uint16_t> v(CWX_IQ3S_MAP_SIZE);
        cwx_build_iq3s_map(v.data());
        return v;
    }();
    return m.data();
}
const uint16_t* iq2s_map() {
    static const std::vector<uint16_t> m = [] {
        std::vector<uint16_t> v(CWX_IQ2S_MAP_SIZE);
        cwx_build_iq2s_map(v.data());
        return v;
    }();
    return m.data();
}
const uint16_t* iq3xxs_map() {
    static const std::vector<uint16_t> m = [] {
        std::vector<uint16_t> v(CWX_IQ3XXS_MAP_SIZE);
        cwx_build_iq3xxs_map(v.data());
        return v;
    }();
    return m.data();
}
const uint16_t* iq2xxs_map() {
    static const std::vector<uint16_t> m = [] {
        std::vector<uint16_t> v(CWX_IQ2XXS_MAP_SIZE);
        cwx_build_iq2xxs_map(v.data());
        return v;
    }();
    return m.data();
}

}  // namespace cwo

using namespace cwo;

extern "C" {

int cwo_block_elems(int type) {
    switch (type) {
        case CWO_F32: return 1;
        case CWO_Q8_0: case CWO_MXFP4: return 32;
        case CWO_Q4_K: case CWO_Q6_K: case CWO_Q8_K: case CWO_IQ2_S: case CWO_IQ3_S: case CWO_IQ2_XXS:
        case CWO_IQ3_XXS: case CWO_IQ4_XS: return 256;
        default: return 0;
    }
}

int cwo_block_bytes(int type) {
    switch (type) {
        case CWO_F32: return 4;
        case CWO_Q8_0: return 34;
        case CWO_MXFP4: return 17;
        case CWO_Q4_K: return 144;
        case CWO_Q6_K: return 210;
        case CWO_Q8_K: return 292;
        case CWO_IQ2_S: return 82;
        case CWO_IQ3_S: return 110;
        case CWO_IQ2_XXS: return 66;
        case CWO_IQ3_XXS: return 98;
        case CWO_IQ4_XS: return 136;
        default: return 0;
    }
}

int64_t cwo_row_bytes(int type, int64_t k) {
    int be = cwo_block_elems(type);
    if (be == 0 || k % be) return -1;
    return k / be * cwo_block_bytes(type);
}

int cwo_vec_dot_type(int type) {
    switch (type) {
        case CWO_Q4_K: case CWO_Q6_K: return CWO_Q8_K;
        case CWO_Q8_0: case CWO_MXFP4: return CWO_Q8_0;
        default: return CWO_F32;
    }
}

int cwo_quantize(int type, const float* x, int64_t n, void* out) {
    int be = cwo_block_elems(type);
    if (be == 0 || n % be) return -1;
    int64_t nb = n / be;
    uint8_t* o = (uint8_t*)out;
    int bb = cwo_block_bytes(type);
    if (type == CWO_IQ3_S) iq3s_map();
    if (type == CWO_IQ2_S) iq2s_map();
    if (type == CWO_IQ3_XXS) iq3xxs_map();
    if (type == CWO_IQ2_XXS) iq2xxs_map();
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < nb; ++i) {
        const float* xi = x + i * be;
        void* yi = o + i * bb;
        switch (type) {
            case CWO_Q4_K: q4k_from_float(xi, (BQ4K*)yi); break;
            case CWO_Q6_K: q6k_from_float(xi, (BQ6K*)yi); break;
            case CWO_Q8_0: q8_0_from_float(xi, (BQ8_0*)yi); break;
            case CWO_Q8_K: q8k_from_float(xi, (BQ8K*)yi); break;
            case CWO_MXFP4: mxfp4_from_float(xi, (BMXFP4*)yi); break;
            case CWO_IQ3_S: cwx_encode_iq3s(xi, (uint8_t*)yi, iq3s_map()); break;
            case CWO_IQ2_S: cwx_encode_iq2s(xi, (uint8_t*)yi, iq2s_map()); break;
            case CWO_IQ2_XXS: cwx_encode_iq2xxs(xi, (uint8_t*)yi, iq2xxs_map()); break;
            case CWO_IQ3_XXS: cwx_encode_iq3xxs(xi, (uint8_t*)yi, iq3xxs_map()); break;
            case CWO_IQ4_XS: cwx_encode_iq4xs(xi, (uint8_t*)yi); break;
            case CWO_F32: memcpy(yi, xi, 4); break;
        }
    }
    return 0;
}

int cwo_dequantize(int type, const void* blocks, int64_t n, float* y) {
    int be = cwo_block_elems(type);
    if (be == 0 || n % be) return -1;
    int64_t nb = n / be;
    const uint8_t* b = (const uint8_t*)blocks;
    int bb = cwo_block_bytes(type);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < nb; ++i) {
        const void* bi = b + i * bb;
        float* yi = y + i * be;
        switch (type) {
            case CWO_Q4_K: q4k_to_float((const BQ4K*)bi, yi); break;
            case CWO_Q6_K: q6k_to_float((const BQ6K*)bi, yi); break;
            case CWO_Q8_0: q8_0_to_float((const BQ8_0*)bi, yi); break;
            case CWO_Q8_K: {
                const BQ8K* q = (const BQ8K*)bi;
                for (int j = 0; j < 256; ++j) yi[j] = q->d * (float)q->qs[j];
                break;
            }
            case CWO_MXFP4: mxfp4_to_float((const BMXFP4*)bi, yi); break;
            case CWO_IQ3_S: iq3s_to_float((const uint8_t*)bi, yi); break;
            case CWO_IQ2_S: iq2s_to_float((const uint8_t*)bi, yi); break;
            case CWO_IQ2_XXS: iq2xxs_to_float((const uint8_t*)bi, yi); break;
            case CWO_IQ3_XXS: iq3xxs_to_float((const uint8_t*)bi, yi); break;
            case CWO_IQ4_XS: iq4xs_to_float((const uint8_t*)bi, yi); break;
            case CWO_F32: memcpy(yi, bi, 4); break;
        }
    }
    return 0;
}

float cwo_vec_dot(int type, int64_t n, const void* w, const void* a) {
    switch (type) {
        case CWO_Q4_K: return q4k_vec_dot(n, (const BQ4K*)w, (const BQ8K*)a);
        case CWO_Q6_K: return q6k_vec_dot(n, (const BQ6K*)w, (const BQ8K*)a);
        case CWO_Q8_0: return q8_0_vec_dot(n, (const BQ8_0*)w, (const BQ8_0*)a);
        case CWO_MXFP4: return mxfp4_vec_dot(n, (const BMXFP4*)w, (const BQ8_0*)a);
        default: return nanf("");
    }
}

}  // extern "C"
