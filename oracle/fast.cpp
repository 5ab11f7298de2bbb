// Vectorised CPU build of the MoE layer -- BENCHMARK BASELINE ONLY (not a parity oracle).
//
// The oracle in moe.cpp restates candle's CPU arithmetic step for step (vec_dot_unopt, scalar
// to_float) and is the checker. This file computes the same layer the way an optimised x86 build
// of the reference would, as the timed CPU baseline: candle's x86 path multiplies Q4_K weights by
// Q8_K activations with AVX2 integer dot products (vendor/candle-core/src/quantized/avx.rs:451,
// repack_x86.rs:43-60); the IQ formats have no CPU path in the reference (k_quants.rs:2955-2993),
// so they are dequantised here through expanded codebook tables and multiplied in f32 with FMA.
// Compiled with -O3 -mavx2 -mfma -ffast-math (the reductions vectorise), OpenMP over
// (expert, row block) tasks of the whole layer. Routing: f32 router logits (as candle's gemm),
// softmax, stable top-k, renormalisation as the oracle. Results agree with O1 within f32
// rounding (tests/test_oracle.py checks the relative L2 distance).
#include <math.h>
#include <omp.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "cw_oracle.h"
#include "iq_grids.h"
#include "oracle_internal.h"
#include "synth_math.h"

namespace {

using namespace cwo;

struct Tables {
    float f16[65536];
    int8_t iq2s[1024][8];
    int8_t iq3s[512][4];
    float sign8[256][8];  // +-1 per bit of a sign byte
    Tables() {
        for (int i = 0; i < 65536; ++i) f16[i] = cwx_f16_bits_to_f32((uint16_t)i);
        for (int e = 0; e < 1024; ++e) {
            uint64_t g = cwx_iq2s_expand(cwx_iq2s_codes[e]);
            for (int j = 0; j < 8; ++j) iq2s[e][j] = (int8_t)((g >> (8 * j)) & 0xFF);
        }
        for (int e = 0; e < 512; ++e) {
            uint32_t g = cwx_iq3s_expand(cwx_iq3s_codes[e]);
            for (int j = 0; j < 4; ++j) iq3s[e][j] = (int8_t)((g >> (8 * j)) & 0xFF);
        }
        for (int s = 0; s < 256; ++s)
            for (int j = 0; j < 8; ++j) sign8[s][j] = (s >> j) & 1 ? -1.f : 1.f;
    }
};

const Tables& tables() {
    static const Tables t;
    return t;
}

// One IQ2_S block (82 bytes) to 256 f32 values.
void iq2s_block(const uint8_t* b, const Tables& T, float* y) {
    const float d = T.f16[b[0] | (b[1] << 8)];
    const uint8_t *qs = b + 2, *signs = b + 34, *qh = b + 66, *scales = b + 74;
    for (int ib = 0; ib < 8; ++ib)
        for (int g = 0; g < 4; ++g) {
            const float dl = d * (0.5f + (float)((scales[ib] >> (4 * (g / 2))) & 0xF)) * 0.25f;
            const int8_t* gr = T.iq2s[qs[4 * ib + g] | (((qh[ib] >> (2 * g)) & 3) << 8)];
            const float* sg = T.sign8[signs[4 * ib + g]];
            float* o = y + 32 * ib + 8 * g;
            for (int j = 0; j < 8; ++j) o[j] = dl * (float)gr[j] * sg[j];
        }
}

// One IQ3_S block (110 bytes) to 256 f32 values.
void iq3s_block(const uint8_t* b, const Tables& T, float* y) {
    const float d = T.f16[b[0] | (b[1] << 8)];
    const uint8_t *qs = b + 2, *qh = b + 66, *signs = b + 74, *scales = b + 106;
    for (int ib = 0; ib < 8; ++ib) {
        const float dl = d * (float)(1 + 2 * ((scales[ib / 2] >> (4 * (ib % 2))) & 0xF));
        for (int g = 0; g < 8; g += 2) {
            const int8_t* g0 = T.iq3s[qs[8 * ib + g] | (((qh[ib] >> g) & 1) << 8)];
            const int8_t* g1 = T.iq3s[qs[8 * ib + g + 1] | (((qh[ib] >> (g + 1)) & 1) << 8)];
            const float* sg = T.sign8[signs[4 * ib + g / 2]];
            float* o = y + 32 * ib + 4 * g;
            for (int j = 0; j < 4; ++j) o[j] = dl * (float)g0[j] * sg[j];
            for (int j = 0; j < 4; ++j) o[4 + j] = dl * (float)g1[j] * sg[4 + j];
        }
    }
}

float dot_f32(const float* a, const float* b, int n) {
    float s = 0.f;
#pragma omp simd reduction(+ : s)
    for (int i = 0; i < n; ++i) s += a[i] * b[i];
    return s;
}

// Q4_K row x Q8_K activation row: integer sums per 32-column sub-block (vectorised), the
// block's scales and mins applied in f32.
float q4k_dot(const BQ4K* x, const BQ8K* y, int nb, const Tables& T) {
    float acc = 0.f;
    for (int b = 0; b < nb; ++b) {
        uint8_t sc[8], mn[8];
        const uint8_t* s = x[b].scales;
        for (int j = 0; j < 8; ++j) {
            if (j < 4) {
                sc[j] = s[j] & 63;
                mn[j] = s[j + 4] & 63;
            } else {
                sc[j] = (uint8_t)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
                mn[j] = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
            }
        }
        int sumi = 0, summ = 0;
        for (int c = 0; c < 4; ++c) {
            const uint8_t* q = x[b].qs + 32 * c;
            const int8_t* a0 = y[b].qs + 64 * c;
            const int8_t* a1 = a0 + 32;
            int s0 = 0, s1 = 0;
#pragma omp simd reduction(+ : s0, s1)
            for (int l = 0; l < 32; ++l) {
                s0 += (int)(q[l] & 0xF) * (int)a0[l];
                s1 += (int)(q[l] >> 4) * (int)a1[l];
            }
            sumi += s0 * sc[2 * c] + s1 * sc[2 * c + 1];
        }
        for (int j = 0; j < 16; ++j) summ += (int)y[b].bsums[j] * (int)mn[j / 2];
        acc += T.f16[x[b].d] * y[b].d * (float)sumi - T.f16[x[b].dmin] * y[b].d * (float)summ;
    }
    return acc;
}

// One expert matrix (n rows x k) against `rows` activation rows, output rows 0 .. n-1 of each.
// IQ2_S / IQ3_S: f32 activations; Q4_K: Q8_K activations; other formats through the oracle's
// dequantisation and an f32 dot.
struct Mat {
    int type;
    const uint8_t* base;  // the expert's bytes
    int64_t n, k, row_bytes;
};

void mat_rows(const Mat& m, int64_t r0, int64_t r1, const float* const* xr, const BQ8K* const* q8, int rows,
              float* const* out, float* tmp, const Tables& T) {
    for (int64_t r = r0; r < r1; ++r) {
        const uint8_t* w = m.base + r * m.row_bytes;
        if (m.type == CWO_Q4_K) {
            for (int p = 0; p < rows; ++p) out[p][r] = q4k_dot((const BQ4K*)w, q8[p], (int)(m.k / 256), T);
            continue;
        }
        if (m.type == CWO_IQ2_S)
            for (int64_t b = 0; b < m.k / 256; ++b) iq2s_block(w + b * 82, T, tmp + 256 * b);
        else if (m.type == CWO_IQ3_S)
            for (int64_t b = 0; b < m.k / 256; ++b) iq3s_block(w + b * 110, T, tmp + 256 * b);
        else
            cwo_dequantize(m.type, w, m.k, tmp);
        for (int p = 0; p < rows; ++p) out[p][r] = dot_f32(tmp, xr[p], (int)m.k);
    }
}

float silu(float v) { return v / (1.0f + expf(-v)); }

}  // namespace

extern "C" int cwo_moe_forward_fast(const cwo_moe_layer* L, const float* x, int T, float* out) {
    if (L->act != CWO_ACT_SILU) return -2;  // the baseline covers the SiLU layers (configs 0, 1, 2, 4)
    const Tables& TB = tables();
    const int H = L->hidden, E = L->n_experts, K = L->top_k, I = L->inter;
    const int64_t n = (int64_t)T * K;
    // router (f32, vectorised) and route
    std::vector<float> logits((size_t)T * E);
#pragma omp parallel for collapse(2) schedule(static)
    for (int t = 0; t < T; ++t)
        for (int e = 0; e < E; ++e) {
            float l = dot_f32(x + (int64_t)t * H, L->router_w + (int64_t)e * H, H);
            logits[(size_t)t * E + e] = L->router_b ? l + L->router_b[e] : l;
        }
    std::vector<uint32_t> ids((size_t)n);
    std::vector<float> w((size_t)n);
    if (cwo_route(logits.data(), T, E, K, L->norm_topk_prob, ids.data(), w.data())) return -1;
    // piles
    std::vector<std::vector<int64_t>> picks((size_t)E);
    for (int64_t i = 0; i < n; ++i) picks[ids[i]].push_back(i);
    std::vector<int> used;
    for (int e = 0; e < E; ++e)
        if (!picks[e].empty()) used.push_back(e);
    const int64_t rb_g = cwo_row_bytes(L->gate_type, H), rb_u = cwo_row_bytes(L->up_type, H);
    const int64_t rb_d = cwo_row_bytes(L->down_type, I);
    // activation rows quantised once per token when a routed or shared matrix takes Q8_K
    auto needs_q8 = [](int t) { return t == CWO_Q4_K; };
    std::vector<BQ8K> xq;
    const bool sh = L->shared_inter > 0;
    if (needs_q8(L->gate_type) || (sh && needs_q8(L->sh_gate_type))) {
        xq.resize((size_t)T * (H / 256));
#pragma omp parallel for
        for (int t = 0; t < T; ++t)
            for (int b = 0; b < H / 256; ++b) q8k_from_float(x + (int64_t)t * H + 256 * b, &xq[(size_t)t * (H / 256) + b]);
    }
    std::vector<float> g((size_t)n * I), u((size_t)n * I), h((size_t)n * I), y((size_t)n * H);
    const int RB = 64;
    // task lists: (used expert, row block)
    auto run = [&](int stage) {
        const int64_t rows_m = stage == 0 ? I : H;
        const int64_t nblk = (rows_m + RB - 1) / RB;
        const int64_t ntask = (int64_t)used.size() * nblk;
#pragma omp parallel
        {
            std::vector<float> tmp((size_t)(H > I ? H : I));
            std::vector<const float*> xr;
            std::vector<const BQ8K*> q8;
            std::vector<float*> o0, o1;
            std::vector<BQ8K> hq;
#pragma omp for schedule(dynamic, 1)
            for (int64_t task = 0; task < ntask; ++task) {
                const int e = used[(size_t)(task / nblk)];
                const int64_t r0 = (task % nblk) * RB, r1 = std::min<int64_t>(r0 + RB, rows_m);
                const std::vector<int64_t>& pl = picks[(size_t)e];
                const int np = (int)pl.size();
                xr.resize(np);
                q8.resize(np);
                o0.resize(np);
                o1.resize(np);
                if (stage == 0) {
                    for (int p = 0; p < np; ++p) {
                        const int64_t tok = pl[p] / K;
                        xr[p] = x + tok * H;
                        q8[p] = xq.empty() ? nullptr : &xq[(size_t)tok * (H / 256)];
                        o0[p] = &g[(size_t)pl[p] * I];
                        o1[p] = &u[(size_t)pl[p] * I];
                    }
                    Mat mg{L->gate_type, (const uint8_t*)L->gate_bank + (int64_t)e * rb_g * I, I, H, rb_g};
                    Mat mu{L->up_type, (const uint8_t*)L->up_bank + (int64_t)e * rb_u * I, I, H, rb_u};
                    mat_rows(mg, r0, r1, xr.data(), q8.data(), np, o0.data(), tmp.data(), TB);
                    mat_rows(mu, r0, r1, xr.data(), q8.data(), np, o1.data(), tmp.data(), TB);
                } else {
                    if (needs_q8(L->down_type)) hq.resize((size_t)np * (I / 256));
                    for (int p = 0; p < np; ++p) {
                        xr[p] = &h[(size_t)pl[p] * I];
                        if (needs_q8(L->down_type)) {
                            for (int b = 0; b < I / 256; ++b) q8k_from_float(xr[p] + 256 * b, &hq[(size_t)p * (I / 256) + b]);
                            q8[p] = &hq[(size_t)p * (I / 256)];
                        }
                        o0[p] = &y[(size_t)pl[p] * H];
                    }
                    Mat md{L->down_type, (const uint8_t*)L->down_bank + (int64_t)e * rb_d * H, H, I, rb_d};
                    mat_rows(md, r0, r1, xr.data(), q8.data(), np, o0.data(), tmp.data(), TB);
                }
            }
        }
    };
    run(0);
#pragma omp parallel for
    for (int64_t i = 0; i < n * I; ++i) h[i] = silu(g[i]) * u[i];
    run(1);
    // shared expert: every token through one Q4_K (or other) expert
    std::vector<float> ys;
    std::vector<float> sgate((size_t)T, 0.f);
    if (sh) {
        const int Is = L->shared_inter;
        const int64_t sg_rb = cwo_row_bytes(L->sh_gate_type, H), su_rb = cwo_row_bytes(L->sh_up_type, H);
        const int64_t sd_rb = cwo_row_bytes(L->sh_down_type, Is);
        std::vector<float> gs((size_t)T * Is), us((size_t)T * Is), hs((size_t)T * Is);
        ys.resize((size_t)T * H);
        std::vector<BQ8K> hsq;
        auto stage = [&](const Mat& m, const std::vector<const float*>& xr, const std::vector<const BQ8K*>& q8,
                         std::vector<float*>& o) {
            const int64_t nblk = (m.n + RB - 1) / RB;
#pragma omp parallel
            {
                std::vector<float> tmp((size_t)m.k);
#pragma omp for schedule(dynamic, 1)
                for (int64_t b = 0; b < nblk; ++b)
                    mat_rows(m, b * RB, std::min<int64_t>(b * RB + RB, m.n), xr.data(), q8.data(), T, o.data(),
                             tmp.data(), TB);
            }
        };
        std::vector<const float*> xr(T);
        std::vector<const BQ8K*> q8(T);
        std::vector<float*> og(T), ou(T), od(T);
        for (int t = 0; t < T; ++t) {
            xr[t] = x + (int64_t)t * H;
            q8[t] = xq.empty() ? nullptr : &xq[(size_t)t * (H / 256)];
            og[t] = &gs[(size_t)t * Is];
            ou[t] = &us[(size_t)t * Is];
            od[t] = &ys[(size_t)t * H];
        }
        stage(Mat{L->sh_gate_type, (const uint8_t*)L->sh_gate, Is, H, sg_rb}, xr, q8, og);
        stage(Mat{L->sh_up_type, (const uint8_t*)L->sh_up, Is, H, su_rb}, xr, q8, ou);
        for (size_t i = 0; i < hs.size(); ++i) hs[i] = silu(gs[i]) * us[i];
        if (needs_q8(L->sh_down_type)) {
            hsq.resize((size_t)T * (Is / 256));
            for (int t = 0; t < T; ++t)
                for (int b = 0; b < Is / 256; ++b) q8k_from_float(&hs[(size_t)t * Is + 256 * b], &hsq[(size_t)t * (Is / 256) + b]);
        }
        for (int t = 0; t < T; ++t) {
            xr[t] = &hs[(size_t)t * Is];
            q8[t] = hsq.empty() ? nullptr : &hsq[(size_t)t * (Is / 256)];
        }
        stage(Mat{L->sh_down_type, (const uint8_t*)L->sh_down, H, Is, sd_rb}, xr, q8, od);
        for (int t = 0; t < T; ++t)
            sgate[t] = 1.0f / (1.0f + expf(-dot_f32(x + (int64_t)t * H, L->sh_gate_inp, H)));
    }
    // weighted combine in pick order, plus the gated shared expert
#pragma omp parallel for
    for (int t = 0; t < T; ++t)
        for (int c = 0; c < H; ++c) {
            float acc = 0.f;
            for (int j = 0; j < K; ++j) acc += y[((size_t)t * K + j) * H + c] * w[(size_t)t * K + j];
            if (sh) acc += ys[(size_t)t * H + c] * sgate[t];
            out[(size_t)t * H + c] = acc;
        }
    return 0;
}
