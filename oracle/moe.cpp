// Oracle: routing, permutation and the MoE layer -- TEST INFRASTRUCTURE ONLY (see cw_oracle.h).
//
//   route            crates/engine/src/experts.rs:2364-2372 (softmax_last_dim, stable descending
//                    arg_sort vendor/candle-core/src/sort.rs:40-52, narrow k, gather, renorm)
//   softmax          candle-nn softmax_last_dim CPU: row max, exp(x - max), vec_reduce_sum
//                    (x86 AVX order, vendor/candle-core/src/cpu/avx.rs:243-257), divide
//   permutation      cw_pile crates/engine/src/fuse_kernel.rs:180-202 (stable by expert)
//   layer, O1        StreamedMoe::reference experts.rs:2500-2537 (group by expert in a BTreeMap,
//                    QMatMul per expert, act, x weight, one index_add in expert order)
//   layer, O2        resident Metal path experts.rs:2562-2614 (weighted_sum in pick order,
//                    fuse_kernel.rs:277-291)
//   activations      ExpertAct experts.rs:2389-2422; silu op.rs:756-758; clamped SwiGLU constants
//                    model_gptoss.rs:16-17
//   shared expert    SharedExpert::forward model_next.rs:731-741
// Router logits use exact f32 products accumulated in f64 and rounded once: candle's gemm
// crate summation order is not restatable, and any correct f32 GEMV lies within its rounding.
// The softmax and the shared-expert gate take exp correctly rounded to f32, computed as exp in f64
// rounded once: glibc's expf (what Rust's f32::exp calls on x86-64 Linux) is within 0.502 ulp but
// misrounds some inputs next to a rounding midpoint, and the reference's own platform (Apple's
// libm, Metal) is a third implementation, so the checker takes the one exact definition. The
// activations (SiLU, clamped SwiGLU) use expf; their outputs are compared within a tolerance.
#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <vector>

#include "cw_oracle.h"
#include "oracle_internal.h"
#include "synth_math.h"

namespace cwo {

float avx_sum(const float* x, int n) {
    int np = n & ~31;
    float acc[4][8] = {{0}};
    for (int i = 0; i < np; i += 32)
        for (int j = 0; j < 4; ++j)
            for (int e = 0; e < 8; ++e) acc[j][e] += x[i + 8 * j + e];
    float X[8];
    for (int e = 0; e < 8; ++e) X[e] = (acc[0][e] + acc[1][e]) + (acc[2][e] + acc[3][e]);
    float t0[4];
    for (int e = 0; e < 4; ++e) t0[e] = X[e] + X[e + 4];
    float r = (t0[0] + t0[1]) + (t0[2] + t0[3]);
    for (int i = np; i < n; ++i) r += x[i];
    return r;
}

static float exp_cr(float x) { return (float)exp((double)x); }

static void softmax_row(const float* x, int n, float* p) {
    float mx = x[0];
    for (int i = 1; i < n; ++i) mx = fmaxf(mx, x[i]);
    for (int i = 0; i < n; ++i) p[i] = exp_cr(x[i] - mx);
    float s = avx_sum(p, n);
    for (int i = 0; i < n; ++i) p[i] = p[i] / s;
}

static float silu(float v) { return v / (1.0f + expf(-v)); }
static float sigmoid(float v) { return 1.0f / (exp_cr(-v) + 1.0f); }

}  // namespace cwo

using namespace cwo;

extern "C" {

void cwo_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}
int cwo_get_threads(void) { return omp_get_max_threads(); }

uint64_t cwo_stream(uint32_t seed, uint32_t layer, uint32_t tensor) { return cwx_stream(seed, layer, tensor); }

void cwo_normal(uint64_t key, uint64_t offset, int64_t n, float std_, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = cwx_normal_std(key, offset + (uint64_t)i, std_);
}

int cwo_synth_matrix(int type, uint64_t key, int64_t e0, int64_t ne, int64_t n, int64_t k, float std_, void* out) {
    int64_t rb = cwo_row_bytes(type, k);
    if (rb < 0) return -1;
    if (type == CWO_IQ3_S) iq3s_map();
    if (type == CWO_IQ2_S) iq2s_map();
    if (type == CWO_IQ3_XXS) iq3xxs_map();
    if (type == CWO_IQ2_XXS) iq2xxs_map();
    uint8_t* o = (uint8_t*)out;
#pragma omp parallel
    {
        std::vector<float> row((size_t)k);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < ne * n; ++r) {
            uint64_t base = (uint64_t)(e0 * n + r) * (uint64_t)k;
            for (int64_t c = 0; c < k; ++c) row[c] = cwx_normal_std(key, base + (uint64_t)c, std_);
            cwo_quantize(type, row.data(), k, o + r * rb);
        }
    }
    return 0;
}

void cwo_router(const float* x, const float* w, const float* b, int T, int H, int E, float* logits) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int t = 0; t < T; ++t)
        for (int e = 0; e < E; ++e) {
            double s = 0.0;
            for (int h = 0; h < H; ++h) s += (double)x[(int64_t)t * H + h] * (double)w[(int64_t)e * H + h];
            float l = (float)s;
            logits[(int64_t)t * E + e] = b ? l + b[e] : l;
        }
}

static float lane_tree(float* a, int n) {  // halves added pairwise until one lane is left
    for (int w = n / 2; w >= 1; w /= 2)
        for (int i = 0; i < w; ++i) a[i] = a[i] + a[i + w];
    return a[0];
}

static float pairwise_sum(const float* x, const float* w, int n) {
    if (n <= 8) {
        float s = 0.0f;
        for (int i = 0; i < n; ++i) s = s + x[i] * w[i];
        return s;
    }
    const int h = n / 2;
    return pairwise_sum(x, w, h) + pairwise_sum(x + h, w + h, n - h);
}

static float dot_f32(const float* x, const float* w, int H, int order) {
    switch (order) {
        case 0: {
            float s = 0.0f;
            for (int i = 0; i < H; ++i) s = s + x[i] * w[i];
            return s;
        }
        case 1: {
            float s = 0.0f;
            for (int i = 0; i < H; ++i) s = fmaf(x[i], w[i], s);
            return s;
        }
        case 2:
        case 3: {
            const int L = order == 2 ? 8 : 16;
            float acc[16] = {0};
            int i = 0;
            for (; i + L <= H; i += L)
                for (int j = 0; j < L; ++j) acc[j] = fmaf(x[i + j], w[i + j], acc[j]);
            float s = lane_tree(acc, L);
            for (; i < H; ++i) s = fmaf(x[i], w[i], s);
            return s;
        }
        case 4: {
            float s = 0.0f;
            for (int k0 = 0; k0 < H; k0 += 256) {
                const int k1 = k0 + 256 < H ? k0 + 256 : H;
                float acc[8] = {0};
                int i = k0;
                for (; i + 8 <= k1; i += 8)
                    for (int j = 0; j < 8; ++j) acc[j] = fmaf(x[i + j], w[i + j], acc[j]);
                float p = lane_tree(acc, 8);
                for (; i < k1; ++i) p = fmaf(x[i], w[i], p);
                s = s + p;
            }
            return s;
        }
        default:
            return pairwise_sum(x, w, H);
    }
}

int cwo_router_f32(const float* x, const float* w, const float* b, int T, int H, int E, int order, float* logits) {
    if (order < 0 || order > 5 || T < 0 || H < 1 || E < 1) return -1;
#pragma omp parallel for collapse(2) schedule(static)
    for (int t = 0; t < T; ++t)
        for (int e = 0; e < E; ++e) {
            float l = dot_f32(x + (int64_t)t * H, w + (int64_t)e * H, H, order);
            logits[(int64_t)t * E + e] = b ? l + b[e] : l;
        }
    return 0;
}

int cwo_route(const float* logits, int T, int E, int k, int norm, uint32_t* ids, float* w) {
    if (k < 1 || k > E) return -1;
    std::vector<float> p((size_t)E);
    std::vector<uint32_t> idx((size_t)E);
    std::vector<float> tw((size_t)k);
    for (int t = 0; t < T; ++t) {
        softmax_row(logits + (int64_t)t * E, E, p.data());
        for (int i = 0; i < E; ++i) idx[i] = (uint32_t)i;
        // sort_by(|&j, &i| p[i].partial_cmp(&p[j]).unwrap_or(Greater)), stable
        std::stable_sort(idx.begin(), idx.end(), [&](uint32_t j, uint32_t i) { return p[i] < p[j]; });
        for (int j = 0; j < k; ++j) {
            ids[(int64_t)t * k + j] = idx[j];
            tw[j] = p[idx[j]];
        }
        if (norm) {
            float s = avx_sum(tw.data(), k);
            for (int j = 0; j < k; ++j) tw[j] = tw[j] / s;
        }
        for (int j = 0; j < k; ++j) w[(int64_t)t * k + j] = tw[j];
    }
    return 0;
}

int cwo_permute(const uint32_t* ids, int T, int k, int E, uint32_t* pairs, uint32_t* heads) {
    int64_t n = (int64_t)T * k;
    std::vector<uint32_t> cnt((size_t)E, 0);
    for (int64_t i = 0; i < n; ++i) {
        if (ids[i] >= (uint32_t)E) return -1;
        cnt[ids[i]]++;
    }
    std::vector<uint32_t> pos((size_t)E, 0);
    uint32_t off = 0;
    for (int e = 0; e < E; ++e) {
        heads[3 * e] = (uint32_t)e;
        heads[3 * e + 1] = off;
        heads[3 * e + 2] = cnt[e];
        pos[e] = off;
        off += cnt[e];
    }
    for (int64_t i = 0; i < n; ++i) pairs[pos[ids[i]]++] = (uint32_t)i;
    return 0;
}

int cwo_matmul(int type, int mode, const void* bank, int64_t n, int64_t k, int64_t bpe, uint32_t expert,
               const float* x, int rows, float* out) {
    int64_t rb = cwo_row_bytes(type, k);
    if (rb < 0) return -1;
    const uint8_t* base = (const uint8_t*)bank + (int64_t)expert * bpe;
    int vdt = cwo_vec_dot_type(type);
    if (mode == CWO_MODE_CANDLE && vdt != CWO_F32) {
        int64_t arb = cwo_row_bytes(vdt, k);
        std::vector<uint8_t> act((size_t)(arb * rows));
        for (int r = 0; r < rows; ++r) cwo_quantize(vdt, x + (int64_t)r * k, k, act.data() + r * arb);
#pragma omp parallel for schedule(static)
        for (int64_t c = 0; c < n; ++c)
            for (int r = 0; r < rows; ++r)
                out[(int64_t)r * n + c] = cwo_vec_dot(type, k, base + c * rb, act.data() + r * arb);
        return 0;
    }
#pragma omp parallel
    {
        std::vector<float> wrow((size_t)k);
#pragma omp for schedule(static)
        for (int64_t c = 0; c < n; ++c) {
            cwo_dequantize(type, base + c * rb, k, wrow.data());
            for (int r = 0; r < rows; ++r) {
                const float* xr = x + (int64_t)r * k;
                double s = 0.0;
                for (int64_t i = 0; i < k; ++i) s += (double)wrow[i] * (double)xr[i];
                out[(int64_t)r * n + c] = (float)s;
            }
        }
    }
    return 0;
}

static void act_hidden(const cwo_moe_layer* L, uint32_t e, const float* g, const float* u, int rows, float* h) {
    int I = L->inter;
    for (int r = 0; r < rows; ++r)
        for (int i = 0; i < I; ++i) {
            float gv = g[(int64_t)r * I + i], uv = u[(int64_t)r * I + i];
            if (L->act == CWO_ACT_SILU) {
                h[(int64_t)r * I + i] = silu(gv) * uv;
            } else {
                if (L->gate_b) gv = gv + L->gate_b[(int64_t)e * I + i];
                gv = fminf(gv, L->limit);
                if (L->up_b) uv = uv + L->up_b[(int64_t)e * I + i];
                uv = fminf(fmaxf(uv, -L->limit), L->limit);
                float glu = gv * sigmoid(gv * L->alpha + 0.0f);
                h[(int64_t)r * I + i] = (uv + 1.0f) * glu;
            }
        }
}

int cwo_moe_forward(const cwo_moe_layer* L, const float* x, int T, int mode, float* out, float* routed_out,
                    float* shared_out, uint32_t* ids_out, float* w_out) {
    const int H = L->hidden, E = L->n_experts, K = L->top_k, I = L->inter;
    std::vector<float> logits((size_t)T * E);
    cwo_router(x, L->router_w, L->router_b, T, H, E, logits.data());
    std::vector<uint32_t> ids((size_t)T * K);
    std::vector<float> w((size_t)T * K);
    if (cwo_route(logits.data(), T, E, K, L->norm_topk_prob, ids.data(), w.data())) return -1;
    if (ids_out) memcpy(ids_out, ids.data(), ids.size() * 4);
    if (w_out) memcpy(w_out, w.data(), w.size() * 4);

    int64_t bpe_g = cwo_row_bytes(L->gate_type, H) * I;
    int64_t bpe_u = cwo_row_bytes(L->up_type, H) * I;
    int64_t bpe_d = cwo_row_bytes(L->down_type, I) * H;
    if (bpe_g < 0 || bpe_u < 0 || bpe_d < 0) return -1;

    // Per-pick down rows (before weights), computed expert by expert.
    std::map<uint32_t, std::vector<int64_t>> picks;  // expert -> flat pick indices in token order
    for (int64_t i = 0; i < (int64_t)T * K; ++i) picks[ids[i]].push_back(i);
    std::vector<float> down((size_t)T * K * H);
    for (auto& kv : picks) {
        uint32_t e = kv.first;
        const std::vector<int64_t>& pl = kv.second;
        int ne = (int)pl.size();
        std::vector<float> xe((size_t)ne * H), g((size_t)ne * I), u((size_t)ne * I), h((size_t)ne * I), y((size_t)ne * H);
        for (int r = 0; r < ne; ++r) memcpy(&xe[(size_t)r * H], x + (pl[r] / K) * H, (size_t)H * 4);
        cwo_matmul(L->gate_type, mode, L->gate_bank, I, H, bpe_g, e, xe.data(), ne, g.data());
        cwo_matmul(L->up_type, mode, L->up_bank, I, H, bpe_u, e, xe.data(), ne, u.data());
        act_hidden(L, e, g.data(), u.data(), ne, h.data());
        cwo_matmul(L->down_type, mode, L->down_bank, H, I, bpe_d, e, h.data(), ne, y.data());
        for (int r = 0; r < ne; ++r)
            for (int c = 0; c < H; ++c) {
                float v = y[(size_t)r * H + c];
                if (L->act == CWO_ACT_CLAMPED_SWIGLU && L->down_b) v = v + L->down_b[(int64_t)e * H + c];
                down[(size_t)pl[r] * H + c] = v;
            }
    }
    std::vector<float> routed((size_t)T * H, 0.0f);
    if (mode == CWO_MODE_CANDLE) {
        for (auto& kv : picks)  // index_add in ascending expert order
            for (int64_t i : kv.second)
                for (int c = 0; c < H; ++c) routed[(size_t)(i / K) * H + c] += down[(size_t)i * H + c] * w[i];
    } else {
        for (int t = 0; t < T; ++t)
            for (int c = 0; c < H; ++c) {
                float acc = 0.0f;
                for (int j = 0; j < K; ++j) acc += down[((size_t)t * K + j) * H + c] * w[(size_t)t * K + j];
                routed[(size_t)t * H + c] = acc;
            }
    }
    std::vector<float> shared((size_t)T * H, 0.0f);
    if (L->shared_inter > 0) {
        int Is = L->shared_inter;
        int64_t sg = cwo_row_bytes(L->sh_gate_type, H) * Is, su = cwo_row_bytes(L->sh_up_type, H) * Is;
        int64_t sd = cwo_row_bytes(L->sh_down_type, Is) * H;
        std::vector<float> g((size_t)T * Is), u((size_t)T * Is), h((size_t)T * Is), y((size_t)T * H);
        cwo_matmul(L->sh_gate_type, mode, L->sh_gate, Is, H, sg, 0, x, T, g.data());
        cwo_matmul(L->sh_up_type, mode, L->sh_up, Is, H, su, 0, x, T, u.data());
        for (size_t i = 0; i < h.size(); ++i) h[i] = silu(g[i]) * u[i];
        cwo_matmul(L->sh_down_type, mode, L->sh_down, H, Is, sd, 0, h.data(), T, y.data());
        std::vector<float> prod((size_t)H);
        for (int t = 0; t < T; ++t) {
            for (int c = 0; c < H; ++c) prod[c] = x[(size_t)t * H + c] * L->sh_gate_inp[c];
            float gate = sigmoid(avx_sum(prod.data(), H));
            for (int c = 0; c < H; ++c) shared[(size_t)t * H + c] = y[(size_t)t * H + c] * gate;
        }
    }
    for (size_t i = 0; i < routed.size(); ++i) out[i] = routed[i] + shared[i];
    if (routed_out) memcpy(routed_out, routed.data(), routed.size() * 4);
    if (shared_out) memcpy(shared_out, shared.data(), shared.size() * 4);
    return 0;
}

// add_norm (fuse_kernel.rs:433-471) with candle-nn's CPU RmsNorm: the sum of squares is a plain
// left-to-right f32 sum (an iterator sum in the Rust source), then sqrt(sum2 / dim + eps) and
// v / m * alpha, every operation rounded to f32.
int cwo_add_rms_norm(const float* a, const float* b, const float* c, const float* alpha, float eps, int64_t rows,
                     int hidden, float* sum, float* out) {
    if (!a || !b || !alpha || !sum || !out || rows < 0 || hidden <= 0) return 1;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const size_t o = (size_t)r * hidden;
        float sum2 = 0.0f;
        for (int i = 0; i < hidden; ++i) {
            float v = a[o + i] + b[o + i];
            if (c) v = v + c[o + i];
            sum[o + i] = v;
            sum2 = sum2 + v * v;
        }
        const float m = sqrtf(sum2 / (float)hidden + eps);
        for (int i = 0; i < hidden; ++i) out[o + i] = sum[o + i] / m * alpha[i];
    }
    return 0;
}

}  // extern "C"
