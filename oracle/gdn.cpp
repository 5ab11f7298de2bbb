// CPU oracle of the attention steps before the MoE block -- TEST INFRASTRUCTURE ONLY (the checker
// of cwx_gdn_word / cwx_delta_word / cwx_attn_word; the product library never links it).
//
// cwo_gdn_word restates the reference's one-kernel word step, coachwhip_gdn_word
// (crates/engine/src/attn_kernel.rs:24-143), as its threadgroups compute it, one value head after
// another, in f32 with every sum taken in the kernel's own order (one thread per column, the norms
// summed by thread 0 from i = 0 up). The reference builds that Metal source with the default
// compile options, so its own bits depend on Apple's compiler (fast math); this restatement rounds
// each operation as written (-ffp-contract=off) and is the f32 semantics the GPU is held to within
// a stated tolerance, not bit for bit.
//
// cwo_delta_steps restates the op-by-op delta rule of model_next.rs:17-38 (delta_steps, the path
// crates/engine/tests/linear_attention.rs:24-41 holds as the word-by-word truth): per word
// S = g S, sk = k S, d = (v - sk) beta, S = S + k^T d, o = q S.
//
// cwo_gdn_word_ops restates the op-by-op layer middle of LinearAttn::forward for one word
// (model_next.rs:581-620): sigmoid / softplus gates, the window conv (oldest row first), SiLU, l2_norm
// then 1/sqrt(dk) on q, delta_steps, then candle's RmsNorm (x / sqrt(mean(x^2) + eps) * w) and the
// SiLU gate. The reference states that its fused kernel keeps the op-by-op arithmetic; the tests
// check the two restatements against each other.
//
// cwo_attn_word (below) restates the gated full-attention word step.
//
// Parity unpinned at the bit level: the reference holds no vectors for these steps and its kernels
// run on Metal only.
#include <math.h>
#include <string.h>

#include <vector>

#include "cw_oracle.h"

static float silu_f(float x) { return x / (1.0f + expf(-x)); }

extern "C" int cwo_gdn_word(int n_k, int n_v, int dk, int dv, int taps, int cycle, float eps, const float* qkv,
                            const float* z, const float* ba, const float* conv_state, const float* conv_w,
                            const float* dt_bias, const float* a_vec, const float* norm_w, const float* s, float* o,
                            float* s_out, float* conv_out) {
    if (n_k < 1 || n_v < 1 || n_v % n_k || dk < 1 || dv < 1 || taps < 2) return 1;
    const int channels = 2 * n_k * dk + n_v * dv;
    const int per_group = n_v / n_k;
    std::vector<float> q_sh(dk), k_sh(dk);
    for (int h = 0; h < n_v; ++h) {
        const int kh = cycle ? h % n_k : h / per_group;
        // 1. conv + silu of the head's q, k channels; the window moves one word on
        for (int i = 0; i < dk; ++i) {
            const int cq = kh * dk + i, ck = n_k * dk + kh * dk + i;
            float xq = 0.0f, xk = 0.0f;
            for (int t = 0; t + 1 < taps; ++t) {
                xq += conv_w[(size_t)cq * taps + t] * conv_state[(size_t)t * channels + cq];
                xk += conv_w[(size_t)ck * taps + t] * conv_state[(size_t)t * channels + ck];
            }
            xq += conv_w[(size_t)cq * taps + taps - 1] * qkv[cq];
            xk += conv_w[(size_t)ck * taps + taps - 1] * qkv[ck];
            q_sh[i] = silu_f(xq);
            k_sh[i] = silu_f(xk);
            for (int t = 0; t + 2 < taps; ++t) {
                conv_out[(size_t)t * channels + cq] = conv_state[(size_t)(t + 1) * channels + cq];
                conv_out[(size_t)t * channels + ck] = conv_state[(size_t)(t + 1) * channels + ck];
            }
            conv_out[(size_t)(taps - 2) * channels + cq] = qkv[cq];
            conv_out[(size_t)(taps - 2) * channels + ck] = qkv[ck];
        }
        // 2. L2 norms (thread 0's sequential sums), query scale
        float sq = 0.0f, sk = 0.0f;
        for (int i = 0; i < dk; ++i) {
            sq += q_sh[i] * q_sh[i];
            sk += k_sh[i] * k_sh[i];
        }
        const float rq = sqrtf(sq + eps), rk = sqrtf(sk + eps);
        const float qscale = 1.0f / (rq * sqrtf((float)dk));
        const float kscale = 1.0f / rk;
        for (int i = 0; i < dk; ++i) {
            q_sh[i] *= qscale;
            k_sh[i] *= kscale;
        }
        // 3. gates
        const float beta = 1.0f / (1.0f + expf(-ba[h]));
        const float alpha = ba[n_v + h];
        const float g = expf(logf(expf(alpha + dt_bias[h]) + 1.0f) * a_vec[h]);
        // 4. the delta rule, one column at a time
        const float* sh = s + (size_t)h * dk * dv;
        float* so = s_out + (size_t)h * dk * dv;
        for (int j = 0; j < dv; ++j) {
            const int cv = 2 * n_k * dk + h * dv + j;
            float xv = 0.0f;
            for (int t = 0; t + 1 < taps; ++t) xv += conv_w[(size_t)cv * taps + t] * conv_state[(size_t)t * channels + cv];
            xv += conv_w[(size_t)cv * taps + taps - 1] * qkv[cv];
            const float v = silu_f(xv);
            for (int t = 0; t + 2 < taps; ++t)
                conv_out[(size_t)t * channels + cv] = conv_state[(size_t)(t + 1) * channels + cv];
            conv_out[(size_t)(taps - 2) * channels + cv] = qkv[cv];
            float skv = 0.0f;
            for (int i = 0; i < dk; ++i) skv += k_sh[i] * sh[(size_t)i * dv + j];
            skv *= g;
            const float d = (v - skv) * beta;
            float acc = 0.0f;
            for (int i = 0; i < dk; ++i) {
                const float ns = g * sh[(size_t)i * dv + j] + k_sh[i] * d;
                so[(size_t)i * dv + j] = ns;
                acc += q_sh[i] * ns;
            }
            o[(size_t)h * dv + j] = acc;
        }
        // 5. output RMS norm and silu gate
        float ss = 0.0f;
        for (int j = 0; j < dv; ++j) {
            const float x = o[(size_t)h * dv + j];
            ss += x * x;
        }
        const float rms = 1.0f / sqrtf(ss / (float)dv + eps);
        for (int j = 0; j < dv; ++j) {
            const float x = o[(size_t)h * dv + j] * rms * norm_w[j];
            o[(size_t)h * dv + j] = x * silu_f(z[(size_t)h * dv + j]);
        }
    }
    return 0;
}

extern "C" int cwo_delta_steps(int l, int n_v, int dk, int dv, const float* q, const float* k, const float* v,
                               const float* beta, const float* log_decay, float* s, float* o) {
    if (l < 0 || n_v < 1 || dk < 1 || dv < 1) return 1;
    std::vector<float> sk(dv), d(dv);
    for (int t = 0; t < l; ++t) {
        for (int h = 0; h < n_v; ++h) {
            const float* qt = q + ((size_t)t * n_v + h) * dk;
            const float* kt = k + ((size_t)t * n_v + h) * dk;
            const float* vt = v + ((size_t)t * n_v + h) * dv;
            const float bt = beta[(size_t)t * n_v + h];
            const float gt = expf(log_decay[(size_t)t * n_v + h]);
            float* sh = s + (size_t)h * dk * dv;
            for (size_t e = 0; e < (size_t)dk * dv; ++e) sh[e] = sh[e] * gt;
            for (int j = 0; j < dv; ++j) {
                float acc = 0.0f;
                for (int i = 0; i < dk; ++i) acc += kt[i] * sh[(size_t)i * dv + j];
                sk[j] = acc;
                d[j] = (vt[j] - sk[j]) * bt;
            }
            for (int i = 0; i < dk; ++i)
                for (int j = 0; j < dv; ++j) sh[(size_t)i * dv + j] = sh[(size_t)i * dv + j] + kt[i] * d[j];
            float* ot = o + ((size_t)t * n_v + h) * dv;
            for (int j = 0; j < dv; ++j) {
                float acc = 0.0f;
                for (int i = 0; i < dk; ++i) acc += qt[i] * sh[(size_t)i * dv + j];
                ot[j] = acc;
            }
        }
    }
    return 0;
}

extern "C" int cwo_gdn_word_ops(int n_k, int n_v, int dk, int dv, int taps, int cycle, float eps, const float* qkv,
                                const float* z, const float* ba, const float* conv_state, const float* conv_w,
                                const float* dt_bias, const float* a_vec, const float* norm_w, const float* s,
                                float* o, float* s_out, float* conv_out) {
    if (n_k < 1 || n_v < 1 || n_v % n_k || dk < 1 || dv < 1 || taps < 2) return 1;
    const int channels = 2 * n_k * dk + n_v * dv;
    const int per_group = n_v / n_k;
    // gates: beta = sigmoid(b), log decay = softplus(alpha + dt_bias) * A
    std::vector<float> beta(n_v), log_decay(n_v);
    for (int h = 0; h < n_v; ++h) {
        beta[h] = 1.0f / (1.0f + expf(-ba[h]));
        log_decay[h] = logf(expf(ba[n_v + h] + dt_bias[h]) + 1.0f) * a_vec[h];
    }
    // window conv, oldest row first, then SiLU; the window keeps the last taps - 1 rows
    std::vector<float> conv(channels);
    for (int c = 0; c < channels; ++c) {
        float acc = conv_state[c] * conv_w[(size_t)c * taps];
        for (int w = 1; w < taps; ++w) {
            const float x = w + 1 < taps ? conv_state[(size_t)w * channels + c] : qkv[c];
            acc = acc + x * conv_w[(size_t)c * taps + w];
        }
        conv[c] = silu_f(acc);
        for (int t = 0; t + 2 < taps; ++t) conv_out[(size_t)t * channels + c] = conv_state[(size_t)(t + 1) * channels + c];
        conv_out[(size_t)(taps - 2) * channels + c] = qkv[c];
    }
    // l2_norm of q and k per key head, widened to the value heads; q times 1/sqrt(dk)
    std::vector<float> qn((size_t)n_k * dk), kn((size_t)n_k * dk);
    for (int kh = 0; kh < n_k; ++kh) {
        for (int which = 0; which < 2; ++which) {
            const float* x = conv.data() + (size_t)which * n_k * dk + (size_t)kh * dk;
            float ss = 0.0f;
            for (int i = 0; i < dk; ++i) ss += x[i] * x[i];
            const float n = sqrtf(ss + eps);
            float* y = (which ? kn.data() : qn.data()) + (size_t)kh * dk;
            for (int i = 0; i < dk; ++i) y[i] = x[i] / n;
        }
    }
    const float qs = (float)(1.0 / sqrt((double)dk));
    std::vector<float> q((size_t)n_v * dk), k((size_t)n_v * dk), v((size_t)n_v * dv);
    for (int h = 0; h < n_v; ++h) {
        const int kh = cycle ? h % n_k : h / per_group;
        for (int i = 0; i < dk; ++i) {
            q[(size_t)h * dk + i] = qn[(size_t)kh * dk + i] * qs;
            k[(size_t)h * dk + i] = kn[(size_t)kh * dk + i];
        }
        for (int j = 0; j < dv; ++j) v[(size_t)h * dv + j] = conv[(size_t)2 * n_k * dk + (size_t)h * dv + j];
    }
    memcpy(s_out, s, sizeof(float) * (size_t)n_v * dk * dv);
    cwo_delta_steps(1, n_v, dk, dv, q.data(), k.data(), v.data(), beta.data(), log_decay.data(), s_out, o);
    // RmsNorm over each head's dv values, times the SiLU gate
    for (int h = 0; h < n_v; ++h) {
        float* x = o + (size_t)h * dv;
        float ss = 0.0f;
        for (int j = 0; j < dv; ++j) ss += x[j] * x[j];
        const float r = sqrtf(ss / (float)dv + eps);
        for (int j = 0; j < dv; ++j) x[j] = (x[j] / r) * norm_w[j] * silu_f(z[(size_t)h * dv + j]);
    }
    return 0;
}

// ---------------------------------------------------------------- full attention, one word
// FullAttn::forward for one word of one sequence (crates/engine/src/model_next.rs:666-720): the
// per-head RmsNorm of q and k (candle's x / sqrt(mean(x^2) + eps) * w, the squares summed in
// order), rope on the first rot values (rope :653-664: inverse frequencies 1 / base^(2i/rot) in f64
// rounded to f32, angle pos * inv in f32, candle's non-interleaved rope: x1 cos - x2 sin,
// x1 sin + x2 cos), the new row appended to the cache (KvBuf::append without its roll), then per
// query head the scores q.k in order times 1/sqrt(hd) (an f32 scalar), softmax (max, exp(s - max),
// sum in order, divide), the probabilities times V summed over the rows in order, times
// sigmoid(gate). k_cache, v_cache (n_kv, cap, hd) are updated at row len.
static void norm_rope(const float* x, const float* w, int hd, int rot, float eps, double base, int pos, float* y) {
    float ss = 0.0f;
    for (int d = 0; d < hd; ++d) ss += x[d] * x[d];
    const float m = sqrtf(ss / (float)hd + eps);
    for (int d = 0; d < hd; ++d) y[d] = x[d] / m * w[d];
    const int half = rot / 2;
    for (int i = 0; i < half; ++i) {
        const float inv = (float)(1.0 / pow(base, 2.0 * i / (double)rot));
        const float f = (float)pos * inv;
        const float c = cosf(f), s = sinf(f);
        const float a = y[i], b = y[i + half];
        y[i] = a * c - b * s;
        y[i + half] = a * s + b * c;
    }
}

extern "C" int cwo_attn_word(int n_head, int n_kv, int hd, int rot, float eps, double freq_base, int cap, int len,
                             int pos, const float* qg, const float* k_new, const float* v_new, const float* q_norm_w,
                             const float* k_norm_w, float* k_cache, float* v_cache, float* out) {
    if (n_head < 1 || n_kv < 1 || n_head % n_kv || hd < 1 || rot < 0 || rot > hd || rot % 2 || len < 0 || len >= cap)
        return 1;
    const int g = n_head / n_kv;
    const float scale = (float)(1.0 / sqrt((double)hd));
    std::vector<float> q(hd), sc(len + 1);
    for (int kv = 0; kv < n_kv; ++kv) {
        float* kr = k_cache + ((size_t)kv * cap + len) * hd;
        norm_rope(k_new + (size_t)kv * hd, k_norm_w, hd, rot, eps, freq_base, pos, kr);
        memcpy(v_cache + ((size_t)kv * cap + len) * hd, v_new + (size_t)kv * hd, sizeof(float) * hd);
    }
    for (int h = 0; h < n_head; ++h) {
        const int kv = h / g;
        norm_rope(qg + (size_t)h * 2 * hd, q_norm_w, hd, rot, eps, freq_base, pos, q.data());
        const float* K = k_cache + (size_t)kv * cap * hd;
        const float* V = v_cache + (size_t)kv * cap * hd;
        float m = -INFINITY;
        for (int p = 0; p <= len; ++p) {
            float s = 0.0f;
            for (int d = 0; d < hd; ++d) s += q[d] * K[(size_t)p * hd + d];
            sc[p] = s * scale;
            m = fmaxf(m, sc[p]);
        }
        float sum = 0.0f;
        for (int p = 0; p <= len; ++p) {
            sc[p] = expf(sc[p] - m);
            sum += sc[p];
        }
        for (int p = 0; p <= len; ++p) sc[p] = sc[p] / sum;
        const float* gate = qg + (size_t)h * 2 * hd + hd;
        for (int d = 0; d < hd; ++d) {
            float acc = 0.0f;
            for (int p = 0; p <= len; ++p) acc += sc[p] * V[(size_t)p * hd + d];
            out[(size_t)h * hd + d] = acc * (1.0f / (1.0f + expf(-gate[d])));
        }
    }
    return 0;
}
