// CPU oracle for the MoE hot path -- TEST INFRASTRUCTURE ONLY.
//
// A C++ restatement of the reference's arithmetic (candle CPU path and the Metal shader
// dequant for IQ types), used only by tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline as the checker. The product library (coachwhip_b200) never links or calls it.
//
// Two oracles, one per semantic the reference has:
//   O1 "candle CPU" (mode CWO_MODE_CANDLE): per matrix, activations quantised to the format's
//      VecDotType (Q8_K for K-quants, Q8_0 for Q8_0/MXFP4) and integer block dots
//      (vendor/candle-core/src/quantized/k_quants.rs:2551-2668). IQ types have no CPU path in
//      the reference (k_quants.rs:2955-2993 panic), so their matrices use O2 arithmetic.
//      Expert contributions summed in ascending expert order (experts.rs:2500-2537).
//   O2 "reference GPU" (mode CWO_MODE_F32): weights dequantised bit-exactly, f32 activations,
//      dot products accumulated in f64 and rounded once; picks summed in pick order
//      (fuse_kernel.rs:277-291).
//
// Parity pins: route() known answers from crates/engine/tests/router.rs and rank() order from
// crates/engine/tests/lookahead.rs; dequantisation of every format against ggml's gguf Python
// package (an independent implementation of the same formats). Quantisers (from_float) are
// restated from candle and unpinned by any reference test vector.
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    CWO_F32 = 0,
    CWO_Q8_0 = 8,
    CWO_Q4_K = 12,
    CWO_Q6_K = 14,
    CWO_Q8_K = 15,
    CWO_IQ2_XXS = 16,
    CWO_IQ3_XXS = 18,
    CWO_IQ3_S = 21,
    CWO_IQ2_S = 22,
    CWO_IQ4_XS = 23,
    CWO_MXFP4 = 39,
};

enum { CWO_MODE_CANDLE = 0, CWO_MODE_F32 = 1 };
enum { CWO_ACT_SILU = 0, CWO_ACT_CLAMPED_SWIGLU = 1 };

int cwo_block_elems(int type);
int cwo_block_bytes(int type);
int64_t cwo_row_bytes(int type, int64_t k);

// from_float for Q4_K, Q6_K, Q8_0, Q8_K, MXFP4 (candle); own encoder for IQ2_S, IQ3_S.
int cwo_quantize(int type, const float* x, int64_t n, void* out);
// to_float, bit-exact restatement.
int cwo_dequantize(int type, const void* blocks, int64_t n, float* y);
// vec_dot_unopt of one weight row against one row of activation blocks (the VecDotType).
float cwo_vec_dot(int type, int64_t n, const void* w_blocks, const void* act_blocks);
// VecDotType of a weight type (CWO_Q8_K, CWO_Q8_0) or CWO_F32 when the reference has no CPU dot.
int cwo_vec_dot_type(int type);

// Synthetic data (the same generator the library's bank synthesis uses).
uint64_t cwo_stream(uint32_t seed, uint32_t layer, uint32_t tensor);
void cwo_normal(uint64_t key, uint64_t offset, int64_t n, float std_, float* out);
// Quantised bytes of experts [e0, e0+ne) of an (E, n, k) tensor drawn N(0, std^2) from key.
int cwo_synth_matrix(int type, uint64_t key, int64_t e0, int64_t ne, int64_t n, int64_t k, float std_, void* out);

// Router logits (T, E) = x (T, H) . W (E, H)^T (+ b), products exact, f64 accumulation.
void cwo_router(const float* x, const float* w, const float* b, int T, int H, int E, float* logits);
// Router logits with every product and sum rounded to f32, in one of the summation orders an f32
// GEMV may use (the reference computes them with the gemm crate, whose order is not restated):
//   0 sequential, 1 sequential fused multiply-add, 2 eight strided lanes (AVX2) then a lane tree,
//   3 sixteen strided lanes (AVX-512) then a lane tree, 4 blocks of 256 columns with eight lanes
//   each, the block sums added in order (a K-blocked GEMM), 5 pairwise (recursive halves).
// Used by the routing-margin test, not by the layer oracle.
int cwo_router_f32(const float* x, const float* w, const float* b, int T, int H, int E, int order, float* logits);
// route(): softmax over all E, stable descending order, top k, renormalised when norm.
int cwo_route(const float* logits, int T, int E, int k, int norm, uint32_t* ids, float* w);
// Expert piles: pairs = flat pick indices i = t*k + j grouped stably by expert,
// heads[3e] = e, heads[3e+1] = first pair, heads[3e+2] = count, for every e < E.
int cwo_permute(const uint32_t* ids, int T, int k, int E, uint32_t* pairs, uint32_t* heads);

// out (rows, n) = x (rows, k) . W_e^T for expert e of a bank; mode CWO_MODE_CANDLE / _F32.
int cwo_matmul(int type, int mode, const void* bank, int64_t n, int64_t k, int64_t bytes_per_expert,
               uint32_t expert, const float* x, int rows, float* out);

typedef struct {
    int hidden, n_experts, top_k, inter, norm_topk_prob;
    const float* router_w;  // (E, H)
    const float* router_b;  // (E) or NULL
    int gate_type, up_type, down_type;
    const void* gate_bank;  // (E, inter, hidden) quantised
    const void* up_bank;
    const void* down_bank;  // (E, hidden, inter)
    int act;                // CWO_ACT_*
    float alpha, limit;
    const float* gate_b;  // (E, inter) or NULL
    const float* up_b;
    const float* down_b;  // (E, hidden)
    int shared_inter;     // 0 = no shared expert
    int sh_gate_type, sh_up_type, sh_down_type;
    const void* sh_gate;
    const void* sh_up;
    const void* sh_down;
    const float* sh_gate_inp;  // (H)
} cwo_moe_layer;

// One MoE layer. routed (T, H) and shared (T, H) may be NULL; ids/w (T, k) may be NULL.
// out (T, H) = routed + shared contribution.
int cwo_moe_forward(const cwo_moe_layer* L, const float* x, int T, int mode, float* out, float* routed,
                    float* shared, uint32_t* ids, float* w);

// The same layer (candle policy, SiLU layers) vectorised for speed: the timed CPU baseline, not
// a checker (oracle/fast.cpp). out (T, H).
int cwo_moe_forward_fast(const cwo_moe_layer* L, const float* x, int T, float* out);

// add_norm (crates/engine/src/fuse_kernel.rs:433-471, the residual step of model_next.rs:1432-1436
// and its unfused form ((routed + shared) + h, then the next layer's RmsNorm)): per row of
// `hidden`, sum = (a + b) + c (c may be NULL) and out = rms_norm(sum) * alpha with candle-nn's
// CPU RmsNorm arithmetic: sum2 = sequential f32 sum of v * v, m = sqrt(sum2 / hidden + eps),
// out = v / m * alpha.
/* Gated DeltaNet word step (gdn.cpp): the reference's one-kernel step (attn_kernel.rs:24-143) for
 * one word of one sequence, its op-by-op form (model_next.rs:581-620), and the word-by-word delta
 * rule (model_next.rs:17-38) over l words (s updated in place). */
int cwo_gdn_word(int n_k, int n_v, int dk, int dv, int taps, int cycle, float eps, const float* qkv, const float* z,
                 const float* ba, const float* conv_state, const float* conv_w, const float* dt_bias,
                 const float* a_vec, const float* norm_w, const float* s, float* o, float* s_out, float* conv_out);
int cwo_gdn_word_ops(int n_k, int n_v, int dk, int dv, int taps, int cycle, float eps, const float* qkv,
                     const float* z, const float* ba, const float* conv_state, const float* conv_w,
                     const float* dt_bias, const float* a_vec, const float* norm_w, const float* s, float* o,
                     float* s_out, float* conv_out);
int cwo_delta_steps(int l, int n_v, int dk, int dv, const float* q, const float* k, const float* v, const float* beta,
                    const float* log_decay, float* s, float* o);
/* Full-attention word step (gdn.cpp): FullAttn::forward for one word of one sequence
 * (model_next.rs:666-720); k_cache / v_cache (n_kv, cap, hd) get the new row at len. */
int cwo_attn_word(int n_head, int n_kv, int hd, int rot, float eps, double freq_base, int cap, int len, int pos,
                  const float* qg, const float* k_new, const float* v_new, const float* q_norm_w,
                  const float* k_norm_w, float* k_cache, float* v_cache, float* out);
int cwo_add_rms_norm(const float* a, const float* b, const float* c, const float* alpha, float eps, int64_t rows,
                     int hidden, float* sum, float* out);

// Threads used by the OpenMP regions (0 = runtime default).
void cwo_set_threads(int n);
int cwo_get_threads(void);

#ifdef __cplusplus
}
#endif
