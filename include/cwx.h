/* cwx: B200-native mixture-of-experts layer for coachwhip -- C ABI.
 *
 * The drop-in boundary for coachwhip's resident MoE path. Every entry point takes plain
 * pointers and sizes; device pointers are CUDA device addresses, `stream` is a cudaStream_t
 * passed as void* (NULL = the legacy default stream). Calls are stream-ordered and do not
 * synchronise unless documented. No call throws or aborts: each returns a cwx status code and
 * cwx_last_error() gives a thread-local message for the last failure.
 *
 * Reference interfaces replaced (paths inside the coachwhip tree):
 *   cwx_bank_create / cwx_bank_destroy
 *       ExpertStore::resident_op + exact_load   crates/engine/src/experts.rs:1949-1998, 98-119
 *   cwx_expert_matmul
 *       MoeMatvec::metal_fwd (CustomOp2)         crates/engine/src/experts.rs:2183-2309
 *   cwx_route
 *       route() / fuse_kernel::route             crates/engine/src/experts.rs:2364-2372,
 *                                                crates/engine/src/fuse_kernel.rs:20-75, 347-352
 *   cwx_permute
 *       fuse_kernel::piles (cw_pile)             crates/engine/src/fuse_kernel.rs:180-202, 567-582
 *   cwx_moe_forward
 *       StreamedMoe::forward, resident branch    crates/engine/src/experts.rs:2539-2614
 *       + SharedExpert::forward                  crates/engine/src/model_next.rs:731-741
 */
#ifndef CWX_H
#define CWX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define CWX_OK 0
#define CWX_EINVAL 1       /* bad argument: shape, null pointer, out-of-range value */
#define CWX_EUNSUPPORTED 2 /* quant type or shape this build does not handle */
#define CWX_ECUDA 3        /* a CUDA runtime call failed */
#define CWX_ETIMEOUT 4     /* a bounded device-side wait gave up (see cwx_ctx_status) */
#define CWX_ENOMEM 5       /* device or host allocation failed */
#define CWX_EDEVICE 6      /* a kernel recorded an error (bad expert id, shape) */
#define CWX_ECOMM 7        /* the expert-parallel transport (NCCL) failed */

/* GGUF tensor type ids (ggml_type) of the supported expert formats. */
#define CWX_TYPE_F32 0
#define CWX_TYPE_Q8_0 8
#define CWX_TYPE_Q4_K 12
#define CWX_TYPE_Q6_K 14
#define CWX_TYPE_IQ2_XXS 16
#define CWX_TYPE_IQ3_XXS 18
#define CWX_TYPE_IQ3_S 21
#define CWX_TYPE_IQ2_S 22
#define CWX_TYPE_IQ4_XS 23
#define CWX_TYPE_MXFP4 39

/* Activation policy of the expert products.
 * CANDLE: a matrix whose format has a CPU dot product in the reference (Q4_K, Q6_K: Q8_K;
 *         Q8_0, MXFP4: Q8_0) is multiplied with its activations quantised exactly as candle's
 *         CPU QMatMul does (k_quants.rs:2595-2603); IQ formats use f32 activations.
 * F32:    every matrix is multiplied with f32 activations (the reference's Metal semantics). */
#define CWX_ACT_MODE_CANDLE 0
#define CWX_ACT_MODE_F32 1

/* Expert activation (ExpertAct, crates/engine/src/experts.rs:2376-2385). */
#define CWX_ACT_SILU 0
#define CWX_ACT_CLAMPED_SWIGLU 1

typedef struct cwx_bank cwx_bank; /* one (n_experts, n, k) quantised expert matrix in HBM */
typedef struct cwx_ctx cwx_ctx;   /* a device binding: workspace, error word; one per thread */

/* Description of one expert matrix as stored in a GGUF file: n_experts x n rows x k columns,
 * rows = output features, each row k/block_elems quant blocks; bytes_per_expert = n * row bytes.
 * host_ptr points at n_experts * bytes_per_expert bytes (the tensor's data, verbatim). */
typedef struct {
    int32_t ggml_type;
    int64_t n;
    int64_t k;
    int64_t n_experts;
    int64_t bytes_per_expert;
    const void* host_ptr;
} cwx_matrix_desc;

const char* cwx_last_error(void);
int cwx_version(void);

/* Context: binds `device`, owns a growing workspace and a device error word. */
int cwx_ctx_create(int device, cwx_ctx** out);
int cwx_ctx_destroy(cwx_ctx* ctx);
/* Grow the workspace for up to `tokens` tokens of `layer` (call before stream capture). */
int cwx_ctx_reserve(cwx_ctx* ctx, const void* layer, int32_t tokens);
/* Synchronises `stream`, returns CWX_OK or the first device-side error recorded (and clears it). */
int cwx_ctx_status(cwx_ctx* ctx, void* stream);
/* Diagnostic of the failure path: one device-side wait, bounded like every wait of the library,
 * on a barrier that nothing completes. After limit_us (1 .. 1e6) it gives up and records the
 * timeout; the next cwx_ctx_status reports CWX_ETIMEOUT and clears it, and the context stays
 * usable. */
int cwx_ctx_check_wait(cwx_ctx* ctx, int32_t limit_us, void* stream);

/* Bank: copy a GGUF expert tensor into HBM (replaces ExpertStore::resident_op's exact_load).
 * IQ2_S, IQ3_S, IQ2_XXS, IQ3_XXS, IQ4_XS and MXFP4 banks are stored in 16-row groups and need a
 * multiple of 16 rows (CWX_EUNSUPPORTED otherwise). */
int cwx_bank_create(int device, const cwx_matrix_desc* desc, cwx_bank** out);
/* Bank filled on the device with the synthetic N(0, std^2) weights of stream `key`
 * (test and benchmark workloads; same values as the CPU generator). */
int cwx_bank_synth(cwx_ctx* ctx, int32_t ggml_type, int64_t n, int64_t k, int64_t n_experts, uint64_t key,
                   float std_, cwx_bank** out);
/* Experts [first, first + n_experts) of that synthetic tensor (an expert-parallel rank's slice;
 * the values follow the global expert index). */
int cwx_bank_synth_experts(cwx_ctx* ctx, int32_t ggml_type, int64_t n, int64_t k, int64_t first, int64_t n_experts,
                           uint64_t key, float std_, cwx_bank** out);
/* Synthetic bank of the listed experts (host array of count global expert indices), in list
 * order: the same weights as cwx_bank_synth's bank of all experts holds for them (an
 * expert-parallel rank's banks under a placement). */
int cwx_bank_synth_list(cwx_ctx* ctx, int32_t ggml_type, int64_t n, int64_t k, const int64_t* experts, int64_t count,
                        uint64_t key, float std_, cwx_bank** out);
int cwx_bank_destroy(cwx_bank* bank);
/* out[i] = std * N(0,1) element (offset + i) of stream `key`, i < n (synthetic router weights,
 * biases and inputs; same values as the CPU generator). */
int cwx_synth_normal(cwx_ctx* ctx, uint64_t key, uint64_t offset, int64_t n, float std_, float* out, void* stream);
/* Shape of a bank (host_ptr of the result is NULL). */
int cwx_bank_desc(const cwx_bank* bank, cwx_matrix_desc* out);
/* GGUF bytes of experts [e0, e0+ne) back into host memory (blocking). */
int cwx_bank_download(const cwx_bank* bank, int64_t e0, int64_t ne, void* host_dst);
/* Dequantised f32 rows of one expert, (n, k), into device memory. */
int cwx_bank_dequantize(const cwx_bank* bank, int64_t expert, float* out, void* stream);

/* GGUF files (replace candle's gguf_file::Content::read and tensor lookup,
 * vendor/candle-core/src/quantized/gguf_file.rs:469-563, as used by ExpertStore::new,
 * crates/engine/src/experts.rs:697-717, and the model loaders' metadata and dense-tensor reads,
 * crates/engine/src/model.rs:140-175, model_next.rs:1036-1053, model_gptoss.rs:115-175).
 * Versions 1-3; the file stays mapped read-only until cwx_gguf_close. Names are GGUF tensor
 * names ("blk.3.ffn_gate_exps.weight"); ne[] is innermost first (ne[0] = columns). */
typedef struct cwx_gguf cwx_gguf;
int cwx_gguf_open(const char* path, cwx_gguf** out);
int cwx_gguf_close(cwx_gguf* file);
/* version, tensor count, alignment and file offset of the tensor data (each optional). */
int cwx_gguf_info(const cwx_gguf* file, int32_t* version, int64_t* n_tensors, int64_t* alignment,
                  int64_t* data_offset);
/* ggml type, dimensions, ne[4] (unused dims 1) and the tensor's file offset (each optional). */
int cwx_gguf_tensor_info(const cwx_gguf* file, const char* name, int32_t* ggml_type, int32_t* n_dims, int64_t* ne,
                         int64_t* offset);
/* A 2-D (n, k) or 3-D (n_experts, n, k) tensor of an expert format as a bank descriptor whose
 * host_ptr points into the mapping (valid while the file is open). */
int cwx_gguf_tensor(const cwx_gguf* file, const char* name, cwx_matrix_desc* out);
/* Bank of experts [first, first + n_experts) of that tensor (n_experts < 0: through the last);
 * an expert-parallel rank loads its own slice. */
int cwx_bank_from_gguf(int device, const cwx_gguf* file, const char* name, int64_t first, int64_t n_experts,
                       cwx_bank** out);
/* An F32 / F16 / BF16 tensor of n elements as f32, into host memory (router weights and
 * biases, expert biases, the shared expert's gate). */
int cwx_gguf_tensor_f32(const cwx_gguf* file, const char* name, float* out, int64_t n);
/* Metadata values: any integer type (widened), F32/F64, strings (copied NUL-terminated into
 * buf of cap bytes, truncated to fit; *len = full length). */
int cwx_gguf_meta_int(const cwx_gguf* file, const char* key, int64_t* out);
int cwx_gguf_meta_f64(const cwx_gguf* file, const char* key, double* out);
int cwx_gguf_meta_str(const cwx_gguf* file, const char* key, char* buf, int64_t cap, int64_t* len);

/* route(): logits (tokens, n_experts) f32 -> ids (tokens, top_k) u32 best first (ties: lowest
 * id), weights (tokens, top_k) f32 = softmax over all experts, renormalised over the picks when
 * norm != 0. n_experts <= 1024, top_k <= 16. All device pointers. */
int cwx_route(cwx_ctx* ctx, const float* logits, int32_t tokens, int32_t n_experts, int32_t top_k, int32_t norm,
              uint32_t* ids, float* weights, void* stream);

/* Expert piles: ids (tokens, top_k) -> pairs (tokens*top_k) = flat pick indices t*top_k + j
 * grouped by expert, ascending pick index within an expert; heads (3*n_experts) = (e, first
 * pair, count) for every expert. Device pointers. An id >= n_experts records CWX_EDEVICE. */
int cwx_permute(cwx_ctx* ctx, const uint32_t* ids, int32_t tokens, int32_t top_k, int32_t n_experts,
                uint32_t* pairs, uint32_t* heads, void* stream);

/* cwx_permute for callers that must not allocate (no counterpart in the reference; it has no
 * such constraint). For code that cannot let a call allocate device memory: an engine whose own
 * pool owns all device memory, a loop that cannot take cudaMalloc's implicit device
 * synchronisation, or a caller without a cwx_ctx. Same pairs and heads as
 * cwx_permute; the scratch is a fixed 1 MiB device array of this library, so the call makes no
 * allocation. Limits: n_experts <= 4096 and
 * ceil(tokens*top_k / 1024) * n_experts + 3 * n_experts + 8 <= CWX_NOALLOC_SCRATCH_WORDS;
 * larger calls return CWX_EINVAL. Runs on the current device (stream must belong to it). The
 * array is shared per device, so calls on one device must not overlap (one stream, or ordered
 * streams); overlapping calls race. The first call on a device looks up the array's address:
 * make it outside stream capture. dev_status (optional device int) receives 0, or nonzero when
 * an id was >= n_experts. */
#define CWX_NOALLOC_SCRATCH_WORDS 262144
int cwx_permute_noalloc(const uint32_t* ids, int32_t tokens, int32_t top_k, int32_t n_experts, uint32_t* pairs,
                        uint32_t* heads, int32_t* dev_status, void* stream);

/* MoeMatvec: out (tokens, nei0, n) f32 = for each token t and pick j, one input row times the
 * bank matrix of expert ids[t][j]. x is (tokens, k) f32 when rows_per_expert == 0, else
 * (tokens*nei0, k) with one row per pick. act_mode: CWX_ACT_MODE_*. Device pointers. */
int cwx_expert_matmul(cwx_ctx* ctx, const cwx_bank* bank, const float* x, int32_t rows_per_expert,
                      const uint32_t* ids, int32_t tokens, int32_t nei0, int32_t act_mode, float* out,
                      void* stream);

/* One MoE layer's weights (all device pointers; banks from cwx_bank_*). */
typedef struct {
    int32_t hidden, n_experts, top_k, inter, norm_topk_prob;
    const float* router_w; /* (n_experts, hidden) f32 */
    const float* router_b; /* (n_experts) or NULL */
    const cwx_bank* gate;  /* (n_experts, inter, hidden) */
    const cwx_bank* up;    /* (n_experts, inter, hidden) */
    const cwx_bank* down;  /* (n_experts, hidden, inter) */
    int32_t act;           /* CWX_ACT_SILU / CWX_ACT_CLAMPED_SWIGLU */
    float alpha, limit;    /* clamped SwiGLU constants (1.702, 7.0 for gpt-oss) */
    const float* gate_b;   /* (n_experts, inter) or NULL */
    const float* up_b;     /* (n_experts, inter) or NULL */
    const float* down_b;   /* (n_experts, hidden) or NULL */
    const cwx_bank* sh_gate; /* shared expert (1, shared_inter, hidden), or NULL for none */
    const cwx_bank* sh_up;
    const cwx_bank* sh_down; /* (1, hidden, shared_inter) */
    const float* sh_gate_inp; /* (hidden) f32: sigmoid gate of the shared expert */
    int32_t act_mode;         /* CWX_ACT_MODE_* */
} cwx_moe_layer;

/* Per-call tensors (device pointers). x, out: (tokens, hidden) f32. residual: optional
 * (tokens, hidden) added to out. ids/weights/pairs/heads: optional taps of the routing. */
typedef struct {
    const float* x;
    int32_t tokens;
    float* out;
    const float* residual;
    uint32_t* ids_out;
    float* weights_out;
    uint32_t* pairs_out;
    uint32_t* heads_out;
    /* Optional: the next layer's RMSNorm fused after the combine, as the reference's residual
     * step does with add_norm (crates/engine/src/model_next.rs:1432-1436): with norm_w set,
     * norm_out (tokens, hidden) = rms_norm(out) * norm_w, norm_w (hidden) f32, norm_out a buffer
     * of its own. NULL norm_w: no norm (norm_eps and norm_out ignored). */
    const float* norm_w;
    float norm_eps;
    float* norm_out;
} cwx_moe_args;

/* out = routed experts (weighted) + shared expert * sigmoid(x . sh_gate_inp) (+ residual)
 * (+ norm_out = rms_norm(out) * norm_w when args->norm_w is set). */
int cwx_moe_forward(cwx_ctx* ctx, const cwx_moe_layer* layer, const cwx_moe_args* args, void* stream);

/* add_norm (crates/engine/src/fuse_kernel.rs:433-471): per row of `hidden`, sum = a + b (+ c)
 * and out = rms_norm(sum) * alpha, rms_norm as candle's RmsNorm (v / sqrt(mean(v^2) + eps)).
 * a, b, c (NULL for none), sum, out: (rows, hidden) f32 device; alpha (hidden) f32. sum may be
 * a, b or c (in place); out must be a buffer of its own. The reference's errors ("f32 only",
 * "metal only") have no analogue here: CWX_EINVAL for null pointers, rows < 0, hidden <= 0 or
 * out aliasing an input. */
int cwx_add_rms_norm(const float* a, const float* b, const float* c, const float* alpha, float eps, int64_t rows,
                     int32_t hidden, float* sum, float* out, void* stream);

/* The Gated DeltaNet mixer's middle for one word (the linear-attention step before the MoE block of
 * Qwen3-Next / Qwen3.5 / Qwen3.6 layers). The layer's constants: n_k key heads and n_v value heads
 * (n_v a multiple of n_k) of dims dk and dv; conv_w (channels, taps) with channels = 2 n_k dk +
 * n_v dv (q of all key heads, k of all key heads, v of all value heads); dt_bias, a (n_v); norm_w
 * (dv). cycle = 0: value head h reads key head h / (n_v / n_k) (Qwen3-Next's fused projection);
 * cycle = 1: key head h % n_k (Qwen3.5 / 3.6). The fields of the reference's GdnWord
 * (crates/engine/src/attn_kernel.rs:780-800) other than the per-word tensors. */
typedef struct cwx_gdn_layer {
    int32_t n_k, n_v, dk, dv, taps, cycle;
    float eps;
    const float* conv_w;
    const float* dt_bias;
    const float* a;
    const float* norm_w;
} cwx_gdn_layer;

/* coachwhip_gdn_word / gdn_word (crates/engine/src/attn_kernel.rs:24-143, 880-895) for one word of
 * each of n_seq independent sequences: conv over the window + SiLU, L2 norms of q and k, q scaled
 * by 1/sqrt(dk), beta = sigmoid(b), g = exp(softplus(alpha + dt_bias) * a), the delta rule on each
 * head's memory (S' = g S + k d^T, d = (v - g k.S) beta, o = q.S'), o RMS-normed times norm_w
 * times silu(z). Per sequence: qkv (channels), z (n_v dv), ba (2 n_v: the raw beta of every value
 * head, then the raw alpha), conv_state (taps - 1, channels), s (n_v, dk, dv); out: o (n_v dv),
 * s_out (n_v, dk, dv), conv_out (taps - 1, channels); sequences follow one another in each array.
 * All f32 device pointers. The reference's packed result is o | s_out | conv_out of one buffer.
 * s_out may be s (the memory updated in place); conv_out must be a buffer of its own (CWX_EINVAL).
 * CWX_EUNSUPPORTED for dk > 512 or dv > 256; CWX_EINVAL for bad dims, taps < 2, n_seq outside
 * 0 .. 65535 or null pointers. */
int cwx_gdn_word(const cwx_gdn_layer* layer, int32_t n_seq, const float* qkv, const float* z, const float* ba,
                 const float* conv_state, const float* s, float* o, float* s_out, float* conv_out, void* stream);

/* The gated full-attention layer's constants (FullAttn, crates/engine/src/model_next.rs:636-650):
 * n_head query heads over n_kv kv heads (n_head a multiple of n_kv, at most 16 per kv head), head
 * dim hd (64, 128 or 256), rope on the first rot values of each head (even, <= hd) with base
 * freq_base, q_norm_w and k_norm_w (hd) the per-head RmsNorm weights with eps. */
typedef struct cwx_attn_layer {
    int32_t n_head, n_kv, hd, rot;
    float eps;
    double freq_base;
    const float* q_norm_w;
    const float* k_norm_w;
} cwx_attn_layer;

/* FullAttn::forward for one word (crates/engine/src/model_next.rs:666-720, rope :653-664, KvBuf
 * append :74-130 without its roll) of each of n_seq sequences, between the projections:
 * q = q_norm(qg's first hd values per head), gate = its second hd values, k = k_norm(k_new), rope
 * (non-interleaved halves) on q and k at position pos[s], k and v_new appended to the caches at row
 * len[s], per query head softmax(q.K^T / sqrt(hd)) over rows 0 .. len[s] of its kv head (head h reads
 * kv head h / (n_head / n_kv)) times V, times sigmoid(gate). Per sequence: qg (n_head, 2 hd), k_new
 * and v_new (n_kv, hd), k_cache and v_cache (n_kv, cap, hd) 16-byte aligned, out (n_head hd); len and
 * pos (n_seq) int32 in device memory (read on the device, so a captured graph can replay with
 * moving lengths; the caller advances len). f32 device pointers; uses the context's workspace
 * (about n_seq (n_head hd + n_head ceil(cap/32) (hd + 2)) floats: call once outside a graph capture
 * so that it is there). Three launches (prep, chunks of 32 cache rows, merge). A len outside
 * 0 .. cap-1 skips that sequence and is reported by cwx_ctx_status as CWX_EDEVICE.
 * CWX_EUNSUPPORTED for other head dims or more than 16 query heads per kv head. */
int cwx_attn_word(cwx_ctx* ctx, const cwx_attn_layer* layer, int32_t n_seq, int32_t cap, const float* qg,
                  const float* k_new, const float* v_new, float* k_cache, float* v_cache, const int32_t* len,
                  const int32_t* pos, float* out, void* stream);

/* coachwhip_delta_word (crates/engine/src/delta_kernel.rs:20-50): the delta rule alone for one word,
 * in the reference's layout: qk (heads, 2 dk) q then k (already normed and scaled), vbd (heads,
 * dv + 2) v then beta then the decay g, s (heads, dk, dv); out (heads, dk dv + dv) the new memory
 * then the read-out o. f32 device pointers; out must not be s. CWX_EUNSUPPORTED for dk > 512. */
int cwx_delta_word(int32_t heads, int32_t dk, int32_t dv, const float* qk, const float* vbd, const float* s,
                   float* out, void* stream);

/* Expert parallelism (no counterpart in the reference, which runs one device): the experts are
 * split over `world` ranks, epr = n_experts / world each: contiguously (rank r owns experts
 * [r*epr, (r+1)*epr)) or, when the group carries a placement, expert e on rank placement[e] / epr
 * at local index placement[e] % epr (a permutation of 0 .. n_experts-1 in device memory, e.g. one
 * that balances the ranks' expected picks); every rank routes its own tokens. A token sends its row once to each rank that owns any of its picks (a
 * unit), with one record per pick: (unit index in that message, the expert's index on that rank,
 * the pick's weight) as three int32 (the weight's f32 bits). A layer is three calls around two
 * all-to-all exchanges the caller makes (NCCL, or any transport):
 *   1. cwx_ep_dispatch: router and route over all n_experts; for each destination d (in rank
 *      order) its units in token order and their records in pick order: send_counts[2d] units
 *      and send_counts[2d+1] records; unit_of (tokens, world) receives each token's unit index in
 *      send_rows per destination, or -1;
 *   (exchange send_counts, then the rows (unit splits) and the records (record splits))
 *   2. cwx_ep_experts: the received records through this rank's experts, then each unit's
 *      weighted sum in record order -> y_units (n_units, hidden) f32, in the order received;
 *      src_units / src_picks (host arrays of n_src) are the per-source counts received;
 *   (exchange y_units back with the reverse unit splits: each rank gets its units in send order)
 *   3. cwx_ep_combine: out[t] = sum over destinations in rank order of its returned unit rows,
 *      + shared expert (on the local tokens) * sgate, + residual.
 * Rows are f16 when cwx_ep_rows_f16(layer): IQ gate/up banks (their tensor-core products read
 * f16 activations) and a down matrix that takes f32 activations; else f32 (a down matrix that
 * re-quantises its input to Q8 would turn the f16 rounding into flipped codes). The layer's n_experts and router are global; its
 * banks (and expert biases) hold this rank's epr experts. send_rows holds up to
 * tokens * min(top_k, world) rows, send_picks tokens * top_k records. */
typedef struct {
    int32_t world, rank, experts_per_rank;
    const int32_t* placement; /* device array of n_experts slots, or NULL: contiguous ranges */
} cwx_ep_group;
int cwx_ep_rows_f16(const cwx_moe_layer* layer);
int cwx_ep_dispatch(cwx_ctx* ctx, const cwx_moe_layer* layer, const cwx_ep_group* group, const float* x,
                    int32_t tokens, uint32_t* ids, float* weights, float* sgate, int32_t* unit_of, void* send_rows,
                    int32_t* send_picks, int32_t* send_counts, void* stream);
int cwx_ep_experts(cwx_ctx* ctx, const cwx_moe_layer* layer, const cwx_ep_group* group, const void* rows,
                   const int32_t* picks, int32_t n_units, int32_t n_picks, int32_t n_src, const int32_t* src_units,
                   const int32_t* src_picks, float* y_units, void* stream);
int cwx_ep_combine(cwx_ctx* ctx, const cwx_moe_layer* layer, const cwx_ep_group* group, const float* x,
                   int32_t tokens, const int32_t* unit_of, const float* back_rows, const float* sgate,
                   const float* residual, float* out, void* stream);

/* Expert parallelism with the transport inside the library (no counterpart in the reference): an
 * NCCL communicator per rank (NCCL is bound at run time from libnccl.so.2; without it these calls
 * return CWX_EUNSUPPORTED). Rank 0 makes a unique id (128 bytes) and shares it with the others by
 * any host transport; every rank then creates its communicator (a collective call), or wraps an
 * ncclComm_t the caller already has (cwx_ep_comm_wrap; the caller keeps ownership).
 * cwx_ep_forward runs a whole expert-parallel layer on `stream`: dispatch (router, route, units),
 * one NCCL group exchanging the per-peer counts, unit rows and pick records, this rank's experts,
 * one NCCL group returning the unit sums, and the combine (+ shared expert on the local tokens,
 * + residual); out (tokens, hidden) f32. Exchanges have fixed per-peer sizes (cap_tokens units,
 * cap_tokens * min(top_k, experts per rank) records) and the receivers read the counts on the
 * device, so a layer never waits on the host. Every rank calls it for the same layer with the same
 * cap_tokens >= its own tokens (0 tokens allowed). ids_out (tokens, top_k), optional, receives the
 * local tokens' expert ids. The layer's banks hold this rank's experts, as for cwx_ep_dispatch. A
 * peer that stops calling makes the exchange wait: a watchdog thread may end it with
 * cwx_ep_comm_abort (the communicator is unusable afterwards). */
typedef struct cwx_ep_comm cwx_ep_comm;
int cwx_ep_unique_id(void* out, int64_t cap);
int cwx_ep_comm_create(int device, const void* unique_id, int32_t world, int32_t rank, cwx_ep_comm** out);
int cwx_ep_comm_wrap(void* nccl_comm, int32_t world, int32_t rank, int device, cwx_ep_comm** out);
int cwx_ep_comm_abort(cwx_ep_comm* comm);
int cwx_ep_comm_destroy(cwx_ep_comm* comm);
int cwx_ep_forward(cwx_ctx* ctx, cwx_ep_comm* comm, const cwx_moe_layer* layer, const cwx_ep_group* group,
                   const float* x, int32_t tokens, int32_t cap_tokens, const float* residual, float* out,
                   uint32_t* ids_out, void* stream);

/* Per-phase timing of cwx_moe_forward, the analogue of the reference's --profile Stats
 * (crates/engine/src/experts.rs:2541-2552): with profiling on, each call records a CUDA event
 * pair around every phase on its stream (also inside stream capture, where the events become
 * graph nodes and record again on every replay). */
#define CWX_PHASE_ROUTER 0  /* router logits */
#define CWX_PHASE_ROUTE 1   /* softmax, top-k, shared gate */
#define CWX_PHASE_PILES 2   /* permutation */
#define CWX_PHASE_PREP 3    /* activation preparation (all prep launches) */
#define CWX_PHASE_GATE_UP 4 /* gate/up expert products */
#define CWX_PHASE_DOWN 5    /* down expert products */
#define CWX_PHASE_COMBINE 6 /* weighted combine + shared expert + residual */
/* phases of cwx_ep_forward (its expert products also record GATE_UP / DOWN / PREP) */
#define CWX_PHASE_EP_DISPATCH 7  /* router, route and the units of every destination */
#define CWX_PHASE_EP_EXCHANGE 8  /* counts, unit rows and pick records to the peers (NCCL) */
#define CWX_PHASE_EP_EXPERTS 9   /* this rank's experts over the received records, unit sums */
#define CWX_PHASE_EP_RETURN 10   /* the unit sums back to their sources (NCCL) */
#define CWX_PHASE_EP_COMBINE 11  /* shared expert on the local tokens, combine, residual */
#define CWX_PHASE_DECODE_FUSED 12 /* the fused decode layer (every phase of a small batch in one launch) */
#define CWX_N_PHASES 13
int cwx_ctx_set_profiling(cwx_ctx* ctx, int enabled);
/* Layers whose routed banks are all IQ2_S / IQ3_S (SiLU, hidden and inter multiples of 256) run
 * their routed products on the tensor cores (tcgen05) when the batch gives at least min_pile
 * picks per expert on average (tokens * top_k / n_experts, rounded up); smaller batches use the
 * grouped mma.sync products. Default 32; 0 keeps every batch on the mma.sync products. */
int cwx_ctx_set_mma_min_pile(cwx_ctx* ctx, int min_pile);
/* Batches of up to max_tokens tokens (at most 4, and tokens * top_k <= 32) run the whole layer as
 * one cooperative launch (router, route, piles, gate/up with SiLU, down, combine; phases separated
 * by grid-wide barriers whose waits are bounded) when the layer allows it: SiLU, routed banks
 * IQ2_S gate/up with IQ3_S down (or IQ3_S / IQ2_S, IQ2_XXS / IQ3_XXS, IQ3_XXS / IQ2_XXS), hidden a
 * multiple of 256 up to 2048, inter and the shared expert's a multiple of 256 up to 1024, at most
 * 512 experts, a Q4_K shared expert or none (a fused RMSNorm is included). Default 4; 0 turns it off. Same
 * results as the general path within f32 rounding (ids, weights and piles identical). */
int cwx_ctx_set_fused_decode(cwx_ctx* ctx, int max_tokens);
/* Synchronises the device; adds each recorded phase's elapsed milliseconds into ms[phase] and
 * its occurrences into count[phase] (arrays of CWX_N_PHASES; either may be NULL); keeps the
 * recorded events, so a replayed graph can be read again after each replay. */
int cwx_ctx_read_profile(cwx_ctx* ctx, double* ms, int64_t* count);
/* Drops the recorded events. */
int cwx_ctx_reset_profile(cwx_ctx* ctx);
/* Kernel launches issued through this context since creation. */
int64_t cwx_ctx_launches(const cwx_ctx* ctx);

#ifdef __cplusplus
}
#endif

#endif /* CWX_H */
