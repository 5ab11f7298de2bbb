// Argument blocks and host launchers of the cwx kernels (route.cu, gemv.cu, act.cu), used by
// api.cu.
#pragma once
#include "cwx_common.cuh"

namespace cwx {

struct MatRef {
    const uint8_t* base;  // tiled bank bytes
    Layout L;
};

// One matrix of a grouped-product launch.
struct GemvJob {
    MatRef m;
    int shared;         // 0: routed piles (rows by pick); 1: every token (the shared expert)
    const uint8_t* b;   // packed activation rows (act.cu), bstride bytes apart
    int64_t bstride;
    int bdiv;           // routed: activation row = pick index / bdiv
    const uint32_t* rowmap;  // or, when set: activation row = rowmap[pick index]
    float* out;         // output rows: pick index (routed) or token (shared)
    int64_t ostride;
    int split;          // products carried to ~22 bits (weights and activations as f16 hi + lo)
    int qint;           // activation rows hold Q8_K codes (f16 integers) and each piece's f32 scale
    const float* bias;  // (n_experts, n) added to the outputs, or NULL
    int rows;           // rows per work item (set by the launcher)
    int exact;          // the bank needs the exact path (an MXFP4 bank with cwx_bank::mx_wide)
};

struct GemvArgs {
    int njobs;
    GemvJob job[4];
    const uint32_t* pairs;
    const uint32_t* used3;  // (expert, first pair, count) per used expert
    const uint32_t* n_used;
    int s_count;  // tokens of the shared jobs
    int tok_est;   // upper bound on the picks of one expert (sizes the passes of small batches)
    int pile_est;  // average picks per expert (large piles take passes of 16 or 32 picks)
    int* err;
    // set by the launcher
    int tokcap;      // picks per pass
    int slot_bytes;   // weight bytes of one K-slice of a step
    int wslot_bytes;  // one weight slot (KS K-slices)
    int bslot_bytes;  // one activation slot (step header + activation rows)
    int nst;          // slots per ring
    int bhi;          // activation copies carry the hi halves only
    int brow;         // bytes from one activation row of a slot to the next
};

// Bytes of one packed activation row of k columns (1024 per 256-column piece).
__host__ __device__ inline int64_t packed_row_bytes(int64_t k) { return (k + PIECE_K - 1) / PIECE_K * 1024; }

int launch_router(const float* x, const float* w, const float* b, int T, int H, int E, float* logits,
                  cudaStream_t st);
int launch_route(const float* logits, int T, int E, int K, int norm, uint32_t* ids, float* w, const float* x,
                 const float* g_inp, int H, float* sgate, cudaStream_t st);
size_t perm_scratch_bytes(int64_t n, int E);
int perm_launches(int64_t n, int E);  // kernels launch_permute issues
// n_dev (optional, device): only the first *n_dev of the n pick slots are picks.
int launch_permute(const uint32_t* ids, int64_t n, int E, uint32_t* pairs, uint32_t* heads, uint32_t* used3,
                   uint32_t* n_used, uint32_t* scratch, int* err, cudaStream_t st, const int32_t* n_dev = nullptr);

// Activation preparation: rows (R, K) -> packed f16 hi/lo rows in the order the grouped products
// read. With `up` set, the input is the activation of (gate, up): SiLU, or clamped SwiGLU with
// per-expert biases (expert of row r = ids[r], rows being pick indices).
struct PrepArgs {
    const float* src;  // (R, K) f32: x, or gate outputs
    const float* up;   // (R, K) up outputs, or NULL
    int64_t R, K;
    int mode;          // ActMode
    int act;           // CWX_ACT_* when up is set
    float alpha, limit;
    const float* gate_b;
    const float* up_b;
    const uint32_t* ids;
    uint8_t* out;
};
int launch_prep(const PrepArgs& p, cudaStream_t st);
int launch_prep2(const PrepArgs* p, int njobs, cudaStream_t st);  // up to two preparations in one launch
int launch_combine(const float* rows, const float* w, int T, int K, int H, const float* shared, const float* sgate,
                   const float* residual, float* out, cudaStream_t st, const uint32_t* idx = nullptr);
// sum = a + b (+ c), out = rms_norm(sum) * alpha per row of H (act.cu).
int launch_add_norm(const float* a, const float* b, const float* c, const float* alpha, float eps, int64_t rows,
                    int H, float* sum, float* out, cudaStream_t st);
// launch_combine's sum into out, then norm_out = rms_norm(out) * alpha per token.
int launch_combine_norm(const float* rows, const float* w, int T, int K, int H, const float* shared,
                        const float* sgate, const float* residual, const float* alpha, float eps, float* out,
                        float* norm_out, cudaStream_t st, const uint32_t* idx = nullptr);

// Expert parallelism (ep.cu): units (token, destination rank) and their pick records.
struct EpOffsets {  // received records of source s: [pstart[s], pstart[s+1]); its units from ustart[s]
    int n;
    int64_t pstart[65];
    int64_t ustart[65];
};
// Dispatch: cnt/upos/pbase are (T, W) scratch; upos ends as each unit's index in the send buffer
// (-1: no picks there); tot (W, 2) = units and records per destination.
// cap > 0: the fixed-capacity layout (destination d's units from row d * cap, records from
// d * cap_rec); 0: destinations packed one after the other.
int launch_ep_units(const float* x, int T, int H, int K, int W, int epr, const int32_t* place, int E,
                    const uint32_t* ids, const float* w, int32_t* cnt, int32_t* upos, int32_t* pbase, int32_t* tot,
                    bool f16, void* send_rows, int32_t* send_picks, cudaStream_t st, int cap = 0, int cap_rec = 0);
// The fixed-capacity receive side: records packed into picks (count into n_picks), unit runs.
int launch_ep_recv_cap(const int32_t* picks, const int32_t* rcnt, int W, int cap, int cap_rec, uint32_t* rowmap,
                       uint32_t* eid, float* wgt, int32_t* first, int32_t* end, int32_t* n_picks, cudaStream_t st);
int launch_ep_unit_sum_cap(const float* y, const float* wgt, const int32_t* first, const int32_t* end,
                           const int32_t* rcnt, int W, int cap, int H, float* yu, cudaStream_t st);
int launch_ep_recv(const int32_t* picks, int64_t P, const EpOffsets& off, uint32_t* rowmap, uint32_t* eid,
                   float* wgt, int32_t* first, cudaStream_t st);
int launch_ep_unit_sum(const float* y, const float* wgt, const int32_t* first, int64_t U, int64_t P, int H, float* yu,
                       cudaStream_t st);
int launch_ep_combine(const float* back, const int32_t* unit, int T, int W, int H, const float* shared,
                      const float* sgate, const float* residual, float* out, cudaStream_t st);
int launch_f16_to_f32(const __half* x, int64_t n, float* y, cudaStream_t st);
// The library's expert-parallel transport (ep_nccl.cu).
int ep_comm_info(const cwx_ep_comm* c, int* world, int* rank, int* device);
int ep_comm_buffer(cwx_ep_comm* c, size_t bytes, cudaStream_t st, void** out);
int ep_comm_exchange(cwx_ep_comm* c, int nbuf, const void* const* send, void* const* recv, const size_t* bytes,
                     cudaStream_t st);
// experts_est: the number of experts expected to have picks (sizes the grid and the K split).
int launch_gemv(const GemvArgs& a, int64_t experts_est, int device, int sm_count, cudaStream_t st);

// The fused decode layer (decode_layer.cu): the whole layer of a small batch in one cooperative
// launch (router, route, piles, gate/up with the SiLU, down, combine), phases separated by two
// bounded grid-wide barriers.
constexpr int DL_MAX_T = 4;        // tokens
constexpr int DL_MAX_PICKS = 32;   // tokens x top_k
constexpr int DL_MAX_E = 512;      // routed experts
constexpr int DL_MAX_H = 2048;     // hidden (a multiple of 1024)
constexpr int DL_MAX_I = 1024;     // expert and shared intermediate
struct DecodeArgs {
    const float* x;         // (T, H)
    const float* residual;  // (T, H) or null
    float* out;             // (T, H)
    const float* norm_w;    // (H) the next layer's RMSNorm fused after the combine, or null
    float norm_eps;
    float* norm_out;        // (T, H)
    int norm_vec;           // out, norm_w and norm_out 16-byte aligned
    int T, H, E, K, I, Is, norm;
    const float* router_w;
    const float* router_b;
    MatRef gate, up, down;  // routed banks (IQ formats)
    MatRef sg, su, sd;      // shared expert (Q4_K) or base == null
    const float* sg_inp;
    int sh_qint;            // shared products on Q8_K activation codes (candle policy), else f16
    // workspace
    float* logits;          // (T, E)
    uint8_t* hpk;           // (T * K) hidden rows per pick: f16 (hi parts) in the packed order, 512 B per piece
    float* hs;              // (T, Is) shared hidden rows
    unsigned long long* bar;  // grid barrier counter: arrivals since it was zeroed (context creation, or
                              // a status read after a device error)
    int* err;
    // optional taps
    uint32_t* ids_out;
    float* w_out;
    uint32_t* pairs_out;
    uint32_t* heads_out;
};
// Whether the fused layer has an instantiation for these routed formats.
bool decode_fused_formats(int gate_fmt, int down_fmt);
int launch_decode_layer(const DecodeArgs& a, int device, int sm_count, cudaStream_t st);

// Tensor-core (tcgen05) expert products for large piles (mma.cu).
struct MmaArgs {
    MatRef a0, a1;       // weights; a1: the up matrix of a fused gate/up launch
    int fused;           // 1: gate/up rows side by side, SwiGLU epilogue writing f16 h rows
    const uint8_t* b;    // activation rows (f16), bstride bytes apart
    const uint8_t* blo;  // or null: the rows' lo parts (MXFP4 under the Q8_0 policy: x = hi + lo)
    int64_t bstride;
    int64_t brows;       // activation rows (their offsets must fit 32 bits)
    int bdiv;            // activation row = pair / bdiv
    const uint32_t* rowmap;  // or, when set: activation row = rowmap[pair]
    const uint32_t* pairs;
    const uint32_t* used3;
    const uint32_t* n_used;
    float* out;          // plain: f32 output rows per pick
    __half* hout;        // fused: f16 h rows per pick
    int64_t ostride;     // elements between output rows
    int* err;
    int mtiles;          // row tiles per expert (set by the launcher)
    // fused: the activation (CWX_ACT_SILU, or the clamped SwiGLU with its expert biases), and
    // whether h goes through Q8_0 (per 32 features) before f16, as the down products' input
    int act;
    float alpha, limit;
    const float* gate_b;
    const float* up_b;
    int h_q80;
    const float* bias;   // plain: expert bias added to each output row (E x n), or null
};
bool mma_supports(const MmaArgs& a);
int launch_mma(const MmaArgs& a, int device, int sm_count, cudaStream_t st);
int launch_f16rows(const float* x, int64_t n, __half* y, cudaStream_t st);
// x (rows of K, K a multiple of 32) through Q8_0 per 32 columns, then f16 (y), and the rest of
// each value as a second f16 (ylo, when not null; y + ylo is the Q8_0 value exactly).
int launch_f16rows_q80(const float* x, int64_t n, __half* y, __half* ylo, cudaStream_t st);
int launch_all_tokens(uint32_t* pairs, int T, uint32_t* used3, uint32_t* n_used, cudaStream_t st);

}  // namespace cwx
