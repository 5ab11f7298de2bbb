// Argument blocks and host launchers of the cwx kernels (route.cu, gemv.cu), used by api.cu.
#pragma once
#include "cwx_common.cuh"

namespace cwx {

struct MatRef {
    const uint8_t* base;  // tiled bank bytes
    Layout L;
};

// One grouped-product launch: routed piles of one or two matrices (+ optional shared expert).
struct GemvArgs {
    int two;  // 1: gate and up (+ activation) -> hidden rows; 0: one matrix -> output rows
    MatRef ra, rb;
    const __half* rbh;  // activation rows (hi part), f16, (rows, K)
    const __half* rbl;  // activation rows (lo part)
    int64_t r_bstride;
    int r_bdiv;  // activation row = pick index / r_bdiv
    float* rout;
    int64_t r_ostride;
    const uint32_t* pairs;
    const uint32_t* used3;  // (expert, first pair, count) per used expert
    const uint32_t* n_used;
    int has_shared;
    MatRef sa, sb;
    const __half* sbh;
    const __half* sbl;
    int64_t s_bstride;
    float* sout;
    int64_t s_ostride;
    int s_count;
    int act;
    float alpha, limit;
    const float* gate_b;
    const float* up_b;
    const float* down_b;
    int split_r, split_s;  // weights carried as an f16 hi + lo pair (routed, shared items)
    int* err;
    int stage_bytes;  // set by launch_gemv
    int stage_b_off;
    int nst;
};

int launch_router(const float* x, const float* w, const float* b, int T, int H, int E, float* logits,
                  cudaStream_t st);
int launch_route(const float* logits, int T, int E, int K, int norm, uint32_t* ids, float* w, const float* x,
                 const float* g_inp, int H, float* sgate, cudaStream_t st);
size_t perm_scratch_bytes(int64_t n, int E);
int launch_permute(const uint32_t* ids, int64_t n, int E, uint32_t* pairs, uint32_t* heads, uint32_t* used3,
                   uint32_t* n_used, uint32_t* scratch, int* err, cudaStream_t st);
int launch_prep(const float* src, int64_t R, int64_t K, int mode, __half* hi, __half* lo, cudaStream_t st);
int launch_combine(const float* rows, const float* w, int T, int K, int H, const float* shared, const float* sgate,
                   const float* residual, float* out, cudaStream_t st);
int launch_gemv(GemvArgs a, int64_t max_items, int device, int sm_count, cudaStream_t st);

}  // namespace cwx
