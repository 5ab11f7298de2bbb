// Oracle internals -- TEST INFRASTRUCTURE ONLY. GGUF block structs (candle k_quants.rs:89-200,
// 631-635; repr(C) layouts) and the per-format routines of formats.cpp.
#pragma once
#include <stdint.h>

namespace cwo {

#pragma pack(push, 1)
struct BQ4K {
    uint16_t d, dmin;
    uint8_t scales[12];
    uint8_t qs[128];
};
struct BQ6K {
    uint8_t ql[128];
    uint8_t qh[64];
    int8_t scales[16];
    uint16_t d;
};
struct BQ8_0 {
    uint16_t d;
    int8_t qs[32];
};
struct BMXFP4 {
    uint8_t e;
    uint8_t qs[16];
};
#pragma pack(pop)
struct BQ8K {
    float d;
    int8_t qs[256];
    int16_t bsums[16];
};
static_assert(sizeof(BQ4K) == 144, "Q4_K block");
static_assert(sizeof(BQ6K) == 210, "Q6_K block");
static_assert(sizeof(BQ8_0) == 34, "Q8_0 block");
static_assert(sizeof(BMXFP4) == 17, "MXFP4 block");
static_assert(sizeof(BQ8K) == 292, "Q8_K block");

void q8k_from_float(const float* x, BQ8K* y);
void q8_0_from_float(const float* x, BQ8_0* y);
const uint16_t* iq3s_map();
const uint16_t* iq2s_map();
const uint16_t* iq3xxs_map();
const uint16_t* iq2xxs_map();

// candle's x86 AVX f32 sum (vendor/candle-core/src/cpu/avx.rs:243-257 with vec_reduce 51-66):
// 4 x 8 lanes over whole 32-element steps, the fixed pairwise lane reduction, then the tail
// added one by one. Used by softmax and by sum_keepdim on contiguous rows.
float avx_sum(const float* x, int n);

}  // namespace cwo
