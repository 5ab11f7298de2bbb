// Seeded synthetic weights and inputs, bit-identical on the host (C/C++) and the device (CUDA).
//
// Every value is a function of (stream, element index) alone, so any slice of any tensor can be
// regenerated independently on either side: the oracle rebuilds one expert of a 40-layer bank
// without touching the rest, and the GPU writes a whole bank in HBM in one pass.
//
//   normal(stream, i): SplitMix64 (Steele, Lea & Flood 2014) counter hashing -> two 24-bit
//   uniforms -> Box-Muller, evaluated in f32 with only IEEE basic operations (+ - * / sqrt),
//   each a separately rounded step. ln is the atanh series ln m = 2 atanh((m-1)/(m+1)) after
//   exponent extraction; sin/cos are Taylor series on [0, pi/4] after quadrant reduction. No
//   libm or CUDA math-library call is involved, so host and device agree bit for bit.
//
// These values define the synthetic workload; they are not a reference algorithm.
#pragma once
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define CWX_SHD __host__ __device__ __forceinline__
#else
#define CWX_SHD static inline
#endif

#if defined(__CUDA_ARCH__)
#define CWX_FMUL(a, b) __fmul_rn((a), (b))
#define CWX_FADD(a, b) __fadd_rn((a), (b))
#define CWX_FSUB(a, b) __fsub_rn((a), (b))
#define CWX_FDIV(a, b) __fdiv_rn((a), (b))
#define CWX_FSQRT(a) __fsqrt_rn((a))
#else
#include <math.h>
#define CWX_FMUL(a, b) ((float)((a) * (b)))
#define CWX_FADD(a, b) ((float)((a) + (b)))
#define CWX_FSUB(a, b) ((float)((a) - (b)))
#define CWX_FDIV(a, b) ((float)((a) / (b)))
#define CWX_FSQRT(a) sqrtf((a))
#endif

// Tensor tags: which tensor of a layer a stream belongs to.
enum {
    CWX_T_GATE_EXPS = 0,
    CWX_T_UP_EXPS = 1,
    CWX_T_DOWN_EXPS = 2,
    CWX_T_ROUTER_W = 3,
    CWX_T_ROUTER_B = 4,
    CWX_T_SH_GATE = 5,
    CWX_T_SH_UP = 6,
    CWX_T_SH_DOWN = 7,
    CWX_T_SH_GATE_INP = 8,
    CWX_T_GATE_B = 9,
    CWX_T_UP_B = 10,
    CWX_T_DOWN_B = 11,
    CWX_T_INPUT = 12,
};

CWX_SHD uint64_t cwx_splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// The stream of one tensor of one layer under a config seed.
CWX_SHD uint64_t cwx_stream(uint32_t seed, uint32_t layer, uint32_t tensor) {
    return cwx_splitmix64(((uint64_t)seed << 40) ^ ((uint64_t)layer << 16) ^ (uint64_t)tensor);
}

CWX_SHD uint32_t cwx_f2u(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}
CWX_SHD float cwx_u2f(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// ln(u) for u in [2^-24, 1], basic operations only.
CWX_SHD float cwx_ln(float u) {
    uint32_t b = cwx_f2u(u);
    int e = (int)((b >> 23) & 0xFF) - 126;  // u = m * 2^e, m in [0.5, 1)
    float m = cwx_u2f((b & 0x7FFFFFu) | (126u << 23));
    if (m < 0.70710677f) {
        m = CWX_FMUL(m, 2.0f);
        e -= 1;
    }
    float s = CWX_FDIV(CWX_FSUB(m, 1.0f), CWX_FADD(m, 1.0f));
    float s2 = CWX_FMUL(s, s);
    float p = CWX_FADD(0.111111111f, CWX_FMUL(s2, 0.0909090936f));  // 1/9 + s2/11
    p = CWX_FADD(0.142857149f, CWX_FMUL(s2, p));                        // 1/7
    p = CWX_FADD(0.200000003f, CWX_FMUL(s2, p));                        // 1/5
    p = CWX_FADD(0.333333343f, CWX_FMUL(s2, p));                        // 1/3
    p = CWX_FADD(1.0f, CWX_FMUL(s2, p));
    float lnm = CWX_FMUL(CWX_FMUL(2.0f, s), p);
    return CWX_FADD(CWX_FMUL((float)e, 0.693147182f), lnm);
}

// sin and cos of x in [0, pi/4] by Taylor series, basic operations only.
CWX_SHD void cwx_sincos_q(float x, float* s, float* c) {
    float x2 = CWX_FMUL(x, x);
    float ps = CWX_FADD(2.75573188e-06f, CWX_FMUL(x2, -2.50521084e-08f));  // 1/9! - x2/11!
    ps = CWX_FADD(-1.98412701e-04f, CWX_FMUL(x2, ps));                        // -1/7!
    ps = CWX_FADD(8.33333377e-03f, CWX_FMUL(x2, ps));                         // 1/5!
    ps = CWX_FADD(-0.166666672f, CWX_FMUL(x2, ps));                           // -1/3!
    *s = CWX_FADD(x, CWX_FMUL(CWX_FMUL(x, x2), ps));
    float pc = CWX_FADD(-2.75573188e-07f, CWX_FMUL(x2, 2.08767570e-09f));  // -1/10! + x2/12!
    pc = CWX_FADD(2.48015876e-05f, CWX_FMUL(x2, pc));                         // 1/8!
    pc = CWX_FADD(-1.38888892e-03f, CWX_FMUL(x2, pc));                        // -1/6!
    pc = CWX_FADD(4.16666679e-02f, CWX_FMUL(x2, pc));                         // 1/4!
    pc = CWX_FADD(-0.5f, CWX_FMUL(x2, pc));
    *c = CWX_FADD(1.0f, CWX_FMUL(x2, pc));
}

// cos and sin of 2*pi*f for f = k * 2^-24 in [0, 1).
CWX_SHD void cwx_sincos_turn(float f, float* sn, float* cs) {
    float t = CWX_FMUL(f, 4.0f);  // exact
    int q = (int)t;
    float r = CWX_FSUB(t, (float)q);  // exact, in [0, 1)
    float s, c;
    const float half_pi = 1.57079637f;
    if (r <= 0.5f) {
        cwx_sincos_q(CWX_FMUL(r, half_pi), &s, &c);
    } else {
        float cc, ss;
        cwx_sincos_q(CWX_FMUL(CWX_FSUB(1.0f, r), half_pi), &ss, &cc);
        s = cc;
        c = ss;
    }
    switch (q & 3) {
        case 0: *cs = c; *sn = s; break;
        case 1: *cs = -s; *sn = c; break;
        case 2: *cs = -c; *sn = -s; break;
        default: *cs = s; *sn = -c; break;
    }
}

// Element i of the standard-normal stream `key` (key = cwx_stream(...)).
CWX_SHD float cwx_normal(uint64_t key, uint64_t i) {
    uint64_t p = i >> 1;
    uint64_t r1 = cwx_splitmix64(key + 2 * p);
    uint64_t r2 = cwx_splitmix64(key + 2 * p + 1);
    float u1 = CWX_FMUL((float)((r1 >> 40) + 1), 5.96046448e-08f);  // (0, 1], exact
    float u2 = CWX_FMUL((float)(r2 >> 40), 5.96046448e-08f);        // [0, 1), exact
    float rad = CWX_FSQRT(CWX_FMUL(-2.0f, cwx_ln(u1)));
    float s, c;
    cwx_sincos_turn(u2, &s, &c);
    return CWX_FMUL(rad, (i & 1) ? s : c);
}

// std * normal, the N(0, std^2) draw the configs ask for.
CWX_SHD float cwx_normal_std(uint64_t key, uint64_t i, float std_) {
    return CWX_FMUL(std_, cwx_normal(key, i));
}

// Round-to-nearest-even f32 -> IEEE half bits, and back (exact), without library calls.
CWX_SHD uint16_t cwx_f32_to_f16_bits(float f) {
    uint32_t x = cwx_f2u(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | (ax > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to >= 65520 -> inf
    if (ax < 0x38800000u) {                                   // below 2^-14: subnormal half
        if (ax < 0x33000000u) return (uint16_t)sign;          // below 2^-25: rounds to 0
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126u - e;  // 14..25 -> value = m * 2^(e-150); half sub = q * 2^-24
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 112u;  // rebias 127 -> 15
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

CWX_SHD float cwx_f16_bits_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    if (e == 0) {
        if (m == 0) return cwx_u2f(sign);
        // subnormal: m * 2^-24
        float v = CWX_FMUL((float)m, 5.96046448e-08f);
        return sign ? -v : v;
    }
    if (e == 31) return cwx_u2f(sign | 0x7F800000u | (m << 13));
    return cwx_u2f(sign | ((e + 112u) << 23) | (m << 13));
}
