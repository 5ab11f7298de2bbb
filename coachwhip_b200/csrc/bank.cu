// Expert banks in HBM: upload of GGUF bytes into the tiled layout, synthetic banks generated on
// the device, download back to GGUF order, and dequantisation for checks.
//
// The upload replaces ExpertStore::resident_op's whole-tensor read and exact_load
// (crates/engine/src/experts.rs:1949-1998, 98-119): the bytes of every expert are copied once and
// stay resident; only their order changes (64-row x 256-column pieces, see cwx_common.cuh).
//
// The synthetic generator quantises with the same arithmetic as candle's from_float for Q4_K,
// Q6_K, Q8_0 and MXFP4 (vendor/candle-core/src/quantized/k_quants.rs:1694-1753, 2267-2337,
// 784-820, 694-731; utils.rs:62-284) and with the project's own IQ2_S/IQ3_S encoder
// (iq_encode.h). This file is compiled with -fmad=false so each f32 step rounds as in the Rust
// code; the bytes equal the CPU generator's.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "cwx_common.cuh"
#include "decode.cuh"
#include "iq_encode.h"
#include "synth_math.h"

namespace cwx {

// ---------------------------------------------------------------- layout copies
// One warp per (expert, row): move the row's bytes between GGUF order and the tiled layout.
__global__ void k_repack(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, Layout L, int64_t e0,
                         int64_t ne, int to_tiled) {
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= ne * L.n) return;
    const int64_t e = w / L.n, r = w % L.n;
    const int64_t rt = r / TILE_ROWS, rr = r % TILE_ROWS;
    const int64_t gguf_row = e * (L.n * L.row_bytes) + r * L.row_bytes;
    const int64_t ebase = (e0 + e) * L.expert_bytes;
    for (int kp = 0; kp < L.n_kp; ++kp) {
        const int64_t prb = piece_row_bytes(L, kp);
        for (int64_t i = lane; i < prb; i += 32) {
            const int64_t goff = gguf_row + (int64_t)kp * L.kp_row_bytes + i;
            const int64_t toff = ebase + tiled_offset(L, rt, rr, kp, i);
            if (to_tiled) dst[toff] = src[goff];
            else dst[goff] = src[toff];
        }
    }
}

// f32 rows of one expert: one thread per (row, 16 columns).
__global__ void k_dequant(const uint8_t* __restrict__ bank, Layout L, int64_t e, float* __restrict__ out) {
    extern __shared__ __align__(16) uint8_t tsm[];
    load_htables(reinterpret_cast<uint4*>(tsm), reinterpret_cast<uint2*>(tsm + 16384),
                 reinterpret_cast<uint4*>(tsm + 20480));
    __syncthreads();
    const HTables t{reinterpret_cast<const uint4*>(tsm), reinterpret_cast<const uint2*>(tsm + 16384),
                    reinterpret_cast<const uint4*>(tsm + 20480)};
    const int64_t units_per_row = L.k / 16;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= L.n * units_per_row) return;
    const int64_t r = i / units_per_row, uk = i % units_per_row;
    const int kp = (int)(uk / 16), kofs = (int)(uk % 16) * 16;
    const int64_t rt = r / TILE_ROWS, rr = r % TILE_ROWS;
    const uint8_t* piece = bank + e * L.expert_bytes + piece_offset(L, rt, kp);
    float w[16];
    dec16_exact<true>(L.fmt, piece, (int)rr, piece_row_bytes(L, kp), kofs, w, t);
    float* o = out + r * L.k + uk * 16;
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j] = w[j];
}

// ---------------------------------------------------------------- device quantisers
__device__ inline int nearest_int(float v) { return (int)roundf(v); }

__device__ void q8_0_from_float_d(const float* x, uint8_t* y) {
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    float d = amax / 127.f;
    float id = d != 0.f ? 1.f / d : 0.f;
    uint16_t dh = cwx_f32_to_f16_bits(d);
    y[0] = (uint8_t)dh;
    y[1] = (uint8_t)(dh >> 8);
    for (int i = 0; i < 32; ++i) {
        float v = roundf(x[i] * id);
        v = v < -128.f ? -128.f : (v > 127.f ? 127.f : v);
        y[2 + i] = (uint8_t)(int8_t)v;
    }
}

__device__ void mxfp4_from_float_d(const float* x, uint8_t* y) {
    const int8_t kv[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    uint8_t e = 0;
    if (amax > 0.f) {
        // floor of the correctly rounded f32 log2 (what log2f returns on the host)
        float l = (float)log2((double)amax);
        float v = floorf(l) - 2.0f + 127.0f;
        e = v <= 0.f ? 0 : (v >= 255.f ? 255 : (uint8_t)v);
    }
    y[0] = e;
    float d = e8m0_to_f32_half(e);
    for (int j = 0; j < 16; ++j) {
        uint8_t b[2];
        for (int h = 0; h < 2; ++h) {
            float xv = x[j + 16 * h];
            uint8_t best = 0;
            float best_err = fabsf((float)kv[0] * d - xv);
            for (int i = 1; i < 16; ++i) {
                float err = fabsf((float)kv[i] * d - xv);
                if (err < best_err) {
                    best = (uint8_t)i;
                    best_err = err;
                }
            }
            b[h] = best;
        }
        y[1 + j] = (uint8_t)(b[0] | (b[1] << 4));
    }
}

__device__ void make_qkx1_quants_d(int nmax, int ntry, const float* x, float* scale_out, float* min_out) {
    const int n = 32;
    uint8_t L[32];
    for (int i = 0; i < n; ++i) L[i] = 0;
    float mn = x[0], mx = x[0];
    for (int i = 1; i < n; ++i) {
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

__device__ void q4k_from_float_d(const float* x, uint8_t* b) {
    float mins[8], scales[8];
    for (int j = 0; j < 8; ++j) make_qkx1_quants_d(15, 5, x + 32 * j, &scales[j], &mins[j]);
    float max_scale = 0.f, max_min = 0.f;
    for (int j = 0; j < 8; ++j) {
        max_scale = fmaxf(scales[j], max_scale);
        max_min = fmaxf(mins[j], max_min);
    }
    float inv_scale = max_scale > 0.f ? 63.f / max_scale : 0.f;
    float inv_min = max_min > 0.f ? 63.f / max_min : 0.f;
    uint8_t* sc = b + 4;
    for (int j = 0; j < 12; ++j) sc[j] = 0;
    for (int j = 0; j < 8; ++j) {
        int lsi = nearest_int(inv_scale * scales[j]);
        int lmi = nearest_int(inv_min * mins[j]);
        uint8_t ls = (uint8_t)(lsi < 63 ? lsi : 63);
        uint8_t lm = (uint8_t)(lmi < 63 ? lmi : 63);
        if (j < 4) {
            sc[j] = ls;
            sc[j + 4] = lm;
        } else {
            sc[j + 4] = (uint8_t)((ls & 0xF) | ((lm & 0xF) << 4));
            sc[j - 4] |= (uint8_t)((ls >> 4) << 6);
            sc[j] |= (uint8_t)((lm >> 4) << 6);
        }
    }
    uint16_t dh = cwx_f32_to_f16_bits(max_scale / 63.f), mh = cwx_f32_to_f16_bits(max_min / 63.f);
    b[0] = (uint8_t)dh;
    b[1] = (uint8_t)(dh >> 8);
    b[2] = (uint8_t)mh;
    b[3] = (uint8_t)(mh >> 8);
    float df = cwx_f16_bits_to_f32(dh), mf = cwx_f16_bits_to_f32(mh);
    uint8_t* qs = b + 16;
    for (int j = 0; j < 128; ++j) qs[j] = 0;
    for (int j = 0; j < 8; ++j) {
        int s, m;
        get_scale_min_k4(j, sc, &s, &m);
        float d = df * (float)s;
        for (int ii = 0; ii < 32; ++ii) {
            uint8_t l = 0;
            if (d != 0.f) {
                float dm = mf * (float)m;
                int li = nearest_int((x[32 * j + ii] + dm) / d);
                l = (uint8_t)(li < 0 ? 0 : (li > 15 ? 15 : li));
            }
            // byte (j/2)*32 + ii holds element 64*(j/2) + ii (low) and + 32 (high)
            qs[(j / 2) * 32 + ii] |= (uint8_t)(l << (4 * (j & 1)));
        }
    }
}

__device__ float make_qx_quants_d(int n, int nmax, const float* x, int8_t* ls) {
    // rmse_type 1 (weights x*x), the only form Q6_K uses
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
    float sumlx = 0.f, suml2 = 0.f;
    for (int i = 0; i < n; ++i) {
        int l = nearest_int(iscale * x[i]);
        l = l < -nmax ? -nmax : (l > nmax - 1 ? nmax - 1 : l);
        ls[i] = (int8_t)(l + nmax);
        float w = x[i] * x[i];
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
            float w = x[i] * x[i];
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
            float w = x[i] * x[i];
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
    return scale;
}

__device__ void q6k_from_float_d(const float* x, uint8_t* y) {
    int8_t L[256];
    float scales[16];
    float max_scale = 0.f, max_abs_scale = 0.f;
    for (int ib = 0; ib < 16; ++ib) {
        float scale = make_qx_quants_d(16, 32, x + 16 * ib, L + 16 * ib);
        scales[ib] = scale;
        float as = fabsf(scale);
        if (as > max_abs_scale) {
            max_abs_scale = as;
            max_scale = scale;
        }
    }
    float iscale = -128.f / max_scale;
    uint16_t dh = cwx_f32_to_f16_bits(1.0f / iscale);
    int8_t* ysc = (int8_t*)(y + 192);
    for (int ib = 0; ib < 16; ++ib) {
        int v = nearest_int(iscale * scales[ib]);
        ysc[ib] = (int8_t)(v < 127 ? v : 127);
    }
    float df = cwx_f16_bits_to_f32(dh);
    for (int j = 0; j < 16; ++j) {
        float d = df * (float)ysc[j];
        if (d == 0.f) continue;
        for (int ii = 0; ii < 16; ++ii) {
            int ll = nearest_int(x[16 * j + ii] / d);
            ll = ll < -32 ? -32 : (ll > 31 ? 31 : ll);
            L[16 * j + ii] = (int8_t)(ll + 32);
        }
    }
    uint8_t* ql = y;
    uint8_t* qh = y + 128;
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
    y[208] = (uint8_t)dh;
    y[209] = (uint8_t)(dh >> 8);
}

// One thread per (expert, row, K-piece): draw the piece's values and quantise them in place.
// Experts e0 .. e0+ne-1 of the bank; `first` is the bank's first expert in the synthetic tensor
// (the values follow the global expert index, so a slice equals those experts of the whole).
struct SynthMaps {
    const uint16_t *iq3s, *iq2s, *iq3xxs, *iq2xxs;
};

__global__ void k_synth(uint8_t* __restrict__ bank, Layout L, int64_t e0, int64_t ne, int64_t first, uint64_t key,
                        float std_, SynthMaps maps) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t total = ne * L.n * L.n_kp;
    if (i >= total) return;
    int kp = (int)(i % L.n_kp);
    int64_t er = i / L.n_kp;
    int64_t e = er / L.n + e0, r = er % L.n;
    int64_t rt = r / TILE_ROWS, rr = r % TILE_ROWS;
    int64_t prb = piece_row_bytes(L, kp);
    uint8_t blk[272];  // the row's bytes of this piece, written to the tiled layout below
    uint8_t* dst = blk;
    int64_t c0 = (int64_t)kp * PIECE_K;
    int64_t klen = L.k - c0 < PIECE_K ? L.k - c0 : PIECE_K;
    float x[256];
    uint64_t base = (uint64_t)((e + first) * L.n + r) * (uint64_t)L.k + (uint64_t)c0;
    for (int c = 0; c < klen; ++c) x[c] = cwx_normal_std(key, base + c, std_);
    switch (L.fmt) {
        case F_Q4_K: q4k_from_float_d(x, dst); break;
        case F_Q6_K: q6k_from_float_d(x, dst); break;
        case F_IQ3_S: cwx_encode_iq3s(x, dst, maps.iq3s); break;
        case F_IQ2_S: cwx_encode_iq2s(x, dst, maps.iq2s); break;
        case F_IQ3_XXS: cwx_encode_iq3xxs(x, dst, maps.iq3xxs); break;
        case F_IQ2_XXS: cwx_encode_iq2xxs(x, dst, maps.iq2xxs); break;
        case F_IQ4_XS: cwx_encode_iq4xs(x, dst); break;
        case F_Q8_0:
            for (int b = 0; b < klen / 32; ++b) q8_0_from_float_d(x + 32 * b, dst + 34 * b);
            break;
        case F_MXFP4:
            for (int b = 0; b < klen / 32; ++b) mxfp4_from_float_d(x + 32 * b, dst + 17 * b);
            break;
    }
    uint8_t* ebank = bank + (e - e0) * L.expert_bytes;
    for (int64_t b = 0; b < prb; ++b) ebank[tiled_offset(L, rt, rr, kp, b)] = blk[b];
}

__global__ void k_normal(float* __restrict__ out, int64_t n, uint64_t key, uint64_t offset, float std_) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = cwx_normal_std(key, offset + (uint64_t)i, std_);
}

static int upload_map(uint16_t** dst, void (*build)(uint16_t*), int size) {
    std::vector<uint16_t> m(size);
    build(m.data());
    CWX_CUDA(cudaMalloc(dst, m.size() * 2));
    CWX_CUDA(cudaMemcpy(*dst, m.data(), m.size() * 2, cudaMemcpyHostToDevice));
    return CWX_OK;
}

// The encoder maps of the IQ codebook formats, on the context's device (built on first use).
static int ensure_maps(cwx_ctx* ctx) {
    int rc;
    if (!ctx->d_iq3s_map && (rc = upload_map(&ctx->d_iq3s_map, cwx_build_iq3s_map, CWX_IQ3S_MAP_SIZE))) return rc;
    if (!ctx->d_iq2s_map && (rc = upload_map(&ctx->d_iq2s_map, cwx_build_iq2s_map, CWX_IQ2S_MAP_SIZE))) return rc;
    if (!ctx->d_iq3xxs_map && (rc = upload_map(&ctx->d_iq3xxs_map, cwx_build_iq3xxs_map, CWX_IQ3XXS_MAP_SIZE)))
        return rc;
    if (!ctx->d_iq2xxs_map && (rc = upload_map(&ctx->d_iq2xxs_map, cwx_build_iq2xxs_map, CWX_IQ2XXS_MAP_SIZE)))
        return rc;
    return CWX_OK;
}

}  // namespace cwx

using namespace cwx;

static int supported_type(int t) {
    return t == F_Q8_0 || t == F_Q4_K || t == F_Q6_K || t == F_IQ3_S || t == F_IQ2_S || t == F_MXFP4 ||
           t == F_IQ2_XXS || t == F_IQ3_XXS || t == F_IQ4_XS;
}

// MXFP4 banks, one thread per (expert, row, piece): bit 0 of flag when a whole 256-column piece
// or a 2-block tail piece has block scales e more than 24 apart (the grouped products' f16 fast
// paths), bit 1 when any
// block scale lies outside [104, 140] (the tensor-core products need every weight exact in f16).
constexpr int MX_F16_MIN = 104, MX_F16_MAX = 140;
__global__ void k_mx_spread(const uint8_t* __restrict__ d, Layout L, int64_t ne, int* flag) {
    const int64_t per_e = L.n * L.n_kp;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= ne * per_e) return;
    const int64_t e = i / per_e, rem = i % per_e, r = rem / L.n_kp;
    const int kp = (int)(rem % L.n_kp);
    const int nb = (int)(piece_row_bytes(L, kp) / 17);
    const uint8_t* x = d + e * L.expert_bytes;
    int mx = 0, mn = 255;
    for (int b = 0; b < nb; ++b) {
        const int v = x[tiled_offset(L, r / TILE_ROWS, r % TILE_ROWS, kp, 17 * b)];
        mx = max(mx, v);
        mn = min(mn, v);
    }
    int f = 0;
    if ((nb == 8 || nb == 2) && mx - mn > 24) f |= 1;  // (whole pieces and the 2-block tail: fast paths)
    if (mn < MX_F16_MIN || mx > MX_F16_MAX) f |= 2;
    if (f) atomicOr(flag, f);
}

// Sets b->mx_wide and b->mx_f16 for an MXFP4 bank whose tiled bytes are on the device.
static int mx_check(cwx_bank* b, int64_t ne) {
    b->mx_wide = 0;
    b->mx_f16 = 0;
    if (b->L.fmt != F_MXFP4 || ne <= 0) return CWX_OK;
    int* flag = nullptr;
    CWX_CUDA(cudaMalloc(&flag, sizeof(int)));
    cudaError_t e = cudaMemset(flag, 0, sizeof(int));
    const int64_t items = ne * b->L.n * b->L.n_kp;
    if (e == cudaSuccess) {
        k_mx_spread<<<(unsigned)((items + 255) / 256), 256>>>(b->d, b->L, ne, flag);
        e = cudaGetLastError();
    }
    int h = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&h, flag, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(flag);
    if (e != cudaSuccess) return cuda_fail(e, "MXFP4 scale check");
    b->mx_wide = h & 1;
    b->mx_f16 = (h & 2) ? 0 : 1;
    return CWX_OK;
}

static int alloc_bank(int device, int type, int64_t n, int64_t k, int64_t ne, cwx_bank** out) {
    if (!out) return fail(CWX_EINVAL, "cwx_bank: null output pointer");
    *out = nullptr;
    if (!supported_type(type)) return fail(CWX_EUNSUPPORTED, "cwx_bank: unsupported ggml type %d", type);
    Layout L;
    if (!make_layout(type, n, k, ne, &L)) return fail(CWX_EINVAL, "cwx_bank: bad shape n=%lld k=%lld experts=%lld for type %d",
                                                      (long long)n, (long long)k, (long long)ne, type);
    // the IQ formats are stored in groups of 16 rows (a partial group would not fit its piece)
    if (fmt_soa(type) && n % 16)
        return fail(CWX_EUNSUPPORTED, "cwx_bank: type %d needs a multiple of 16 rows, got n=%lld", type, (long long)n);
    CWX_CUDA(cudaSetDevice(device));
    cwx_bank* b = new cwx_bank();
    b->device = device;
    b->L = L;
    b->bytes_per_expert_gguf = n * L.row_bytes;
    cudaError_t e = cudaMalloc(&b->d, (size_t)(L.expert_bytes * ne));
    if (e != cudaSuccess) {
        delete b;
        cudaGetLastError();
        return fail(CWX_ENOMEM, "cwx_bank: cannot allocate %lld bytes on device %d", (long long)(L.expert_bytes * ne), device);
    }
    *out = b;
    return CWX_OK;
}

extern "C" int cwx_bank_create(int device, const cwx_matrix_desc* desc, cwx_bank** out) {
    if (!desc || !desc->host_ptr) return fail(CWX_EINVAL, "cwx_bank_create: null descriptor or data");
    int rc = alloc_bank(device, desc->ggml_type, desc->n, desc->k, desc->n_experts, out);
    if (rc) return rc;
    cwx_bank* b = *out;
    if (desc->bytes_per_expert != b->bytes_per_expert_gguf) {
        cwx_bank_destroy(b);
        *out = nullptr;
        return fail(CWX_EINVAL, "cwx_bank_create: bytes_per_expert %lld, expected %lld for this shape",
                    (long long)desc->bytes_per_expert, (long long)(desc->n * b->L.row_bytes));
    }
    // upload in chunks of experts through one staging buffer, repacking on the device
    int64_t bpe = b->bytes_per_expert_gguf;
    int64_t chunk = bpe >= (256ll << 20) ? 1 : (256ll << 20) / bpe;
    if (chunk > desc->n_experts) chunk = desc->n_experts;
    uint8_t* stage = nullptr;
    cudaError_t e = cudaMalloc(&stage, (size_t)(chunk * bpe));
    if (e != cudaSuccess) {
        cwx_bank_destroy(b);
        *out = nullptr;
        return cuda_fail(e, "cudaMalloc(upload stage)");
    }
    for (int64_t e0 = 0; e0 < desc->n_experts; e0 += chunk) {
        int64_t ne = desc->n_experts - e0 < chunk ? desc->n_experts - e0 : chunk;
        e = cudaMemcpy(stage, (const uint8_t*)desc->host_ptr + e0 * bpe, (size_t)(ne * bpe), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) break;
        int64_t warps = ne * b->L.n;
        k_repack<<<(unsigned)((warps * 32 + 255) / 256), 256>>>(stage, b->d, b->L, e0, ne, 1);
        e = cudaGetLastError();
        if (e != cudaSuccess) break;
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaFree(stage);
    if (e != cudaSuccess) {
        cwx_bank_destroy(b);
        *out = nullptr;
        return cuda_fail(e, "cwx_bank_create upload");
    }
    if ((rc = mx_check(b, desc->n_experts))) {
        cwx_bank_destroy(b);
        *out = nullptr;
        return rc;
    }
    return CWX_OK;
}

extern "C" int cwx_bank_synth(cwx_ctx* ctx, int32_t type, int64_t n, int64_t k, int64_t ne, uint64_t key, float std_,
                              cwx_bank** out) {
    return cwx_bank_synth_experts(ctx, type, n, k, 0, ne, key, std_, out);
}

extern "C" int cwx_bank_synth_experts(cwx_ctx* ctx, int32_t type, int64_t n, int64_t k, int64_t first, int64_t ne,
                                      uint64_t key, float std_, cwx_bank** out) {
    if (!ctx) return fail(CWX_EINVAL, "cwx_bank_synth: null context");
    if (first < 0) return fail(CWX_EINVAL, "cwx_bank_synth_experts: first expert %lld", (long long)first);
    int rc = alloc_bank(ctx->device, type, n, k, ne, out);
    if (rc) return rc;
    cwx_bank* b = *out;
    if ((rc = ensure_maps(ctx))) {
        cwx_bank_destroy(b);
        *out = nullptr;
        return rc;
    }
    cudaError_t e = cudaSuccess;
    {
        int threads = 128;
        // launches of at most ~4M (row, piece) items keep each launch short on very large banks
        int64_t rows_per_launch = (1 << 22) / b->L.n_kp;
        int64_t experts_per_launch = rows_per_launch / n > 0 ? rows_per_launch / n : 1;
        for (int64_t e0 = 0; e0 < ne && e == cudaSuccess; e0 += experts_per_launch) {
            int64_t cnt = ne - e0 < experts_per_launch ? ne - e0 : experts_per_launch;
            int64_t items = cnt * n * b->L.n_kp;
            k_synth<<<(unsigned)((items + threads - 1) / threads), threads>>>(
                b->d + e0 * b->L.expert_bytes, b->L, e0, cnt, first, key, std_,
                SynthMaps{ctx->d_iq3s_map, ctx->d_iq2s_map, ctx->d_iq3xxs_map, ctx->d_iq2xxs_map});
            e = cudaGetLastError();
        }
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cwx_bank_destroy(b);
        *out = nullptr;
        return cuda_fail(e, "cwx_bank_synth");
    }
    if ((rc = mx_check(b, ne))) {
        cwx_bank_destroy(b);
        *out = nullptr;
        return rc;
    }
    return CWX_OK;
}

extern "C" int cwx_bank_synth_list(cwx_ctx* ctx, int32_t type, int64_t n, int64_t k, const int64_t* experts,
                                   int64_t count, uint64_t key, float std_, cwx_bank** out) {
    if (!ctx || !experts || !out) return fail(CWX_EINVAL, "cwx_bank_synth_list: null argument");
    for (int64_t i = 0; i < count; ++i)
        if (experts[i] < 0) return fail(CWX_EINVAL, "cwx_bank_synth_list: expert %lld", (long long)experts[i]);
    int rc = alloc_bank(ctx->device, type, n, k, count, out);
    if (rc) return rc;
    cwx_bank* b = *out;
    if ((rc = ensure_maps(ctx))) {
        cwx_bank_destroy(b);
        *out = nullptr;
        return rc;
    }
    // slot i holds global expert experts[i]: one launch per expert (k_synth's values follow the
    // global index e0 + first, so slot i is its own one-expert bank with first = experts[i])
    cudaError_t e = cudaSuccess;
    const int threads = 128;
    const int64_t items = n * b->L.n_kp;
    for (int64_t i = 0; i < count && e == cudaSuccess; ++i) {
        k_synth<<<(unsigned)((items + threads - 1) / threads), threads>>>(
            b->d + i * b->L.expert_bytes, b->L, 0, 1, experts[i], key, std_,
            SynthMaps{ctx->d_iq3s_map, ctx->d_iq2s_map, ctx->d_iq3xxs_map, ctx->d_iq2xxs_map});
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cwx_bank_destroy(b);
        *out = nullptr;
        return cuda_fail(e, "cwx_bank_synth_list");
    }
    if ((rc = mx_check(b, count))) {
        cwx_bank_destroy(b);
        *out = nullptr;
        return rc;
    }
    return CWX_OK;
}

extern "C" int cwx_bank_destroy(cwx_bank* b) {
    if (!b) return CWX_OK;
    cudaSetDevice(b->device);
    if (b->d) cudaFree(b->d);
    delete b;
    return CWX_OK;
}

extern "C" int cwx_bank_desc(const cwx_bank* b, cwx_matrix_desc* out) {
    if (!b || !out) return fail(CWX_EINVAL, "cwx_bank_desc: null argument");
    out->ggml_type = b->L.fmt;
    out->n = b->L.n;
    out->k = b->L.k;
    out->n_experts = b->L.n_experts;
    out->bytes_per_expert = b->bytes_per_expert_gguf;
    out->host_ptr = nullptr;
    return CWX_OK;
}

extern "C" int cwx_bank_download(const cwx_bank* b, int64_t e0, int64_t ne, void* host_dst) {
    if (!b || !host_dst) return fail(CWX_EINVAL, "cwx_bank_download: null argument");
    if (e0 < 0 || ne < 0 || e0 + ne > b->L.n_experts) return fail(CWX_EINVAL, "cwx_bank_download: experts out of range");
    if (ne == 0) return CWX_OK;
    CWX_CUDA(cudaSetDevice(b->device));
    int64_t bpe = b->bytes_per_expert_gguf;
    uint8_t* stage = nullptr;
    CWX_CUDA(cudaMalloc(&stage, (size_t)(ne * bpe)));
    int64_t warps = ne * b->L.n;
    k_repack<<<(unsigned)((warps * 32 + 255) / 256), 256>>>(b->d, stage, b->L, e0, ne, 0);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpy(host_dst, stage, (size_t)(ne * bpe), cudaMemcpyDeviceToHost);
    cudaFree(stage);
    if (e != cudaSuccess) return cuda_fail(e, "cwx_bank_download");
    return CWX_OK;
}

extern "C" int cwx_bank_dequantize(const cwx_bank* b, int64_t expert, float* out, void* stream) {
    if (!b || !out) return fail(CWX_EINVAL, "cwx_bank_dequantize: null argument");
    if (expert < 0 || expert >= b->L.n_experts) return fail(CWX_EINVAL, "cwx_bank_dequantize: expert out of range");
    if (b->L.k % 16) return fail(CWX_EUNSUPPORTED, "cwx_bank_dequantize: k must be a multiple of 16");
    CWX_CUDA(cudaSetDevice(b->device));
    int64_t units = b->L.n * (b->L.k / 16);
    k_dequant<<<(unsigned)((units + 127) / 128), 128, HTABLES_BYTES, (cudaStream_t)stream>>>(b->d, b->L, expert,
                                                                                              out);
    CWX_CUDA(cudaGetLastError());
    return CWX_OK;
}

extern "C" int cwx_synth_normal(cwx_ctx* ctx, uint64_t key, uint64_t offset, int64_t n, float std_, float* out,
                                void* stream) {
    if (!ctx || (n > 0 && !out) || n < 0) return fail(CWX_EINVAL, "cwx_synth_normal: bad argument");
    if (n == 0) return CWX_OK;
    CWX_CUDA(cudaSetDevice(ctx->device));
    k_normal<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(out, n, key, offset, std_);
    CWX_CUDA(cudaGetLastError());
    return CWX_OK;
}
