// Grouped expert products for decode-sized piles, activation preparation, and the combine.
//
//   expert products  MoeMatvec -> kernel_mul_mv_id_* / kernel_mul_mm_idg_*
//                    (crates/engine/src/experts.rs:2183-2309, crates/engine/src/mv_id.rs:17-384,
//                    vendor/candle-metal-kernels/src/metal_src/quantized.metal:7668-7766)
//   activation       ExpertAct::hidden / finish experts.rs:2389-2422, cw_silu_mul
//                    fuse_kernel.rs:77-96 (fused into the gate/up epilogue here)
//   combine          cw_weighted_sum fuse_kernel.rs:277-291 (pick order) + shared expert
//                    model_next.rs:731-741 + residual model_next.rs:1437
//   Q8 activations   BlockQ8K::from_float k_quants.rs:2495-2534, BlockQ8_0::from_float 784-820
//
// Work items are (expert, 64-row tile) over the experts that have picks (the used list built by
// the pile kernels), plus the shared expert's tiles. A CTA of 4 warps streams each item's
// quantised weight pieces (64 rows x 256 columns, one cp.async.bulk each, several in flight in an
// mbarrier ring) from HBM, each warp dequantises 16 rows x 64 columns at a time into f16 in shared
// memory (exact f32 dequant, one rounding), and the tensor pipe multiplies them with the pile's
// activations: mma.sync m16n8k16, activations as an f16 hi + lo pair so the product carries ~22
// bits of the f32 input, f32 accumulation. Up to 64 picks of one expert share each dequantised
// tile; larger piles take several passes.
#include "cwx_common.cuh"
#include "decode.cuh"
#include "kernels.cuh"

namespace cwx {

constexpr int GEMV_WARPS = 4;
constexpr int GEMV_THREADS = GEMV_WARPS * 32;
constexpr int MAX_PASS_TOK = 64;  // picks per pass (8 n-tiles of 8)
constexpr int NT = MAX_PASS_TOK / 8;

struct Item {
    int shared;
    uint32_t e, first, count;
    int64_t rt;
    int n_kp;
    int passes;
};

__device__ __forceinline__ int tiles_of(const Layout& L) { return (int)((L.n + TILE_ROWS - 1) / TILE_ROWS); }

__device__ __forceinline__ bool get_item(const GemvArgs& a, int64_t it, uint32_t n_used, Item* o) {
    int sh_tiles = a.has_shared ? tiles_of(a.sa.L) : 0;
    if (it < sh_tiles) {
        o->shared = 1;
        o->e = 0;
        o->first = 0;
        o->count = (uint32_t)a.s_count;
        o->rt = it;
        o->n_kp = a.sa.L.n_kp;
    } else {
        int64_t r = it - sh_tiles;
        int tr = tiles_of(a.ra.L);
        int64_t u = r / tr;
        if (u >= n_used) return false;
        o->shared = 0;
        o->e = a.used3[3 * u];
        o->first = a.used3[3 * u + 1];
        o->count = a.used3[3 * u + 2];
        o->rt = r % tr;
        o->n_kp = a.ra.L.n_kp;
    }
    o->passes = (int)((o->count + MAX_PASS_TOK - 1) / MAX_PASS_TOK);
    if (o->passes < 1) o->passes = 1;
    return true;
}

// Cursor over this CTA's (item, pass, piece) steps.
struct Cursor {
    int64_t j;  // local item number
    int pass, kp;
    Item item;
    bool valid;
};

__device__ __forceinline__ void cursor_init(const GemvArgs& a, uint32_t n_used, Cursor* c) {
    c->j = 0;
    c->pass = 0;
    c->kp = 0;
    c->valid = get_item(a, blockIdx.x, n_used, &c->item);
}
__device__ __forceinline__ void cursor_next(const GemvArgs& a, uint32_t n_used, Cursor* c) {
    if (!c->valid) return;
    if (++c->kp < c->item.n_kp) return;
    c->kp = 0;
    if (++c->pass < c->item.passes) return;
    c->pass = 0;
    c->j++;
    c->valid = get_item(a, (int64_t)blockIdx.x + c->j * gridDim.x, n_used, &c->item);
}

__device__ __forceinline__ void issue_step(const GemvArgs& a, const Cursor& c, uint8_t* stage, uint64_t* bar) {
    const MatRef& m0 = c.item.shared ? a.sa : a.ra;
    const MatRef& m1 = c.item.shared ? a.sb : a.rb;
    uint32_t b0 = (uint32_t)piece_bytes(m0.L, c.item.rt, c.kp);
    uint32_t b1 = a.two ? (uint32_t)piece_bytes(m1.L, c.item.rt, c.kp) : 0u;
    mbar_expect_tx(bar, b0 + b1);
    const uint8_t* s0 = m0.base + (int64_t)c.item.e * m0.L.expert_bytes + piece_offset(m0.L, c.item.rt, c.kp);
    bulk_g2s(stage, s0, b0, bar);
    if (a.two) {
        const uint8_t* s1 = m1.base + (int64_t)c.item.e * m1.L.expert_bytes + piece_offset(m1.L, c.item.rt, c.kp);
        bulk_g2s(stage + a.stage_b_off, s1, b1, bar);
    }
}

// Dequantise unit (row = lane % 16, 32-column unit (2*ss + lane/16)) of the warp's 16 rows and
// store it as f16 into the warp's 16 x 64 tile (16-byte chunks XOR-swizzled by row). With a `lo`
// tile, the weights are stored as an f16 pair hi + lo carrying ~22 bits of the exact f32 value.
__device__ __forceinline__ void stage_a(int fmt, const uint8_t* piece, int64_t prb, int row0, int ss, int lane,
                                        __half* abuf, __half* abuf_lo, const Tables& t) {
    int r = lane & 15, uh = lane >> 4;
    float w[32];
    decode_unit(fmt, piece + (int64_t)(row0 + r) * prb, 2 * ss + uh, w, t);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint4 v, vl;
        uint32_t* pv = reinterpret_cast<uint32_t*>(&v);
        uint32_t* pl = reinterpret_cast<uint32_t*>(&vl);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float a = w[8 * q + 2 * i], b = w[8 * q + 2 * i + 1];
            __half2 h = __floats2half2_rn(a, b);
            pv[i] = *reinterpret_cast<uint32_t*>(&h);
            if (abuf_lo) {
                float2 hf = __half22float2(h);
                __half2 l = __floats2half2_rn(__fsub_rn(a, hf.x), __fsub_rn(b, hf.y));
                pl[i] = *reinterpret_cast<uint32_t*>(&l);
            }
        }
        int chunk = 4 * uh + q;
        int off = r * 64 + ((chunk ^ (r & 7)) * 8);
        *reinterpret_cast<uint4*>(abuf + off) = v;
        if (abuf_lo) *reinterpret_cast<uint4*>(abuf_lo + off) = vl;
    }
}

__device__ __forceinline__ void load_a_frag(const __half* abuf, int kk, int lane, uint32_t* a) {
    int m = lane >> 3, rr = lane & 7;
    int row = (m & 1) * 8 + rr;
    int chunk = 2 * kk + (m >> 1);
    ldmatrix_x4(a, abuf + row * 64 + ((chunk ^ (row & 7)) * 8));
}

__device__ __forceinline__ float silu_f(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

__global__ void __launch_bounds__(GEMV_THREADS) k_gemv(GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);  // nst mbarriers
    uint64_t* s_iq2s = reinterpret_cast<uint64_t*>(smem + 128);
    uint32_t* s_iq3s = reinterpret_cast<uint32_t*>(smem + 128 + 8192);
    __half* abufs = reinterpret_cast<__half*>(smem + 128 + 8192 + 2048);  // 4 warps x 4 x 16 x 64
    uint8_t* stages = smem + 128 + 8192 + 2048 + GEMV_WARPS * 4 * 16 * 64 * 2;
    __shared__ int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t n_used = *a.n_used;
    if (tid == 0) {
        for (int s = 0; s < a.nst; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        s_abort = 0;
    }
    load_tables(s_iq2s, s_iq3s);
    __syncthreads();
    Tables tb{s_iq2s, s_iq3s};

    Cursor cc, pc;
    cursor_init(a, n_used, &cc);
    if (!cc.valid) return;
    pc = cc;
    if (tid == 0) {
        for (int s = 0; s < a.nst && pc.valid; ++s) {
            issue_step(a, pc, stages + (int64_t)s * a.stage_bytes, &bars[s]);
            cursor_next(a, n_used, &pc);
        }
    }

    __half* abuf0 = abufs + (warp * 4 + 0) * 16 * 64;
    __half* abuf1 = abufs + (warp * 4 + 1) * 16 * 64;
    __half* abuf0l = abufs + (warp * 4 + 2) * 16 * 64;
    __half* abuf1l = abufs + (warp * 4 + 3) * 16 * 64;
    float acc0[NT][4], acc1[NT][4];
    int64_t boff[NT];
    int ntok = 0;
    const int g = lane >> 2, c4 = lane & 3;

    for (int64_t q = 0; cc.valid; ++q) {
        const int s = (int)(q % a.nst);
        const Item& it = cc.item;
        const MatRef& m0 = it.shared ? a.sa : a.ra;
        const MatRef& m1 = it.shared ? a.sb : a.rb;
        const __half* bh = it.shared ? a.sbh : a.rbh;
        const __half* bl = it.shared ? a.sbl : a.rbl;
        if (cc.kp == 0) {  // new pass: its picks, zeroed accumulators
            {
                uint32_t rem = it.count - (uint32_t)cc.pass * MAX_PASS_TOK;
                ntok = rem < (uint32_t)MAX_PASS_TOK ? (int)rem : MAX_PASS_TOK;
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                int slot = 8 * nt + g;
                boff[nt] = -1;
                if (slot < ntok) {
                    uint32_t idx = (uint32_t)cc.pass * MAX_PASS_TOK + slot;
                    int64_t row = it.shared ? (int64_t)idx : (int64_t)(a.pairs[it.first + idx] / (uint32_t)a.r_bdiv);
                    boff[nt] = row * (it.shared ? a.s_bstride : a.r_bstride);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) acc0[nt][i] = acc1[nt][i] = 0.f;
            }
        }
        bool ok = mbar_wait(&bars[s], (uint32_t)((q / a.nst) & 1), a.err);
        if (!ok) s_abort = 1;
        __syncthreads();
        if (s_abort) return;

        const uint8_t* st = stages + (int64_t)s * a.stage_bytes;
        const int rows = tile_rows(m0.L, it.rt);
        const int row0 = warp * 16;
        const int64_t prb0 = piece_row_bytes(m0.L, cc.kp);
        const int64_t prb1 = a.two ? piece_row_bytes(m1.L, cc.kp) : 0;
        const int64_t kbase = (int64_t)cc.kp * PIECE_K;
        const int klen = (int)(m0.L.k - kbase < PIECE_K ? m0.L.k - kbase : PIECE_K);
        const int n_nt = (ntok + 7) >> 3;
        const bool split = it.shared ? a.split_s : a.split_r;
        if (row0 < rows) {
            for (int ss = 0; ss < klen / 64; ++ss) {
                stage_a(m0.L.fmt, st, prb0, row0, ss, lane, abuf0, split ? abuf0l : nullptr, tb);
                if (a.two) stage_a(m1.L.fmt, st + a.stage_b_off, prb1, row0, ss, lane, abuf1, split ? abuf1l : nullptr, tb);
                __syncwarp();
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    uint32_t af0[4], af1[4], al0[4], al1[4];
                    load_a_frag(abuf0, kk, lane, af0);
                    if (a.two) load_a_frag(abuf1, kk, lane, af1);
                    if (split) {
                        load_a_frag(abuf0l, kk, lane, al0);
                        if (a.two) load_a_frag(abuf1l, kk, lane, al1);
                    }
                    int64_t kg = kbase + ss * 64 + kk * 16 + 2 * c4;
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        if (nt < n_nt) {
                            uint32_t h0 = 0, h1 = 0, l0 = 0, l1 = 0;
                            if (boff[nt] >= 0) {
                                const __half* ph = bh + boff[nt] + kg;
                                const __half* pl = bl + boff[nt] + kg;
                                h0 = *reinterpret_cast<const uint32_t*>(ph);
                                h1 = *reinterpret_cast<const uint32_t*>(ph + 8);
                                l0 = *reinterpret_cast<const uint32_t*>(pl);
                                l1 = *reinterpret_cast<const uint32_t*>(pl + 8);
                            }
                            mma_16816(acc0[nt], af0, h0, h1);
                            mma_16816(acc0[nt], af0, l0, l1);
                            if (split) mma_16816(acc0[nt], al0, h0, h1);
                            if (a.two) {
                                mma_16816(acc1[nt], af1, h0, h1);
                                mma_16816(acc1[nt], af1, l0, l1);
                                if (split) mma_16816(acc1[nt], al1, h0, h1);
                            }
                        }
                    }
                }
                __syncwarp();
            }
            if (cc.kp == it.n_kp - 1) {  // end of pass: epilogue
                float* out = it.shared ? a.sout : a.rout;
                int64_t ostride = it.shared ? a.s_ostride : a.r_ostride;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    if (nt < n_nt) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            int slot = 8 * nt + 2 * c4 + (i & 1);
                            int64_t feat = it.rt * TILE_ROWS + row0 + g + ((i >> 1) ? 8 : 0);
                            if (slot < ntok) {
                                uint32_t idx = (uint32_t)cc.pass * MAX_PASS_TOK + slot;
                                int64_t orow = it.shared ? (int64_t)idx : (int64_t)a.pairs[it.first + idx];
                                float v;
                                if (a.two) {
                                    float gv = acc0[nt][i], uv = acc1[nt][i];
                                    if (a.act == CWX_ACT_SILU || it.shared) {
                                        v = __fmul_rn(silu_f(gv), uv);
                                    } else {
                                        int64_t bo = (int64_t)it.e * m0.L.n + feat;
                                        if (a.gate_b) gv = __fadd_rn(gv, a.gate_b[bo]);
                                        gv = fminf(gv, a.limit);
                                        if (a.up_b) uv = __fadd_rn(uv, a.up_b[bo]);
                                        uv = fminf(fmaxf(uv, -a.limit), a.limit);
                                        float z = __fmul_rn(gv, a.alpha);
                                        float sg = __fdiv_rn(1.0f, __fadd_rn(expf(-z), 1.0f));
                                        v = __fmul_rn(__fadd_rn(uv, 1.0f), __fmul_rn(gv, sg));
                                    }
                                } else {
                                    v = acc0[nt][i];
                                    if (!it.shared && a.down_b) v = __fadd_rn(v, a.down_b[(int64_t)it.e * m0.L.n + feat]);
                                }
                                out[orow * ostride + feat] = v;
                            }
                        }
                    }
                }
            }
        }
        __syncthreads();  // stage s consumed by every warp
        if (tid == 0 && pc.valid) {
            issue_step(a, pc, stages + (int64_t)s * a.stage_bytes, &bars[s]);
            cursor_next(a, n_used, &pc);
        }
        cursor_next(a, n_used, &cc);
    }
}

// ---------------------------------------------------------------- activation preparation
// rows (R, K) f32 -> hi, lo f16 of the activation the weights are multiplied with:
//   AM_F32   the value itself
//   AM_Q8_K  d*q of candle's Q8_K quantisation of each 256-block (max by |x|, first on ties;
//            iscale = -127/max; q = clamp(round(iscale*x)); d = 1/iscale)
//   AM_Q8_0  q * f16(d) of candle's Q8_0 quantisation of each 32-block (d = amax/127)
// One warp per (row, 256 columns).
__global__ void __launch_bounds__(256) k_prep(const float* __restrict__ src, int64_t R, int64_t K, int mode,
                                              __half* __restrict__ hi, __half* __restrict__ lo) {
    int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    int64_t nb = (K + 255) / 256;
    if (w >= R * nb) return;
    int64_t r = w / nb, b = w % nb;
    int64_t c0 = b * 256;
    int len = (int)(K - c0 < 256 ? K - c0 : 256);
    const float* x = src + r * K + c0;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (8 * lane + j < len) ? x[8 * lane + j] : 0.f;
    if (mode == AM_Q8_K) {
        // max |x| with the lowest index among equals, and the signed value there
        float am = -1.f;
        int ai = 1 << 30;
        float mv = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float f = fabsf(v[j]);
            if (f > am) {
                am = f;
                ai = 8 * lane + j;
                mv = v[j];
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            float oa = __shfl_xor_sync(0xffffffffu, am, o);
            int oi = __shfl_xor_sync(0xffffffffu, ai, o);
            float ov = __shfl_xor_sync(0xffffffffu, mv, o);
            if (oa > am || (oa == am && oi < ai)) {
                am = oa;
                ai = oi;
                mv = ov;
            }
        }
        if (am == 0.f) {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = 0.f;
        } else {
            float iscale = __fdiv_rn(-127.f, mv);
            float d = __fdiv_rn(1.0f, iscale);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float qv = roundf(__fmul_rn(iscale, v[j]));
                qv = fminf(fmaxf(qv, -128.f), 127.f);
                v[j] = __fmul_rn(d, qv);
            }
        }
    } else if (mode == AM_Q8_0) {
        // 32-blocks: lanes 4i..4i+3 hold block i
        float am = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) am = fmaxf(am, fabsf(v[j]));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
        float d = __fdiv_rn(am, 127.f);
        float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
        float dh = __half2float(__float2half_rn(d));
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float qv = roundf(__fmul_rn(v[j], id));
            qv = fminf(fmaxf(qv, -128.f), 127.f);
            v[j] = __fmul_rn(qv, dh);
        }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        if (8 * lane + j < len) {
            __half h, l;
            split_f16(v[j], &h, &l);
            hi[r * K + c0 + 8 * lane + j] = h;
            lo[r * K + c0 + 8 * lane + j] = l;
        }
    }
}

// out[t] = sum_j w[t][j] * rows[t*K + j] (pick order, from 0) + sgate[t] * shared[t] + residual[t]
__global__ void __launch_bounds__(256) k_combine(const float* __restrict__ rows, const float* __restrict__ w,
                                                 int T, int K, int H, const float* __restrict__ shared,
                                                 const float* __restrict__ sgate, const float* __restrict__ residual,
                                                 float* __restrict__ out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * H) return;
    int64_t t = i / H, c = i % H;
    float acc = 0.f;
    for (int j = 0; j < K; ++j) acc = __fadd_rn(acc, __fmul_rn(rows[(t * K + j) * H + c], w[t * K + j]));
    if (shared) acc = __fadd_rn(acc, __fmul_rn(shared[t * H + c], sgate[t]));
    if (residual) acc = __fadd_rn(acc, residual[i]);
    out[i] = acc;
}

// ---------------------------------------------------------------- host side
int launch_prep(const float* src, int64_t R, int64_t K, int mode, __half* hi, __half* lo, cudaStream_t st) {
    if (R == 0) return CWX_OK;
    int64_t warps = R * ((K + 255) / 256);
    k_prep<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(src, R, K, mode, hi, lo);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_prep");
}

int launch_combine(const float* rows, const float* w, int T, int K, int H, const float* shared, const float* sgate,
                   const float* residual, float* out, cudaStream_t st) {
    if (T == 0) return CWX_OK;
    int64_t n = (int64_t)T * H;
    k_combine<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(rows, w, T, K, H, shared, sgate, residual, out);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_combine");
}

static int64_t max_piece(const Layout& L) {
    int64_t m = 0;
    for (int kp = 0; kp < L.n_kp; ++kp) {
        int64_t b = piece_bytes(L, 0, kp);
        if (b > m) m = b;
    }
    return m;
}

int launch_gemv(GemvArgs a, int64_t max_items, int device, int sm_count, cudaStream_t st) {
    int64_t b0 = max_piece(a.ra.L), b1 = a.two ? max_piece(a.rb.L) : 0;
    if (a.has_shared) {
        b0 = b0 > max_piece(a.sa.L) ? b0 : max_piece(a.sa.L);
        if (a.two) b1 = b1 > max_piece(a.sb.L) ? b1 : max_piece(a.sb.L);
    }
    a.stage_b_off = (int)pad16(b0);
    a.stage_bytes = (int)pad16(b0 + b1 + 15);
    const int fixed = 128 + 8192 + 2048 + GEMV_WARPS * 4 * 16 * 64 * 2;
    int max_smem = 227 * 1024 - 1024;
    int nst = (max_smem - fixed) / a.stage_bytes;
    if (nst > 6) nst = 6;
    if (nst < 2) return fail(CWX_EUNSUPPORTED, "expert pieces too large for shared memory");
    a.nst = nst;
    int smem = fixed + nst * a.stage_bytes;
    static bool attr_set[64] = {false};
    if (device < 0 || device >= 64 || !attr_set[device]) {
        cudaError_t e = cudaFuncSetAttribute(k_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024 - 1024);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(k_gemv)");
        if (device >= 0 && device < 64) attr_set[device] = true;
    }
    int per_sm = (228 * 1024) / (smem + 1024);
    if (per_sm < 1) per_sm = 1;
    int64_t grid = (int64_t)sm_count * per_sm;
    if (grid > max_items) grid = max_items;
    if (grid < 1) return CWX_OK;
    k_gemv<<<(unsigned)grid, GEMV_THREADS, smem, st>>>(a);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_gemv");
}

}  // namespace cwx
