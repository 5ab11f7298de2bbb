// The fused decode layer: one MoE layer of a small batch (up to 8 tokens) in one launch.
//
//   reference  StreamedMoe::forward, resident decode branch (crates/engine/src/experts.rs:2562-2614):
//              router, route (experts.rs:2364-2372), piles (fuse_kernel.rs:180-202), the gate/up
//              MoeMatvec, ExpertAct::Silu (experts.rs:2389-2406), the down MoeMatvec,
//              cw_weighted_sum (fuse_kernel.rs:277-291) and SharedExpert::forward
//              (crates/engine/src/model_next.rs:731-741) + residual (model_next.rs:1437).
//
// At decode sizes the layer is bound by latency, not bandwidth: a batch of one token reads about
// 10 MB of expert weights, a few microseconds of HBM time, while the eight kernels of the general
// path each pay a launch, a drain and a dependency wait. Here one cooperative grid of one CTA per
// SM (8 warps) runs the layer in three phases with two bounded grid-wide barriers between them:
//   A  router logits (one warp per expert, exact f32 products summed in f64, rounded once) and
//      the shared expert's gates, into the workspace; every CTA also stages the tokens' rows in
//      shared memory and packs their f16 activation fragments (and Q8_K codes for a shared expert
//      under the candle policy);
//   -- barrier --
//   B  every CTA routes every token itself (softmax in candle's AVX order with correctly rounded
//      exp, stable top-k, renormalisation) and builds the piles in shared memory, so no barrier is
//      needed before the products;
//   C  gate/up: work units of (used expert, 16 features) and the shared expert's (16 features),
//      split over four or eight warps along K when a CTA has few of them; the partial sums meet in
//      shared memory and SiLU(gate) * up goes to the hidden rows (f16 per pick in the packed order,
//      f32 rows of the shared expert);
//   -- barrier --
//   D  down and combine: every CTA stages the hidden rows of all picks in shared memory; a CTA owns
//      16 output features; its warps run (used expert, 256-column piece) items and the shared
//      expert's pieces, and the CTA sums each token's picks in pick order, adds the gated shared
//      expert and the residual, and writes the output rows;
//   E  (with a fused RMSNorm only) after a third barrier, one CTA per token normalises its row.
// The expert products are those of the grouped products (products.cuh): exact f16 codebook
// weights on mma.sync with the block scale applied per piece, Q4_K as two exact integer products.
// The weight bytes are read straight from the tiled banks into registers, each warp's loads issued
// ahead of its math; every activation fragment comes from shared memory. The codebook of the
// gate/up format is built during phase A, the down format's after the second barrier in the space
// the staged activation rows leave.
// Each barrier wait is bounded (2 s); on expiry the kernel records CWX_ETIMEOUT and returns.
#include "cwx_common.cuh"
#include "decode.cuh"
#include "kernels.cuh"
#include "products.cuh"

namespace cwx {

constexpr int DL_WARPS = 16, DL_THREADS = DL_WARPS * 32;  // (128 registers a thread)
static_assert(DL_THREADS % NORM_THREADS == 0, "the fused RMSNorm: the first NORM_THREADS threads sum");
static_assert(DL_MAX_T * 16 <= DL_THREADS, "one combine thread per output of a row group");
constexpr int DL_NP = DL_MAX_H / 256;             // pieces of a hidden row
constexpr int DL_MAXPD = DL_MAX_I / 256;          // pieces of an intermediate row
constexpr int DL_HALF = 512;                      // bytes of a piece's hi fragments

struct DlState {
    uint32_t ids[DL_MAX_PICKS];
    float w[DL_MAX_PICKS];
    float sgate[DL_MAX_T];
    uint32_t pairs[DL_MAX_PICKS];    // pick indices grouped by expert (stable)
    uint32_t pos[DL_MAX_PICKS];      // place of pick i in pairs
    uint32_t used[DL_MAX_PICKS][3];  // (expert, first pair, count), ascending expert
    float xqd[DL_MAX_T * DL_NP];     // Q8_K scales of the staged code rows
    unsigned long long target;       // grid barrier count that ends the current barrier (thread 0)
    uint32_t nu;
    int ok;
};

// Shared memory. Phases A to C: the gate/up codebook, the staged activation fragments (f16, then
// Q8_K codes), the tokens' f32 rows and the shared expert's gate row (phase A only), the scratch of
// the routing and of the K-split sums. Phase D, over the same bytes: the down codebook, the hidden
// fragments of every pick, the partial sums and the shared expert's packed rows.
constexpr int DL_XS_BYTES = 2 * DL_MAX_T * DL_NP * DL_HALF;                  // f16 and Q8_K code fragments
constexpr int DL_XF_BYTES = DL_MAX_T * DL_MAX_H * 4;                         // f32 rows
constexpr int DL_HROWS_BYTES = DL_MAX_PICKS * DL_MAXPD * DL_HALF;            // hidden fragments per pick
constexpr int DL_YBUF_FLOATS = DL_MAXPD * DL_MAX_PICKS * 16;                 // per piece, pile place, feature
constexpr int DL_YS_FLOATS = DL_MAXPD * DL_MAX_T * 16;                       // shared expert per piece, token
constexpr int DL_HSP_BYTES = DL_MAX_T * DL_MAXPD * 1024;                     // packed shared hidden rows
constexpr int DL_PHASE_D_BYTES = DL_HROWS_BYTES + (DL_YBUF_FLOATS + DL_YS_FLOATS) * 4 + DL_HSP_BYTES;
constexpr int DL_RED_BYTES = DL_WARPS * 2 * 128 * 4;  // K-slice partial sums; phase B: probabilities
static_assert(DL_RED_BYTES >= DL_MAX_T * DL_MAX_E * 4, "routing rows");
static_assert(DL_XF_BYTES >= (DL_MAX_T * 16 + 16) * 4 + DL_MAX_T * (DL_MAX_E / 32) * DL_MAX_PICKS * 8, "routing scratch");
constexpr int dl_max(int a, int b) { return a > b ? a : b; }

template <int FG, int FD>
struct DlSmem {
    static constexpr int OFF_XS = Tbl<FG>::BYTES, OFF_XF = OFF_XS + DL_XS_BYTES, OFF_GV = OFF_XF + DL_XF_BYTES;
    static constexpr int OFF_RED = OFF_GV + DL_MAX_H * 4;  // phases B and C
    static constexpr int OFF_HROWS = Tbl<FD>::BYTES;
    static constexpr int OFF_ST = dl_max(OFF_RED + DL_RED_BYTES, OFF_HROWS + DL_PHASE_D_BYTES);
    static constexpr int BYTES = OFF_ST + (int)((sizeof(DlState) + 127) & ~(size_t)127);
};

// Grid-wide barrier in two halves (every CTA resident: a cooperative launch), so that a CTA can do
// work of its own between its arrival and the others'. One 64-bit counter holds all arrivals
// since it was zeroed; every barrier of every launch takes exactly gridDim.x of them, so arrival c
// belongs to barrier c / gridDim.x, which is complete when the counter reaches the next multiple.
// Arriving is a single atomic (after the fence that publishes the CTA's writes); waiting polls
// the counter with acquire loads, bounded in time. A barrier that timed out leaves the counter off
// step; the error flag it raises makes the host zero it.
__device__ __forceinline__ void grid_arrive(unsigned long long* bar, DlState* S) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned long long c = atomicAdd(bar, 1ull);
        S->target = (c / gridDim.x + 1) * gridDim.x;
    }
}
__device__ __forceinline__ bool grid_wait(unsigned long long* bar, int* err, DlState* S) {
    if (threadIdx.x == 0) {
        int ok = 1;
        uint64_t t0 = 0;
        for (uint32_t i = 0;; ++i) {
            unsigned long long v;
            asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(bar) : "memory");
            if (v >= S->target) break;
            if (i == 0) t0 = globaltimer_ns();
            else if ((i & 255) == 0 && globaltimer_ns() - t0 > 2000000000ull) {
                dev_error(err, DE_TIMEOUT);
                ok = 0;
                break;
            }
            __nanosleep(20);
        }
        S->ok = ok;
    }
    __syncthreads();
    return S->ok != 0;
}

__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Bytes of the 16-row group starting at feature r0 (a multiple of 16) of expert e, piece kp.
__device__ __forceinline__ const uint8_t* group_ptr(const MatRef& m, uint32_t e, int r0, int kp) {
    const Layout& L = m.L;
    const int64_t rt = r0 / TILE_ROWS, rr = r0 % TILE_ROWS;
    return m.base + (int64_t)e * L.expert_bytes + piece_offset(L, rt, kp) + rr * piece_row_bytes(L, kp);
}

// ---------------------------------------------------------------- phase A
// Router: logits[t][e] for all tokens, one warp per expert; the expert's weight row is loaded into
// wv first (router_row), so its loads are in flight while the CTA stages the tokens' rows.
constexpr int DL_RV = DL_MAX_H / 128;  // float4 of a router row per lane
__device__ __forceinline__ void router_row(const DecodeArgs& a, int e, int lane, float4* wv) {
    const float4* wr = reinterpret_cast<const float4*>(a.router_w + (int64_t)e * a.H);
#pragma unroll
    for (int i = 0; i < DL_RV; ++i)
        if (lane + 32 * i < a.H / 4) wv[i] = wr[lane + 32 * i];
}
__device__ __forceinline__ void router_dot(const DecodeArgs& a, const float* xf, int e, int lane, const float4* wv) {
#pragma unroll 1
    for (int t = 0; t < a.T; ++t) {
        const float4* xr = reinterpret_cast<const float4*>(xf + (int64_t)t * a.H);
        double acc = 0.0;
#pragma unroll
        for (int i = 0; i < DL_RV; ++i)
            if (lane + 32 * i < a.H / 4) {
                const float4 w = wv[i], xv = xr[lane + 32 * i];
                acc = fma((double)w.x, (double)xv.x, acc);
                acc = fma((double)w.y, (double)xv.y, acc);
                acc = fma((double)w.z, (double)xv.z, acc);
                acc = fma((double)w.w, (double)xv.w, acc);
            }
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
            float l = (float)acc;
            if (a.router_b) l = __fadd_rn(l, a.router_b[e]);
            a.logits[(int64_t)t * a.E + e] = l;
        }
    }
}

// The shared expert's gates sigmoid(sum_keepdim(x * gate_inp)), one per token, in candle's AVX
// order (lane L sums the products of columns 32 i + L in order; H is a multiple of 256 here), by
// one warp: gate_load brings gate_inp into the router row's registers, gate_store puts it in shared
// memory (gv), shared_gates writes the gates after the logits (logits[T * E + t]).
__device__ __forceinline__ void gate_load(const DecodeArgs& a, int lane, float4* wv) {
    const float4* src = reinterpret_cast<const float4*>(a.sg_inp);
#pragma unroll
    for (int i = 0; i < DL_RV; ++i)
        if (lane + 32 * i < a.H / 4) wv[i] = src[lane + 32 * i];
}
__device__ __forceinline__ void gate_store(const DecodeArgs& a, const float4* wv, float* gv, int lane) {
#pragma unroll
    for (int i = 0; i < DL_RV; ++i)
        if (lane + 32 * i < a.H / 4) reinterpret_cast<float4*>(gv)[lane + 32 * i] = wv[i];
    __syncwarp();
}
__device__ __forceinline__ void shared_gates(const DecodeArgs& a, const float* xf, const float* gv, int lane) {
#pragma unroll 1
    for (int t = 0; t < a.T; ++t) {
        const float* xr = xf + (int64_t)t * a.H;
        float acc = 0.f;
#pragma unroll 4
        for (int i = lane; i < a.H; i += 32) acc = __fadd_rn(acc, __fmul_rn(xr[i], gv[i]));
        const float sum = avx_lane_tree(acc);
        if (lane == 0) a.logits[(int64_t)a.T * a.E + t] = __fdiv_rn(1.0f, __fadd_rn(exp_cr(-sum), 1.0f));
    }
}

// Piece kp of token t: its f16 (mode AM_F32) or Q8_K code (AM_Q8_K) fragments, hi parts, into the
// staged rows; Q8_K scales into S->xqd.
__device__ __forceinline__ void stage_x(const DecodeArgs& a, const float* xf, int t, int kp, int mode, uint8_t* dst,
                                        DlState* S, int lane) {
    const int np = a.H / 256;
    float v[8];
    const float4* src = reinterpret_cast<const float4*>(xf + (int64_t)t * a.H + kp * 256 + 8 * lane);
    const float4 p0 = src[0], p1 = src[1];
    v[0] = p0.x, v[1] = p0.y, v[2] = p0.z, v[3] = p0.w, v[4] = p1.x, v[5] = p1.y, v[6] = p1.z, v[7] = p1.w;
    uint4 hi, lo;
    float d;
    const int ch = pack_words(mode, v, lane, &hi, &lo, &d);
    *reinterpret_cast<uint4*>(dst + (t * np + kp) * DL_HALF + 16 * ch) = hi;
    if (mode == AM_Q8_K && lane == 0) S->xqd[t * np + kp] = d;
}

// ---------------------------------------------------------------- phase B
// Floats onto unsigned ints, order kept (for the warp's max reduction).
__device__ __forceinline__ unsigned f_key(float f) {
    const unsigned u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_f(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Routing of all T tokens by the whole CTA: each token's picks (best first, ties to the lowest id)
// and weights, with the same arithmetic as k_route (route.cu): softmax over the logits with the
// denominator in candle's AVX order and exp correctly rounded, probabilities compared after the
// division, weights renormalised in pick order. The experts of a token are cut into chunks of 32
// (chunk c of token t: experts 32 c + lane); each warp takes chunks, and every step that needs a
// whole token (its maximum, its denominator, the merge of the chunks' bests) is a short one after
// a barrier. A chunk's best K come out of K rounds of a max reduction over (probability, lowest
// id); a token's picks are the K best of its chunks' candidates, ranked by counting. pr holds the
// token rows (T * E floats), scratch the chunk maxima, the denominators and the candidates. NaN
// probabilities rank below every number.
__device__ __forceinline__ unsigned prob_key(float p) { return p == p ? f_key(p) : 1u; }

__device__ __forceinline__ void route_all(const DecodeArgs& a, DlState* S, float* pr, float* scratch, int warp, int lane) {
    const int T = a.T, E = a.E, K = a.K, nch = (E + 31) / 32, nc = T * nch;
    float* cmax = scratch;                       // (T * nch)
    float* tsum = scratch + DL_MAX_T * 16;       // (T)
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(scratch + DL_MAX_T * 16 + 16);  // (T, nch, K)
    for (int c = warp; c < nc; c += DL_WARPS) {  // the logits, the chunks' maxima
        const int t = c / nch, e = 32 * (c % nch) + lane;
        const float v = e < E ? a.logits[(int64_t)t * E + e] : -INFINITY;
        if (e < E) pr[t * E + e] = v;
        float m = v;
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) cmax[c] = m;
    }
    __syncthreads();
    for (int c = warp; c < nc; c += DL_WARPS) {  // exp(v - max)
        const int t = c / nch, e = 32 * (c % nch) + lane;
        float mx = cmax[t * nch];
        for (int j = 1; j < nch; ++j) mx = fmaxf(mx, cmax[t * nch + j]);
        if (e < E) pr[t * E + e] = exp_cr(__fsub_rn(pr[t * E + e], mx));
    }
    __syncthreads();
    if (warp < T) {  // the denominator: lane L sums experts 32 s + L over the whole steps, in order
        const float* row = pr + warp * E;
        const int whole = E / 32;
        float acc = 0.f;
#pragma unroll 4
        for (int s2 = 0; s2 < whole; ++s2) acc = __fadd_rn(acc, row[32 * s2 + lane]);
        float sum = avx_lane_tree(acc);
        for (int j = whole * 32; j < E; ++j) sum = __fadd_rn(sum, row[j]);  // the tail, in order
        if (lane == 0) tsum[warp] = sum;
    }
    __syncthreads();
    for (int c = warp; c < nc; c += DL_WARPS) {  // each chunk's best K
        const int t = c / nch, e = 32 * (c % nch) + lane;
        unsigned hi = e < E ? prob_key(__fdiv_rn(pr[t * E + e], tsum[t])) : 0u;
        for (int r = 0; r < K; ++r) {
            const unsigned mk = __reduce_max_sync(0xffffffffu, hi);
            const unsigned bi = __reduce_min_sync(0xffffffffu, hi == mk ? (unsigned)e : 0xffffffffu);
            if (lane == 0) cand[(int64_t)c * K + r] = ((unsigned long long)mk << 32) | (0xffffffffu - bi);
            if ((unsigned)e == bi) hi = 0u;  // taken
        }
    }
    __syncthreads();
    if (warp < T) {  // the token's K best candidates, by rank
        const int t = warp, C = nch * K;
        const unsigned long long* ck = cand + (int64_t)t * C;
        for (int i = lane; i < C; i += 32) {
            const unsigned long long k = ck[i];
            int rank = 0;
#pragma unroll 4
            for (int j = 0; j < C; ++j) rank += ck[j] > k;
            if (rank < K) {
                S->ids[t * K + rank] = 0xffffffffu - (uint32_t)k;
                S->w[t * K + rank] = key_f((unsigned)(k >> 32));
            }
        }
        __syncwarp();
        if (a.norm) {
            float tot = 0.f;
            for (int r = 0; r < K; ++r) tot = __fadd_rn(tot, S->w[t * K + r]);
            __syncwarp();
            if (lane < K) S->w[t * K + lane] = __fdiv_rn(S->w[t * K + lane], tot);
        }
    }
}

// Piles of the n <= 32 picks (one warp, lane i = pick i): stable by expert, used experts ascending.
__device__ __forceinline__ void build_piles(DlState* S, int n, int lane) {
    const bool in = lane < n;
    const uint32_t e = in ? S->ids[lane] : 0xffffffffu;
    const unsigned same = __match_any_sync(0xffffffffu, e);  // the picks of this pick's expert
    const bool first = in && __ffs(same) - 1 == lane;
    const uint32_t firsts = __ballot_sync(0xffffffffu, first);
    uint32_t less = 0, dless = 0;  // picks, and used experts, below e
#pragma unroll 8
    for (int j = 0; j < 32; ++j) {
        const uint32_t f = __shfl_sync(0xffffffffu, e, j);
        const bool below = j < n && f < e;
        less += below;
        dless += below && ((firsts >> j) & 1u);
    }
    if (in) {
        const uint32_t rank = __popc(same & ((1u << lane) - 1u));
        S->pos[lane] = less + rank;
        S->pairs[less + rank] = (uint32_t)lane;
        if (first) {
            S->used[dless][0] = e;
            S->used[dless][1] = less;
            S->used[dless][2] = (uint32_t)__popc(same);
        }
    }
    if (lane == 0) S->nu = (uint32_t)__popc(firsts);
}

// ---------------------------------------------------------------- phase C
// A gate/up unit: 16 features (feat0 ..) of used expert e (its pile: first, cnt), or of the
// shared expert; xr = this thread's staged activation row (slot g of the pile) at its chunk.
struct UnitInfo {
    bool routed;
    uint32_t e, first, cnt;
    int feat0;
    const uint8_t* xr;
};
__device__ __forceinline__ UnitInfo unit_info(const DecodeArgs& a, const DlState* S, const uint8_t* xs, int q,
                                              int rgs, int nu, int g, int c4) {
    UnitInfo u;
    const int np = a.H / 256;
    u.routed = q < nu * rgs;
    if (u.routed) {
        const int k = q / rgs;
        u.feat0 = (q % rgs) * 16;
        u.e = S->used[k][0];
        u.first = S->used[k][1];
        u.cnt = S->used[k][2];
        const uint32_t pick = S->pairs[u.first + ((uint32_t)g < u.cnt ? g : 0)];
        u.xr = xs + (int)(pick / a.K) * np * DL_HALF + 16 * c4;
    } else {
        u.feat0 = (q - nu * rgs) * 16;
        u.e = u.first = u.cnt = 0;
        u.xr = nullptr;
    }
    return u;
}

// Rows g and g + 8 of one piece of a shared-expert matrix (Q4_K).
struct ShRows {
    Q4Raw a, b;
};
__device__ __forceinline__ void sh_load(const MatRef& m, int feat0, int kp, int g, int c4, ShRows& r) {
    const uint8_t* p = group_ptr(m, 0, feat0, kp);
    r.a = q4_raw(p + g * 144, c4);
    r.b = q4_raw(p + (g + 8) * 144, c4);
}
// Their products for piece kp: token slot g's staged fragments (f16, or Q8_K codes with the scales
// of the thread's two output tokens).
__device__ __forceinline__ void sh_compute(const DecodeArgs& a, const DlState* S, const uint8_t* xs, const ShRows& r,
                                           int kp, int g, int c4, float* acc) {
    const int np = a.H / 256, T = a.T, tg = g < T ? g : 0;
    const int t0 = 2 * c4 < T ? 2 * c4 : 0, t1 = 2 * c4 + 1 < T ? 2 * c4 + 1 : 0;
    const uint8_t* src = a.sh_qint ? xs + DL_MAX_T * DL_NP * DL_HALF : xs;
    const uint8_t* brow = src + (tg * np + kp) * DL_HALF + 16 * c4;
    const DxAt dx{reinterpret_cast<const uint8_t*>(&S->xqd[t0 * np + kp]),
                  reinterpret_cast<const uint8_t*>(&S->xqd[t1 * np + kp])};
    q4k_rows<1>(q4_row_of(r.a, c4), q4_row_of(r.b, c4), brow, 0, false, a.sh_qint != 0, dx, acc);
}

// h = SiLU(gate) * up of a finished unit: f16 at the features' places of each pick's hidden
// fragments (hi parts, packed order), or f32 rows of the shared expert.
__device__ __forceinline__ void gu_epilogue(const DecodeArgs& a, const DlState* S, const UnitInfo& ui, const float* ag,
                                            const float* au, int g, int c4) {
    const int npd = a.I / 256;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t slot = 2 * c4 + (i & 1);
        const int feat = ui.feat0 + g + ((i >> 1) ? 8 : 0);
        const float h = __fmul_rn(silu_f(ag[i]), au[i]);
        if (ui.routed) {
            if (slot < ui.cnt) {
                const uint32_t pick = S->pairs[ui.first + slot];
                const int kp = feat >> 8, k = feat & 255;
                const int ch = (((k >> 4) & 3) * 2 + ((k >> 3) & 1)) * 4 + (k >> 6);
                *reinterpret_cast<__half*>(a.hpk + ((int64_t)pick * npd + kp) * DL_HALF + ch * 16 + (k & 7) * 2) =
                    __float2half_rn(h);
            }
        } else if (slot < (uint32_t)a.T) {
            a.hs[(int64_t)slot * a.Is + feat] = h;
        }
    }
}

// ---------------------------------------------------------------- phase D
// Routed item m = (used expert m / npd, piece m % npd) of the CTA's 16 output features.
template <int FD>
__device__ __forceinline__ void down_load(const DecodeArgs& a, const DlState* S, int m, int npd, int feat0, int g, int c4,
                                          FastIn& in) {
    fast_load<FD>(group_ptr(a.down, S->used[m / npd][0], feat0, m % npd), 0, g, c4, in);
}
template <int FD>
__device__ __forceinline__ void down_item(const DlState* S, const FastIn& in, int m, int npd, const uint8_t* tl,
                                          const uint8_t* hrows, int g, int c4, float* ybuf) {
    const int u = m / npd, kp = m % npd;
    const uint32_t first = S->used[u][1], cnt = S->used[u][2];
    const uint32_t pick = S->pairs[first + ((uint32_t)g < cnt ? g : 0)];
    const uint8_t* brow = hrows + (pick * npd + kp) * DL_HALF + 16 * c4;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    fast_compute<FD, 1>(in, tl, brow, 0, false, acc);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t slot = 2 * c4 + (i & 1);
        if (slot < cnt) ybuf[(kp * DL_MAX_PICKS + first + slot) * 16 + g + ((i >> 1) ? 8 : 0)] = acc[i];
    }
}

// The l-th of n 128-byte lines of [p, p + bytes) into L2 (every thread of the CTA takes some).
__device__ __forceinline__ void prefetch_share(const uint8_t* p, int64_t bytes, int part, int parts) {
    const int64_t lines = (bytes + 127) / 128, per = (lines + parts - 1) / parts;
    const int64_t l0 = (int64_t)part * per, l1 = l0 + per < lines ? l0 + per : lines;
    for (int64_t l = l0 + threadIdx.x; l < l1; l += blockDim.x) prefetch_l2(p + 128 * l);
}

template <int FG, int FD>
__global__ void __launch_bounds__(DL_THREADS, 1) k_decode_layer(DecodeArgs a) {
    using SM = DlSmem<FG, FD>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* tblG = smem;                                        // phases A - C
    uint8_t* xs = smem + SM::OFF_XS;                             // phases A - C
    float* xf = reinterpret_cast<float*>(smem + SM::OFF_XF);     // phase A
    float* gv = reinterpret_cast<float*>(smem + SM::OFF_GV);     // phase A
    uint8_t* tblD = smem;                                        // phase D
    uint8_t* hrows = smem + SM::OFF_HROWS;                       // phase D
    float* ybuf = reinterpret_cast<float*>(hrows + DL_HROWS_BYTES);
    float* ysb = ybuf + DL_YBUF_FLOATS;
    uint8_t* hsp = reinterpret_cast<uint8_t*>(ysb + DL_YS_FLOATS);
    float* red = reinterpret_cast<float*>(smem + SM::OFF_RED);
    DlState* S = reinterpret_cast<DlState*>(smem + SM::OFF_ST);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, c4 = lane & 3;
    const int T = a.T, H = a.H, K = a.K, n = T * K;
    const int nct = gridDim.x;
    const int np = H / 256;
    const bool shared = a.sg.base != nullptr;

    // ---------------- A: router logits; the tokens' rows staged, their fragments and gates
    {
        // Everything that reads only weights starts before the wait for the kernel before (the
        // weights are written by no kernel): this warp's router row (expert blockIdx + nct * warp)
        // into registers, the shared expert's weights into L2 (a share per CTA; the phases that
        // read them find them there), the gate/up codebook.
        float4 wv[DL_RV];
        const int e0 = (int)blockIdx.x + nct * warp;
        const int nrows = a.E + (shared ? 1 : 0);  // the router rows and the shared expert's gate row
        if (e0 < a.E) router_row(a, e0, lane, wv);
        else if (e0 < nrows) gate_load(a, lane, wv);
        if (shared) {
            prefetch_share(a.sg.base, a.sg.L.expert_bytes, blockIdx.x, nct);
            prefetch_share(a.su.base, a.su.L.expert_bytes, blockIdx.x, nct);
            prefetch_share(a.sd.base, a.sd.L.expert_bytes, blockIdx.x, nct);
        }
        build_tables<FG, DL_THREADS>(tblG, tid);
        pdl_wait();
        for (int i = tid; i < T * H / 4; i += DL_THREADS)
            reinterpret_cast<float4*>(xf)[i] = reinterpret_cast<const float4*>(a.x)[i];
        __syncthreads();
        for (int e = e0; e < nrows; e += nct * DL_WARPS) {
            if (e < a.E) {
                if (e != e0) router_row(a, e, lane, wv);
                router_dot(a, xf, e, lane, wv);
            } else {
                if (e != e0) gate_load(a, lane, wv);
                gate_store(a, wv, gv, lane);
                shared_gates(a, xf, gv, lane);
            }
        }
        // the fragments, by the warps without router rows first
        const int nq8 = shared && a.sh_qint ? T * np : 0;
        for (int u = DL_WARPS - 1 - warp; u < T * np + nq8; u += DL_WARPS) {
            if (u < T * np) stage_x(a, xf, u / np, u % np, AM_F32, xs, S, lane);
            else stage_x(a, xf, (u - T * np) / np, (u - T * np) % np, AM_Q8_K, xs + DL_MAX_T * DL_NP * DL_HALF, S, lane);
        }
        grid_arrive(a.bar, S);  // the logits and gates are written
    }
    if (!grid_wait(a.bar, a.err, S)) return;

    // ---------------- B: routing and piles in every CTA
    if (shared && tid < T) S->sgate[tid] = a.logits[(int64_t)T * a.E + tid];
    route_all(a, S, red, xf, warp, lane);  // (the f32 rows are no longer needed)
    __syncthreads();
    if (warp == 0) build_piles(S, n, lane);
    __syncthreads();
    const int npd = a.I / 256;
    {
        // this CTA's down groups (its output features of every used expert) into L2 while the
        // gate/up products run
        const int nu = (int)S->nu;
        for (int rg = blockIdx.x; rg < H / 16; rg += nct)
            for (int m = warp; m < nu * npd; m += DL_WARPS) {
                const int kp = m % npd;
                const uint8_t* p = group_ptr(a.down, S->used[m / npd][0], rg * 16, kp);
                const int lines = (16 * (int)piece_row_bytes(a.down.L, kp) + 127) / 128;
                for (int l = lane; l < lines; l += 32) prefetch_l2(p + 128 * l);
            }
    }
    if (blockIdx.x == 0) {  // the routing taps
        for (int i = tid; i < n; i += DL_THREADS) {
            if (a.ids_out) a.ids_out[i] = S->ids[i];
            if (a.w_out) a.w_out[i] = S->w[i];
            if (a.pairs_out) a.pairs_out[i] = S->pairs[i];
        }
        if (a.heads_out)
            for (int e = tid; e < a.E; e += DL_THREADS) {
                uint32_t first = 0, cnt = 0;
                for (int i = 0; i < n; ++i) {
                    first += S->ids[i] < (uint32_t)e;
                    cnt += S->ids[i] == (uint32_t)e;
                }
                a.heads_out[3 * e] = (uint32_t)e;
                a.heads_out[3 * e + 1] = first;
                a.heads_out[3 * e + 2] = cnt;
            }
    }

    // ---------------- C: gate/up units (16 features of a used expert, or of the shared expert)
    // A warp's work is a list of items (unit, piece, matrix), each one piece of one matrix.
    {
        const uint8_t* tlG = tblG + tbl_lane(FG, lane);
        const int rgs = a.I / 16, srgs = shared ? a.Is / 16 : 0;
        const int nu = (int)S->nu, nru = nu * rgs;
        const int units = nru + srgs;
        const int mine = units > (int)blockIdx.x ? (units - 1 - (int)blockIdx.x) / nct + 1 : 0;
        // A unit's items: (piece kp, matrix) as 2 kp + (0 gate, 1 up). Few units (small batches):
        // each unit's items split over nks warps (a power of two, as many as the units leave room
        // for), whose partial sums meet in shared memory; more: whole units per warp.
        int nks = 1;  // (mine may be 0: this CTA then has no units and skips the loops below)
        if (mine > 0)
            while (nks < DL_WARPS && nks * 2 * mine <= DL_WARPS) nks *= 2;
        const int ks = warp % nks, lu0 = warp / nks;
        const int i0 = ks * 2 * np / nks, ipu = (ks + 1) * 2 * np / nks - i0;  // this warp's items of a unit
        // this warp's units lu0, lu0 + DL_WARPS, ... below mine; unit q = blockIdx + lu * nct is
        // routed when q < nru, so the routed ones come first
        int nw = 0, nrw = 0;
        for (int lu = lu0; lu < mine; lu += DL_WARPS) {
            ++nw;
            nrw += (int)blockIdx.x + lu * nct < nru;
        }
        auto unit_q = [&](int k) { return (int)blockIdx.x + (lu0 + DL_WARPS * k) * nct; };
        float ag[4] = {0.f, 0.f, 0.f, 0.f}, au[4] = {0.f, 0.f, 0.f, 0.f};
        // Items run in a loop unrolled by the depth of the load queue (four sets of registers,
        // loads three items ahead): each load lands in the set the item before it freed, so no
        // register has to wait for a load to move it.
        {  // routed items
            const int n = nrw * ipu;
            auto load = [&](int i, FastIn& f) {
                const int q = unit_q(i / ipu), r = i0 + i % ipu;
                fast_load<FG>(group_ptr((r & 1) ? a.up : a.gate, S->used[q / rgs][0], (q % rgs) * 16, r >> 1), 0, g, c4, f);
            };
            auto step = [&](int i, const FastIn& cur) {
                const int r = i0 + i % ipu;
                const bool up = r & 1;
                const UnitInfo ui = unit_info(a, S, xs, unit_q(i / ipu), rgs, nu, g, c4);
                float t[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) t[j] = up ? au[j] : ag[j];
                fast_compute<FG, 1>(cur, tlG, ui.xr + (r >> 1) * DL_HALF, 0, false, t);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    au[j] = up ? t[j] : au[j];
                    ag[j] = up ? ag[j] : t[j];
                }
                if (nks == 1 && i % ipu == ipu - 1) {
                    gu_epilogue(a, S, ui, ag, au, g, c4);
#pragma unroll
                    for (int j = 0; j < 4; ++j) ag[j] = au[j] = 0.f;
                }
            };
            FastIn f0, f1, f2, f3;
            if (n > 0) load(0, f0);
            if (n > 1) load(1, f1);
            if (n > 2) load(2, f2);
#pragma unroll 1
            for (int i = 0; i < n; i += 4) {
                if (i + 3 < n) load(i + 3, f3);
                step(i, f0);
                if (i + 1 < n) {
                    if (i + 4 < n) load(i + 4, f0);
                    step(i + 1, f1);
                }
                if (i + 2 < n) {
                    if (i + 5 < n) load(i + 5, f1);
                    step(i + 2, f2);
                }
                if (i + 3 < n) {
                    if (i + 6 < n) load(i + 6, f2);
                    step(i + 3, f3);
                }
            }
        }
        {  // the shared expert's items (from L2: prefetched at the start), one load ahead
            const int n = (nw - nrw) * ipu;
            auto load = [&](int i, ShRows& rr) {
                const int q = unit_q(nrw + i / ipu), r = i0 + i % ipu;
                sh_load((r & 1) ? a.su : a.sg, (q - nru) * 16, r >> 1, g, c4, rr);
            };
            auto step = [&](int i, const ShRows& cur) {
                const int r = i0 + i % ipu;
                const bool up = r & 1;
                float t[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) t[j] = up ? au[j] : ag[j];
                sh_compute(a, S, xs, cur, r >> 1, g, c4, t);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    au[j] = up ? t[j] : au[j];
                    ag[j] = up ? ag[j] : t[j];
                }
                if (nks == 1 && i % ipu == ipu - 1) {
                    gu_epilogue(a, S, unit_info(a, S, xs, unit_q(nrw + i / ipu), rgs, nu, g, c4), ag, au, g, c4);
#pragma unroll
                    for (int j = 0; j < 4; ++j) ag[j] = au[j] = 0.f;
                }
            };
            ShRows f0, f1;
            if (n > 0) load(0, f0);
#pragma unroll 1
            for (int i = 0; i < n; i += 2) {
                if (i + 1 < n) load(i + 1, f1);
                step(i, f0);
                if (i + 1 < n) {
                    if (i + 2 < n) load(i + 2, f0);
                    step(i + 1, f1);
                }
            }
        }
        if (nks > 1) {
            // the K-slices' partial sums meet in shared memory; slice 0 adds them in slice order
            if (ks > 0) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    red[(warp * 2 + 0) * 128 + lane * 4 + i] = ag[i];
                    red[(warp * 2 + 1) * 128 + lane * 4 + i] = au[i];
                }
            }
            __syncthreads();
            if (ks == 0 && nw > 0) {
                for (int k2 = 1; k2 < nks; ++k2)
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        ag[i] = __fadd_rn(ag[i], red[((warp + k2) * 2 + 0) * 128 + lane * 4 + i]);
                        au[i] = __fadd_rn(au[i], red[((warp + k2) * 2 + 1) * 128 + lane * 4 + i]);
                    }
                gu_epilogue(a, S, unit_info(a, S, xs, unit_q(0), rgs, nu, g, c4), ag, au, g, c4);
            }
        }
    }
    // the hidden rows are written; the down codebook is built over the gate/up one while the other
    // CTAs finish theirs
    grid_arrive(a.bar, S);
    build_tables<FD, DL_THREADS>(tblD, tid);
    if (!grid_wait(a.bar, a.err, S)) return;

    // ---------------- D: down products and the combine, 16 output features per CTA
    {
        const int nps = shared ? a.Is / 256 : 0;
        const int64_t hsrow = (int64_t)nps * 1024;
        // every pick's hidden fragments; the shared expert's hidden rows packed (Q8_K codes or f16)
        for (int i = tid; i < n * npd * DL_HALF / 16; i += DL_THREADS)
            reinterpret_cast<uint4*>(hrows)[i] = reinterpret_cast<const uint4*>(a.hpk)[i];
        if (shared) {
            for (int u = warp; u < T * nps; u += DL_WARPS) {
                const int t = u / nps, kp = u % nps;
                float v[8];
                const float4* src = reinterpret_cast<const float4*>(a.hs + (int64_t)t * a.Is + kp * 256 + 8 * lane);
                const float4 p0 = src[0], p1 = src[1];
                v[0] = p0.x, v[1] = p0.y, v[2] = p0.z, v[3] = p0.w, v[4] = p1.x, v[5] = p1.y, v[6] = p1.z, v[7] = p1.w;
                pack_piece(a.sh_qint ? AM_Q8_K : AM_F32, v, hsp + (int64_t)t * hsrow + kp * 1024, lane);
            }
        }
        __syncthreads();
        const uint8_t* tlD = tblD + tbl_lane(FD, lane);
        const int nu = (int)S->nu;
        const int nr = nu * npd;  // routed items (used expert, piece)
        const int cw = nr > warp ? (nr - 1 - warp) / DL_WARPS + 1 : 0;  // this warp's: warp + 8 j
        for (int rg = blockIdx.x; rg < H / 16; rg += nct) {
            const int feat0 = rg * 16;
            // the residual of the combine thread's output, requested first
            const float resv = a.residual && tid < T * 16 ? a.residual[(int64_t)(tid / 16) * H + feat0 + tid % 16] : 0.f;
            // routed items, loads three items ahead of the math (four sets of registers, as in C)
            FastIn f0, f1, f2, f3;
            auto load = [&](int j, FastIn& f) { down_load<FD>(a, S, warp + j * DL_WARPS, npd, feat0, g, c4, f); };
            auto step = [&](int j, const FastIn& cur) {
                down_item<FD>(S, cur, warp + j * DL_WARPS, npd, tlD, hrows, g, c4, ybuf);
            };
            if (cw > 0) load(0, f0);
            if (cw > 1) load(1, f1);
            if (cw > 2) load(2, f2);
#pragma unroll 1
            for (int j = 0; j < cw; j += 4) {
                if (j + 3 < cw) load(j + 3, f3);
                step(j, f0);
                if (j + 1 < cw) {
                    if (j + 4 < cw) load(j + 4, f0);
                    step(j + 1, f1);
                }
                if (j + 2 < cw) {
                    if (j + 5 < cw) load(j + 5, f1);
                    step(j + 2, f2);
                }
                if (j + 3 < cw) {
                    if (j + 6 < cw) load(j + 6, f2);
                    step(j + 3, f3);
                }
            }
            // the shared expert's pieces, on the warps with the fewest routed items
#pragma unroll 1
            for (int kp = DL_WARPS - 1 - warp; kp < nps; kp += DL_WARPS) {
                const uint8_t* p = group_ptr(a.sd, 0, feat0, kp);
                const Q4Raw ra = q4_raw(p + g * 144, c4), rb = q4_raw(p + (g + 8) * 144, c4);
                const int tg = g < T ? g : 0;
                const int t0 = 2 * c4 < T ? 2 * c4 : 0, t1 = 2 * c4 + 1 < T ? 2 * c4 + 1 : 0;
                const uint8_t* brow = hsp + (int64_t)tg * hsrow + (int64_t)kp * 1024 + 16 * c4;
                const DxAt dx{hsp + (int64_t)t0 * hsrow + (int64_t)kp * 1024 + 512,
                              hsp + (int64_t)t1 * hsrow + (int64_t)kp * 1024 + 512};
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                q4k_rows<1>(q4_row_of(ra, c4), q4_row_of(rb, c4), brow, 0, false, a.sh_qint != 0, dx, acc);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int slot = 2 * c4 + (i & 1);
                    if (slot < T) ysb[(kp * DL_MAX_T + slot) * 16 + g + ((i >> 1) ? 8 : 0)] = acc[i];
                }
            }
            __syncthreads();
            // out[t][f] = sum over picks in order of w * y, + sgate * shared, + residual
            if (tid < T * 16) {
                const int t = tid / 16, f = tid % 16;
                float acc = 0.f;
                for (int j = 0; j < K; ++j) {
                    const int i = t * K + j;
                    const uint32_t ps = S->pos[i];
                    float y = ybuf[ps * 16 + f];
                    for (int kp = 1; kp < npd; ++kp) y = __fadd_rn(y, ybuf[(kp * DL_MAX_PICKS + ps) * 16 + f]);
                    acc = __fadd_rn(acc, __fmul_rn(y, S->w[i]));
                }
                if (shared) {
                    float ys = ysb[t * 16 + f];
                    for (int kp = 1; kp < nps; ++kp) ys = __fadd_rn(ys, ysb[(kp * DL_MAX_T + t) * 16 + f]);
                    acc = __fadd_rn(acc, __fmul_rn(ys, S->sgate[t]));
                }
                if (a.residual) acc = __fadd_rn(acc, resv);
                a.out[(int64_t)t * H + feat0 + f] = acc;
            }
            __syncthreads();  // ybuf is reused by the next row group
        }
    }
    if (!a.norm_w) return;
    // ---------------- E: the next layer's RMSNorm of each output row (as k_combine_norm: the same
    // squares in the same order, so norm_out matches the general path and the standalone add_norm)
    grid_arrive(a.bar, S);
    if (!grid_wait(a.bar, a.err, S)) return;
    for (int t = blockIdx.x; t < T; t += nct) {
        const float* row = a.out + (int64_t)t * H;
        double ss = 0.0;
        if (tid < NORM_THREADS)
            for (int q = tid; q < H / 4; q += NORM_THREADS) ss += sq4(reinterpret_cast<const float4*>(row)[q]);
        norm_row<DL_THREADS>(ss, row, a.norm_w, a.norm_eps, H, a.norm_vec != 0, a.norm_out + (int64_t)t * H);
    }
}

template <int FG, int FD>
static int launch_dl(const DecodeArgs& a, int device, int sm_count, cudaStream_t st) {
    static_assert(DlSmem<FG, FD>::BYTES <= 227 * 1024, "k_decode_layer: shared memory above a CTA's 227 KB");
    const int smem = DlSmem<FG, FD>::BYTES;
    static int attr_set[64] = {0};
    if (device < 0 || device >= 64 || !attr_set[device]) {
        cudaError_t e = cudaFuncSetAttribute(k_decode_layer<FG, FD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(k_decode_layer)");
        int nb = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k_decode_layer<FG, FD>, DL_THREADS, smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor(k_decode_layer)");
        if (nb < 1) return fail(CWX_EUNSUPPORTED, "k_decode_layer: no block fits an SM");
        if (device >= 0 && device < 64) attr_set[device] = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)sm_count);
    cfg.blockDim = dim3(DL_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: the grid barriers need it
    at[0].val.cooperative = 1;
    // programmatic serialisation: the codebook build overlaps the end of the kernel before
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    static int pdl_ok = 1;  // cleared if the driver refuses the pair of attributes
    cfg.numAttrs = pdl_ok ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_decode_layer<FG, FD>, a);
    if (e != cudaSuccess && pdl_ok) {
        (void)cudaGetLastError();
        pdl_ok = 0;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, k_decode_layer<FG, FD>, a);
    }
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_decode_layer");
}

bool decode_fused_formats(int gf, int df) {
    return (gf == F_IQ2_S && df == F_IQ3_S) || (gf == F_IQ2_XXS && df == F_IQ3_XXS) ||
           (gf == F_IQ3_S && df == F_IQ2_S) || (gf == F_IQ3_XXS && df == F_IQ2_XXS);
}

int launch_decode_layer(const DecodeArgs& a, int device, int sm_count, cudaStream_t st) {
    const int gf = a.gate.L.fmt, df = a.down.L.fmt;
    if (gf == F_IQ2_S && df == F_IQ3_S) return launch_dl<F_IQ2_S, F_IQ3_S>(a, device, sm_count, st);
    if (gf == F_IQ2_XXS && df == F_IQ3_XXS) return launch_dl<F_IQ2_XXS, F_IQ3_XXS>(a, device, sm_count, st);
    if (gf == F_IQ3_S && df == F_IQ2_S) return launch_dl<F_IQ3_S, F_IQ2_S>(a, device, sm_count, st);
    if (gf == F_IQ3_XXS && df == F_IQ2_XXS) return launch_dl<F_IQ3_XXS, F_IQ2_XXS>(a, device, sm_count, st);
    return fail(CWX_EUNSUPPORTED, "k_decode_layer: formats %d / %d", gf, df);
}

}  // namespace cwx
