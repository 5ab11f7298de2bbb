// Grouped expert products (decode-sized piles): the B200 form of MoeMatvec.
//
//   reference  MoeMatvec (crates/engine/src/experts.rs:2183-2309) -> kernel_mul_mv_id_* and
//              kernel_mul_mm_idg_* (crates/engine/src/mv_id.rs:17-384,
//              vendor/candle-metal-kernels/src/metal_src/quantized.metal:7668-7766, 7868-7911).
//
// A launch runs up to four matrix jobs (routed gate, routed up, shared gate, shared up; or routed
// down, shared down). Work items are (job, expert, R-row tile) over the experts that have picks
// (the used list the pile kernels build) and (job, tile, pass) for the shared expert, walked by a
// persistent grid. A CTA has 8 consumer warps and one producer warp. Consumer warp w owns rows
// 16*(w % (R/16)) of the tile and K-slice w / (R/16) (KS slices, R = 128/KS, so small batches
// split K across warps and still fill the GPU). The producer runs ahead through the CTA's steps:
// for each it writes a small header (item, pass, the pass's output rows) into a free stage and
// brings, in one mbarrier phase, the tile's quantised bytes for KS pieces of 256 columns
// (cp.async.bulk from the tiled bank layout) and the pile's packed activation rows for those
// columns. Producer and consumers meet only on full/empty mbarriers.
//
// Each thread dequantises two rows x 64 contiguous columns of a piece straight into mma.sync
// m16n8k16 A registers, 16 columns per sub-step. The reduction index of an MMA step is permuted
// (thread c of a quad contributes 4 of its own columns), legal because A and B use the same
// permutation; the activation rows arrive packed in exactly that order (act.cu), so every thread
// reads its 16 activation columns with four conflict-free 16-byte loads. Activations are an f16
// hi + lo pair (~22 bits); weights are f16 (IQ formats, F32 policy) or an f16 hi + lo pair when
// the result is re-quantised downstream. f32 accumulation; K-slices summed in a fixed order.
#include "cwx_common.cuh"
#include "decode.cuh"
#include "kernels.cuh"

namespace cwx {

constexpr int GEMV_THREADS = 256;  // consumer threads (the producer warp comes on top)
// K-slice partial sums: slices 1..KS-1 of every m-tile, one 16x8 fragment (128 floats) each;
// (KS - 1) * (R / 16) * 128 <= 7 * 128 floats for every KS, double-buffered by pass parity.
constexpr int RED_FLOATS = 7 * 128;
constexpr int RED_BYTES = 2 * RED_FLOATS * 4;

struct Item {
    int job;
    uint32_t e, first, count;
    int64_t rt;  // tile index in R-row units
    int rows;    // rows of this tile (multiple of 16)
    int n_kp;    // 256-column pieces per row
    int nsk;     // steps per pass (ceil(n_kp / KS))
    int pass0;   // first pass of this item
    int passes;  // passes this item runs
};

template <int KS>
struct Cfg {
    static constexpr int R = 128 / KS;           // rows per item
    static constexpr int MT = R / 16;            // m-tiles per item
    static constexpr int TOKCAP = 8;             // picks per pass (one n-tile)
    static constexpr int BROW = KS * 1024 + 64;  // smem bytes of one activation row (bank-spread)
    static_assert((KS - 1) * MT * 128 <= RED_FLOATS, "K-slice reduction buffer");
};

template <int KS>
__device__ __forceinline__ int64_t tiles(const GemvJob& j) {
    return (j.m.L.n + Cfg<KS>::R - 1) / Cfg<KS>::R;
}

// Item `it` of the launch: the shared jobs' (tile, pass) items first, then per used expert the
// tiles of every routed job (expert-major, so one expert's jobs reuse its activation rows in L2).
template <int KS>
__device__ __forceinline__ bool get_item(const GemvArgs& a, int64_t it, uint32_t n_used, Item* o) {
    using C = Cfg<KS>;
    int64_t routed_tiles = 0;
    const int64_t sp = (a.s_count + C::TOKCAP - 1) / C::TOKCAP;  // passes of a shared tile
    for (int j = 0; j < a.njobs; ++j) {
        const GemvJob& jb = a.job[j];
        if (jb.shared) {
            const int64_t t = tiles<KS>(jb) * sp;
            if (it < t) {
                o->job = j;
                o->e = 0;
                o->first = 0;
                o->count = (uint32_t)a.s_count;
                o->rt = it / sp;
                o->pass0 = (int)(it % sp);
                o->passes = 1;
                goto found;
            }
            it -= t;
        } else {
            routed_tiles += tiles<KS>(jb);
        }
    }
    if (routed_tiles == 0) return false;
    {
        const int64_t u = it / routed_tiles;
        if (u >= n_used) return false;
        int64_t r = it % routed_tiles;
        for (int j = 0; j < a.njobs; ++j) {
            const GemvJob& jb = a.job[j];
            if (jb.shared) continue;
            const int64_t t = tiles<KS>(jb);
            if (r < t) {
                o->job = j;
                o->rt = r;
                break;
            }
            r -= t;
        }
        o->e = a.used3[3 * u];
        o->first = a.used3[3 * u + 1];
        o->count = a.used3[3 * u + 2];
        o->pass0 = 0;
        o->passes = (int)((o->count + C::TOKCAP - 1) / C::TOKCAP);
        if (o->passes < 1) o->passes = 1;
    }
found:
    const Layout& L = a.job[o->job].m.L;
    const int64_t left = L.n - o->rt * C::R;
    o->rows = (int)(left < C::R ? left : C::R);
    o->n_kp = L.n_kp;
    o->nsk = (L.n_kp + KS - 1) / KS;
    return true;
}

struct Cursor {
    int64_t j;
    int pass, sk;
    Item item;
    bool valid;
};

template <int KS>
__device__ __forceinline__ void cursor_init(const GemvArgs& a, uint32_t n_used, Cursor* c) {
    c->j = 0;
    c->sk = 0;
    c->valid = get_item<KS>(a, blockIdx.x, n_used, &c->item);
    c->pass = c->valid ? c->item.pass0 : 0;
}
template <int KS>
__device__ __forceinline__ void cursor_next(const GemvArgs& a, uint32_t n_used, Cursor* c) {
    if (!c->valid) return;
    if (++c->sk < c->item.nsk) return;
    c->sk = 0;
    if (++c->pass < c->item.pass0 + c->item.passes) return;
    c->j++;
    c->valid = get_item<KS>(a, (int64_t)blockIdx.x + c->j * gridDim.x, n_used, &c->item);
    c->pass = c->valid ? c->item.pass0 : 0;
}

// What consumers need to know about a step, written by the producer at the head of its stage.
struct StepHdr {
    int job;  // -1: no more steps
    uint32_t e;
    int64_t rt;
    int rows, n_kp, kp0, pass_start, pass_end;
    uint32_t ntok;
    uint32_t orow[8];  // output row of each slot of the pass (pick index, or token)
};
constexpr int HDR_BYTES = 128;
static_assert(sizeof(StepHdr) <= HDR_BYTES, "step header");

// Stage layout of one step: [header][KS weight slots of R rows x piece bytes][TOKCAP activation rows].
template <int KS>
__host__ __device__ __forceinline__ int64_t slot_bytes(const Layout& L) {
    return pad16((int64_t)Cfg<KS>::R * L.kp_row_bytes);
}

// Issue step c into a stage (all lanes of the producer warp): the tile's rows of KS pieces, and
// the pass's activation rows for those columns.
template <int KS>
__device__ __forceinline__ void issue_step(const GemvArgs& a, const Cursor& c, uint8_t* stage, uint64_t* bar,
                                           int lane) {
    using C = Cfg<KS>;
    const Item& it = c.item;
    const GemvJob& jb = a.job[it.job];
    const Layout& L = jb.m.L;
    const int kp0 = c.sk * KS;
    const int nk = it.n_kp - kp0 < KS ? it.n_kp - kp0 : KS;
    uint32_t ntok = it.count - (uint32_t)c.pass * C::TOKCAP;
    if (ntok > (uint32_t)C::TOKCAP) ntok = C::TOKCAP;
    const int64_t row0 = it.rt * C::R, rowe = row0 + it.rows;
    uint32_t total = 0;
    for (int q = 0; q < nk; ++q) total += (uint32_t)(it.rows * piece_row_bytes(L, kp0 + q));
    const uint32_t bbytes = (uint32_t)nk * 1024;
    total += ntok * bbytes;
    if (lane == 0) mbar_expect_tx(bar, total);
    __syncwarp();
    int idx = 0;
    const uint8_t* ebase = jb.m.base + (int64_t)it.e * L.expert_bytes;
    for (int q = 0; q < nk; ++q) {
        const int kp = kp0 + q;
        const int64_t prb = piece_row_bytes(L, kp);
        uint8_t* dst = stage + q * slot_bytes<KS>(L);
        for (int64_t r = row0; r < rowe;) {
            const int64_t lt = r / TILE_ROWS, rr = r % TILE_ROWS;
            const int64_t rend = (lt + 1) * TILE_ROWS < rowe ? (lt + 1) * TILE_ROWS : rowe;
            if ((idx++ & 31) == lane)
                bulk_g2s(dst + (r - row0) * prb, ebase + piece_offset(L, lt, kp) + rr * prb,
                         (uint32_t)((rend - r) * prb), bar);
            r = rend;
        }
    }
    uint8_t* bdst = stage + KS * slot_bytes<KS>(L);
    for (uint32_t t = lane; t < ntok; t += 32) {
        const uint32_t ip = (uint32_t)c.pass * C::TOKCAP + t;
        const int64_t row = jb.shared ? (int64_t)ip : (int64_t)(a.pairs[it.first + ip] / (uint32_t)jb.bdiv);
        bulk_g2s(bdst + t * C::BROW, jb.b + row * jb.bstride + (int64_t)kp0 * 1024, bbytes, bar);
    }
}

// Header of step c (lanes of the producer warp; lane t < ntok fills output row t).
template <int KS>
__device__ __forceinline__ void write_hdr(const GemvArgs& a, const Cursor& c, StepHdr* h, int lane) {
    using C = Cfg<KS>;
    const Item& it = c.item;
    uint32_t ntok = it.count - (uint32_t)c.pass * C::TOKCAP;
    if (ntok > (uint32_t)C::TOKCAP) ntok = C::TOKCAP;
    if (lane == 0) {
        h->job = it.job;
        h->e = it.e;
        h->rt = it.rt;
        h->rows = it.rows;
        h->n_kp = it.n_kp;
        h->kp0 = c.sk * KS;
        h->pass_start = c.sk == 0;
        h->pass_end = c.sk == it.nsk - 1;
        h->ntok = ntok;
    }
    if ((uint32_t)lane < ntok) {
        const uint32_t ip = (uint32_t)c.pass * C::TOKCAP + lane;
        h->orow[lane] = a.job[it.job].shared ? ip : a.pairs[it.first + ip];
    }
}

template <int KS>
__global__ void __launch_bounds__(GEMV_THREADS + 32, 2) k_gemv(GemvArgs a) {
    using C = Cfg<KS>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);                 // 8 x 8 B
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + 64);           // 8 x 8 B
    uint4* h_g2 = reinterpret_cast<uint4*>(smem + 128);                 // 16 KB
    uint2* h_g3 = reinterpret_cast<uint2*>(smem + 128 + 16384);         // 4 KB
    uint4* h_sg = reinterpret_cast<uint4*>(smem + 128 + 20480);         // 4 KB
    float* red = reinterpret_cast<float*>(smem + 128 + HTABLES_BYTES);  // 2 x RED_FLOATS
    uint8_t* stages = smem + 128 + HTABLES_BYTES + RED_BYTES;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int NCW = GEMV_THREADS / 32;  // consumer warps
    if (tid == 0) {
        for (int s = 0; s < a.nst; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        fence_mbar_init();
    }
    load_htables(h_g2, h_g3, h_sg);
    __syncthreads();

    if (warp == NCW) {
        // ---------------- producer
        const uint32_t n_used = *a.n_used;
        Cursor pc;
        cursor_init<KS>(a, n_used, &pc);
        for (int64_t q = 0;; ++q) {
            const int s = (int)(q % a.nst);
            if (q >= a.nst && !mbar_wait(&empty[s], (uint32_t)(((q / a.nst) + 1) & 1), a.err)) return;
            uint8_t* stage = stages + (int64_t)s * a.stage_bytes;
            StepHdr* h = reinterpret_cast<StepHdr*>(stage);
            if (!pc.valid) {
                if (lane == 0) {
                    h->job = -1;
                    mbar_arrive(&full[s]);
                }
                return;
            }
            write_hdr<KS>(a, pc, h, lane);
            __syncwarp();
            issue_step<KS>(a, pc, stage + HDR_BYTES, &full[s], lane);
            cursor_next<KS>(a, n_used, &pc);
        }
    }

    // ---------------- consumers
    const HTables ht{h_g2, h_g3, h_sg};
    const int mt = warp % C::MT, ks = warp / C::MT;
    const int g = lane >> 2, c4 = lane & 3;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int red_parity = 0;
    for (int64_t q = 0;; ++q) {
        const int s = (int)(q % a.nst);
        if (!mbar_wait(&full[s], (uint32_t)((q / a.nst) & 1), a.err)) return;
        const uint8_t* stage = stages + (int64_t)s * a.stage_bytes;
        const StepHdr* h = reinterpret_cast<const StepHdr*>(stage);
        const int jobi = h->job;
        if (jobi < 0) return;
        const GemvJob& jb = a.job[jobi];
        const Layout& L = jb.m.L;
        const uint32_t ntok = h->ntok;
        if (h->pass_start) acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
        const uint8_t* st = stage + HDR_BYTES;
        const int kp = h->kp0 + ks;
        if (kp < h->n_kp && 16 * mt < h->rows) {
            const int64_t prb = piece_row_bytes(L, kp);
            const uint8_t* wsl = st + ks * slot_bytes<KS>(L);
            const int64_t kleft = L.k - (int64_t)kp * PIECE_K;
            const int klen = (int)(kleft < PIECE_K ? kleft : PIECE_K);
            const bool active = 64 * c4 < klen;  // this thread's 64 columns exist in the piece
            const int rA = 16 * mt + g, rB = rA + 8;
            // this thread's activation row (slot g of the pass), its chunk of this K-slice
            const uint8_t* brow = st + KS * slot_bytes<KS>(L) + g * C::BROW + ks * 1024 + 16 * c4;
            const bool has_tok = (uint32_t)g < ntok;
            const bool split = jb.split;
            const bool fast = !split && fmt_soa(L.fmt);
            IqRun qa, qb;
            if (fast && active) {
                qa = iq_run_load(L.fmt, iq_row_in(L.fmt, wsl, rA, prb), c4);
                qb = iq_run_load(L.fmt, iq_row_in(L.fmt, wsl, rB, prb), c4);
            }
#pragma unroll
            for (int ss = 0; ss < 4; ++ss) {
                uint32_t af[4][4], al[4][4];
                if (!active) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) af[kk][0] = af[kk][1] = af[kk][2] = af[kk][3] = 0u;
                } else if (fast) {
                    uint32_t p0[8], p1[8];
                    iq_run_pairs(L.fmt, qa, ss, p0, ht);
                    iq_run_pairs(L.fmt, qb, ss, p1, ht);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        af[kk][0] = p0[2 * kk];
                        af[kk][1] = p1[2 * kk];
                        af[kk][2] = p0[2 * kk + 1];
                        af[kk][3] = p1[2 * kk + 1];
                    }
                } else {
                    float v0[16], v1[16];
                    const int kofs = 64 * c4 + 16 * ss;
                    dec16_exact(L.fmt, wsl, rA, prb, kofs, v0, ht);
                    dec16_exact(L.fmt, wsl, rB, prb, kofs, v1, ht);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
                        for (int hh = 0; hh < 2; ++hh) {  // hh = 0: columns 4kk, 4kk+1; 1: 4kk+2, 4kk+3
                            const int i = 4 * kk + 2 * hh;
                            __half2 x0 = __floats2half2_rn(v0[i], v0[i + 1]);
                            __half2 x1 = __floats2half2_rn(v1[i], v1[i + 1]);
                            af[kk][2 * hh] = *reinterpret_cast<uint32_t*>(&x0);
                            af[kk][2 * hh + 1] = *reinterpret_cast<uint32_t*>(&x1);
                            if (split) {
                                const float2 f0 = __half22float2(x0), f1 = __half22float2(x1);
                                __half2 l0 = __floats2half2_rn(__fsub_rn(v0[i], f0.x), __fsub_rn(v0[i + 1], f0.y));
                                __half2 l1 = __floats2half2_rn(__fsub_rn(v1[i], f1.x), __fsub_rn(v1[i + 1], f1.y));
                                al[kk][2 * hh] = *reinterpret_cast<uint32_t*>(&l0);
                                al[kk][2 * hh + 1] = *reinterpret_cast<uint32_t*>(&l1);
                            }
                        }
                    }
                }
                // activation chunks (ss, q, h, c): hi cols 0-7, lo 0-7, hi 8-15, lo 8-15
                uint4 h0 = make_uint4(0, 0, 0, 0), h1 = h0, l0 = h0, l1 = h0;
                if (has_tok) {
                    h0 = *reinterpret_cast<const uint4*>(brow + 64 * (4 * ss + 0));
                    l0 = *reinterpret_cast<const uint4*>(brow + 64 * (4 * ss + 1));
                    h1 = *reinterpret_cast<const uint4*>(brow + 64 * (4 * ss + 2));
                    l1 = *reinterpret_cast<const uint4*>(brow + 64 * (4 * ss + 3));
                }
                const uint32_t hb[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
                const uint32_t lb[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    mma_16816(acc, af[kk], hb[2 * kk], hb[2 * kk + 1]);
                    mma_16816(acc, af[kk], lb[2 * kk], lb[2 * kk + 1]);
                    if (split) mma_16816(acc, al[kk], hb[2 * kk], hb[2 * kk + 1]);
                }
            }
        }
        // copy what the epilogue needs out of the stage, then hand the stage back
        const bool pass_end = h->pass_end;
        const uint32_t e = h->e;
        const int64_t rt = h->rt;
        const int rows = h->rows;
        uint32_t orow0 = 0, orow1 = 0;
        if (pass_end) {
            orow0 = h->orow[2 * c4];
            orow1 = h->orow[2 * c4 + 1];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (KS > 1 && pass_end) {
            // K-slices 1..KS-1 hand their partial sums to slice 0 (summed in slice order)
            float* rb0 = red + red_parity * RED_FLOATS;
            if (ks > 0) {
                float* rb = rb0 + ((ks - 1) * C::MT + mt) * 128;
#pragma unroll
                for (int i = 0; i < 4; ++i) rb[lane * 4 + i] = acc[i];
            }
            asm volatile("bar.sync 1, %0;" ::"n"(GEMV_THREADS) : "memory");
            if (ks == 0)
                for (int k2 = 1; k2 < KS; ++k2) {
                    const float* rb = rb0 + ((k2 - 1) * C::MT + mt) * 128;
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc[i] = __fadd_rn(acc[i], rb[lane * 4 + i]);
                }
            red_parity ^= 1;
        }
        if (pass_end && ks == 0 && 16 * mt < rows) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t slot = 2 * c4 + (i & 1);
                if (slot < ntok) {
                    const int64_t feat = rt * C::R + 16 * mt + g + ((i >> 1) ? 8 : 0);
                    const int64_t orow = (i & 1) ? orow1 : orow0;
                    float v = acc[i];
                    if (jb.bias) v = __fadd_rn(v, jb.bias[(int64_t)e * L.n + feat]);
                    jb.out[orow * jb.ostride + feat] = v;
                }
            }
        }
    }
}

// ---------------------------------------------------------------- host side
static constexpr int FIXED_SMEM = 128 + HTABLES_BYTES + RED_BYTES;  // barriers, tables, K-slice sums

template <int KS>
static int launch_ks(GemvArgs a, int64_t max_items, int device, int sm_count, cudaStream_t st) {
    using C = Cfg<KS>;
    int64_t wb = 0;
    for (int j = 0; j < a.njobs; ++j) {
        const int64_t b = KS * slot_bytes<KS>(a.job[j].m.L);
        if (b > wb) wb = b;
    }
    a.stage_bytes = (int)pad16(HDR_BYTES + wb + (int64_t)C::TOKCAP * C::BROW);
    // two CTAs per SM when the stages allow three or more steps in flight each
    int per_cta = (228 * 1024) / 2 - 1024 - FIXED_SMEM;
    int nst = per_cta / a.stage_bytes;
    int ctas_per_sm = 2;
    if (nst < 3) {
        per_cta = 227 * 1024 - 1024 - FIXED_SMEM;
        nst = per_cta / a.stage_bytes;
        ctas_per_sm = 1;
    }
    if (nst > 8) nst = 8;
    if (nst < 2) return fail(CWX_EUNSUPPORTED, "expert pieces too large for shared memory");
    a.nst = nst;
    const int smem = FIXED_SMEM + nst * a.stage_bytes;
    static int attr_set[64][4] = {{0}};
    const int kidx = KS == 1 ? 0 : KS == 2 ? 1 : KS == 4 ? 2 : 3;
    if (device < 0 || device >= 64 || attr_set[device][kidx] < smem) {
        cudaError_t e = cudaFuncSetAttribute(k_gemv<KS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(k_gemv)");
        if (device >= 0 && device < 64) attr_set[device][kidx] = smem;
    }
    int64_t grid = (int64_t)sm_count * ctas_per_sm;
    if (grid > max_items) grid = max_items;
    if (grid < 1) return CWX_OK;
    k_gemv<KS><<<(unsigned)grid, GEMV_THREADS + 32, smem, st>>>(a);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_gemv");
}

// K-slices per item: the largest split (up to the pieces per row) whose items still fill the GPU
// twice, chosen from the expected number of experts with picks.
static int choose_ks(const GemvArgs& a, int64_t experts_est, int sm_count) {
    int n_kp = 1 << 30;
    int64_t rows = 0;
    for (int j = 0; j < a.njobs; ++j)
        if (!a.job[j].shared) {
            if (a.job[j].m.L.n_kp < n_kp) n_kp = a.job[j].m.L.n_kp;
            rows += a.job[j].m.L.n;
        }
    if (rows == 0) return 1;
    int ks = 1;
    while (ks < 8 && ks * 2 <= n_kp) {
        const int64_t items = experts_est * ((rows + 128 / ks - 1) / (128 / ks));
        if (items >= 2 * sm_count) break;
        ks *= 2;
    }
    return ks;
}

int launch_gemv(const GemvArgs& a, int64_t experts_est, int device, int sm_count, cudaStream_t st) {
    const int ks = choose_ks(a, experts_est, sm_count);
    const int64_t R = 128 / ks;
    const int64_t sp = (a.s_count + 7) / 8;
    int64_t items = 0;
    for (int j = 0; j < a.njobs; ++j) {
        const int64_t t = (a.job[j].m.L.n + R - 1) / R;
        items += a.job[j].shared ? t * sp : t * experts_est;
    }
    switch (ks) {
        case 1: return launch_ks<1>(a, items, device, sm_count, st);
        case 2: return launch_ks<2>(a, items, device, sm_count, st);
        case 4: return launch_ks<4>(a, items, device, sm_count, st);
        default: return launch_ks<8>(a, items, device, sm_count, st);
    }
}

}  // namespace cwx
