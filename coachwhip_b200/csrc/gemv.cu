// Grouped expert products (decode-sized piles): the B200 form of MoeMatvec.
//
//   reference  MoeMatvec (crates/engine/src/experts.rs:2183-2309) -> kernel_mul_mv_id_* and
//              kernel_mul_mm_idg_* (crates/engine/src/mv_id.rs:17-384,
//              vendor/candle-metal-kernels/src/metal_src/quantized.metal:7668-7766, 7868-7911).
//
// A launch runs up to four matrix jobs (routed gate, routed up, shared gate, shared up; or routed
// down, shared down). Work items are (job, expert, row tile) over the experts that have picks
// (the used list the pile kernels build) and (job, row tile, pass) for the shared expert, walked
// by a persistent grid of one CTA per SM: 16 consumer warps and one producer warp. Consumer warp
// w owns the 16 rows 16*(w % MT) of the tile and K-slice w / MT (KS slices, MT = 16 / KS, so small
// batches split K across warps and still fill the GPU). The producer resolves the CTA's items 32
// at a time (one per lane, so their loads of the used list and the piles overlap) into a small
// ring in shared memory, then runs ahead through the steps without touching global memory: for
// each it writes a small header (item, pass, the pass's output rows) into a free stage and
// brings, in one mbarrier phase, the tile's quantised bytes for KS pieces of 256 columns
// (cp.async.bulk from the tiled bank layout) and the pass's packed activation rows for those
// columns. Producer and consumers meet only on full/empty mbarriers whose waits are bounded.
//
// Each thread takes two rows x 64 contiguous columns of a piece into mma.sync m16n8k16 A
// registers, 16 columns per sub-step; the reduction index of an MMA step is permuted (thread c of
// a quad contributes 4 of its own columns), legal because A and B use the same permutation, and
// the activation rows arrive packed in exactly that order (act.cu).
//
// IQ2_S / IQ3_S / IQ2_XXS / IQ3_XXS fast path (the routed format of the launch): the codebooks
// live in shared memory replicated (8 copies of an 8-value table, 16 of a 4-value one) and
// interleaved so that the lanes sharing a shared-memory wavefront read different banks whatever
// entries they ask for. The weights go to the tensor cores as exact f16 integers, codebook value x
// sign x (2 * scale + 1) (at most 62 x 31); the block scale d (and the 1/8 of IQ2_S and IQ2_XXS,
// the 1/4 of IQ3_XXS) multiplies the f32 partial sum of each 256-column piece, so no weight is
// rounded. IQ4_XS (no codebook): nibble pairs map through a table to level pairs, times
// (ls - 32) of the 32-column block; exact while the product stays within 2048 (beyond, 11 bits).
// Activations: f16 (hi), plus the lo part when the job asks for ~22-bit products (its outputs are
// re-quantised downstream).
// Other formats (and any job of another format in the same launch): exact f32 dequantisation
// rounded to f16 (hi + lo pairs when the job asks for it), activations hi + lo.
#include <cstddef>

#include "cwx_common.cuh"
#include "decode.cuh"
#include "kernels.cuh"
#include "products.cuh"

namespace cwx {

constexpr int NCW = 16;                            // consumer warps
constexpr int NPW = 4;                             // producer warps (one per SM sub-partition)
constexpr int GEMV_THREADS = (NCW + NPW) * 32;
constexpr int RED_FLOATS = 14 * 128;         // (KS - 1) * MT fragments of 128 floats, KS * MT = 16, KS <= 8
constexpr int BAR_BYTES = 256;
constexpr int HDR_BYTES = 256;
constexpr int MAX_TOKCAP = 32;  // picks per pass: 8 per n-tile of the MMA, up to 4 n-tiles
constexpr int RING_TOK = 8;      // first-pass rows kept in the producer ring (passes of up to 8 picks)
constexpr int SMEM_LIMIT = 227 * 1024;
constexpr int RING_BYTES = 4096;  // the producer's look-ahead ring (PRing)
// Register split: the kernel launches with 96 registers per thread (640 threads fill the 64 K
// register file of an SM); the producer warpgroup then drops to PROD_REGS and the four consumer
// warpgroups rise to CONS_REGS, the decode's lookups and MMAs need more than 96 to overlap.
// 4 warps x 32 x PROD_REGS + 16 warps x 32 x CONS_REGS = 640 x 96 exactly.
constexpr int LAUNCH_REGS = 96, PROD_REGS = 64, CONS_REGS = 104;
static_assert(NPW * PROD_REGS + NCW * CONS_REGS <= (NCW + NPW) * LAUNCH_REGS, "register split");

template <int KS>
struct Cfg {
    static constexpr int MT = NCW / KS;            // m-tiles (16 rows) per item
    static constexpr int R = 16 * MT;              // rows of a routed item
    static_assert((KS - 1) * MT * 128 <= RED_FLOATS, "K-slice reduction buffer");
};

struct Item {
    int job;
    uint32_t e, first, count;
    int64_t rt;  // row tile index (in units of the job's rows per item)
    int rows;    // rows of this tile (multiple of 16)
    int n_kp;    // 256-column pieces per row
    int nsk;     // steps per pass (ceil(n_kp / KS))
    int pass0;   // first pass of this item
    int passes;  // passes this item runs
};

__device__ __forceinline__ int64_t job_tiles(const GemvJob& j) { return (j.m.L.n + j.rows - 1) / j.rows; }

// Item `it` of the launch: the shared jobs' (tile, pass) items first, then per used expert the
// tiles of every routed job (expert-major, so one expert's jobs reuse its activation rows in L2).
template <int KS>
__device__ __forceinline__ bool get_item(const GemvArgs& a, uint32_t it, uint32_t n_used, Item* o) {
    uint32_t routed_tiles = 0;
    const uint32_t sp = ((uint32_t)a.s_count + a.tokcap - 1) / (uint32_t)a.tokcap;  // passes of a shared tile
    for (int j = 0; j < a.njobs; ++j) {
        const GemvJob& jb = a.job[j];
        if (jb.shared) {
            const uint32_t t = (uint32_t)job_tiles(jb) * sp;
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
            routed_tiles += (uint32_t)job_tiles(jb);
        }
    }
    if (routed_tiles == 0) return false;
    {
        const uint32_t u = it / routed_tiles;
        if (u >= n_used) return false;
        uint32_t r = it - u * routed_tiles;
        for (int j = 0; j < a.njobs; ++j) {
            const GemvJob& jb = a.job[j];
            if (jb.shared) continue;
            const uint32_t t = (uint32_t)job_tiles(jb);
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
        o->passes = (int)((o->count + a.tokcap - 1) / (uint32_t)a.tokcap);
        if (o->passes < 1) o->passes = 1;
    }
found:
    const GemvJob& jb = a.job[o->job];
    const int64_t left = jb.m.L.n - o->rt * jb.rows;
    o->rows = (int)(left < jb.rows ? left : jb.rows);
    o->n_kp = jb.m.L.n_kp;
    o->nsk = (jb.m.L.n_kp + KS - 1) / KS;
    return true;
}

// What consumers need to know about a step, written by the producer at the head of its stage.
// Everything the consumers of a fast-path step need is in it, so they read it with a few 16-byte
// loads instead of indexing the launch's job table.
struct __align__(16) StepHdr {
    int job;    // -1: no more steps
    int flags;  // HF_* below, and the job's format in bits 8..15
    int kp0, n_kp;
    int rows, ntok;
    int feat0;  // first output feature of the tile
    int n;      // the job's rows (bias stride)
    float* out;
    int ostride;
    uint32_t e;
    const float* bias;
    int pad[2];
    uint32_t orow[MAX_TOKCAP];  // output row of each slot of the pass (pick index, or token)
};
static_assert(sizeof(StepHdr) <= HDR_BYTES, "step header");
static_assert(offsetof(StepHdr, rows) == 16 && offsetof(StepHdr, out) == 32 && offsetof(StepHdr, ostride) == 40 &&
                  offsetof(StepHdr, e) == 44 && offsetof(StepHdr, bias) == 48 && offsetof(StepHdr, orow) == 64,
              "step header words as the consumers read them");
constexpr int HF_PASS_START = 1, HF_PASS_END = 2, HF_SPLIT = 4, HF_QINT = 8;

__device__ __forceinline__ uint32_t pass_tokens(const Item& it, int pass, int tokcap) {
    const uint32_t done = (uint32_t)pass * (uint32_t)tokcap;
    const uint32_t left = it.count - done;
    return left < (uint32_t)tokcap ? left : (uint32_t)tokcap;
}

// Slot t of a pass: its activation row and its output row (pick index, or token).
__device__ __forceinline__ void pass_rows(const GemvArgs& a, const Item& it, int pass, uint32_t t, uint32_t* arow,
                                          uint32_t* orow) {
    const GemvJob& jb = a.job[it.job];
    const uint32_t ip = (uint32_t)pass * (uint32_t)a.tokcap + t;
    if (jb.shared) {
        *arow = ip;
        *orow = ip;
    } else {
        const uint32_t p = a.pairs[it.first + ip];
        *arow = jb.rowmap ? jb.rowmap[p] : p / (uint32_t)jb.bdiv;
        *orow = p;
    }
}

// A producer warp's look-ahead: the CTA's items resolved 8 at a time (lane L resolves one, so
// their global loads overlap), with the token rows of each item's first pass. Steps then need
// no global load.
constexpr int PBATCH = 8;
struct PRing {
    Item it[PBATCH];
    uint32_t arow[PBATCH][RING_TOK];
    uint32_t orow[PBATCH][RING_TOK];
};
static_assert(NPW * sizeof(PRing) <= RING_BYTES, "producer rings");

// The copies of the current item, one per lane: lane l < KS * nseg brings the 64-row-tile segment
// l % nseg of the item's rows for piece sk * KS + l / nseg of every step, so a step is an address
// add and one bulk copy per lane. Full pieces of a tile are pstride bytes apart; a shorter last
// piece (k not a multiple of 256) is addressed on its own.
struct CopyPlan {
    const uint8_t* src;  // the segment in piece 0
    int64_t pstride;     // bytes from one full piece of the segment's tile to the next
    const uint8_t* tile; // the segment's tile
    int32_t rel;         // the segment's first row inside its tile
    int32_t drow;        // its first row inside the item
    int32_t nrows;       // its rows
    int32_t cq;          // piece of the step (0..KS-1), -1: lane idle
};

template <int KS>
__device__ __forceinline__ CopyPlan plan_copies(const GemvArgs& a, const Item& it, int lane) {
    const GemvJob& jb = a.job[it.job];
    const Layout& L = jb.m.L;
    const int64_t row0 = it.rt * jb.rows, rowe = row0 + it.rows;
    const int64_t lt0 = row0 / TILE_ROWS, nseg = (rowe - 1) / TILE_ROWS - lt0 + 1;
    CopyPlan c;
    c.cq = -1;
    if (lane < KS * nseg) {
        const int64_t lt = lt0 + lane % nseg;
        const int64_t ra = lt * TILE_ROWS > row0 ? lt * TILE_ROWS : row0;
        const int64_t rb = (lt + 1) * TILE_ROWS < rowe ? (lt + 1) * TILE_ROWS : rowe;
        c.cq = lane / (int)nseg;
        c.tile = jb.m.base + (int64_t)it.e * L.expert_bytes + lt * L.full_tile_bytes;
        c.rel = (int32_t)(ra - lt * TILE_ROWS);
        c.drow = (int32_t)(ra - row0);
        c.nrows = (int32_t)(rb - ra);
        c.pstride = pad16((int64_t)tile_rows(L, lt) * L.kp_row_bytes);
        c.src = c.tile + c.rel * L.kp_row_bytes;
    }
    return c;
}

// Step sk of the current item, in two parts: the item's rows of KS pieces into a weight slot
// (completing on wbar), issued as soon as that slot's previous weights have been taken; and the
// pass's activation rows for those columns into an activation slot (completing on bbar; lane
// t < ntok holds the row of slot t), issued once that slot's previous step has finished.
template <int KS>
__device__ __forceinline__ void issue_weights(const GemvArgs& a, const Item& it, const CopyPlan& c, int64_t prb,
                                              int64_t lprb, int sk, uint8_t* wslot, uint64_t* wbar, int lane) {
    const int kp0 = sk * KS;
    const int nk = it.n_kp - kp0 < KS ? it.n_kp - kp0 : KS;
    const bool last_short = kp0 + nk == it.n_kp && lprb != prb;
    const uint32_t wbytes = (uint32_t)(it.rows * (prb * (nk - (last_short ? 1 : 0)) + (last_short ? lprb : 0)));
    if (lane == 0) mbar_expect_tx(wbar, wbytes);
    __syncwarp();
    if (c.cq >= 0 && c.cq < nk) {
        const int kp = kp0 + c.cq;
        uint8_t* dst = wslot + c.cq * a.slot_bytes;
        if (kp == it.n_kp - 1 && lprb != prb)
            bulk_g2s(dst + c.drow * lprb, c.tile + kp * c.pstride + c.rel * lprb, (uint32_t)(c.nrows * lprb), wbar);
        else
            bulk_g2s(dst + c.drow * prb, c.src + kp * c.pstride, (uint32_t)(c.nrows * prb), wbar);
    }
}

template <int KS>
__device__ __forceinline__ void issue_acts(const GemvArgs& a, const Item& it, int sk, uint32_t ntok, const uint8_t* brow,
                                           uint8_t* bslot, uint64_t* bbar, int lane) {
    const int kp0 = sk * KS;
    const int nk = it.n_kp - kp0 < KS ? it.n_kp - kp0 : KS;
    // the hi halves and a Q8_K piece's scale (KS == 1) when no job of the launch reads the lo parts
    const uint32_t bytes = a.bhi ? 528u : (uint32_t)nk * 1024;
    if (lane == 0) mbar_expect_tx(bbar, ntok * bytes);
    __syncwarp();
    if ((uint32_t)lane < ntok)
        bulk_g2s(bslot + HDR_BYTES + lane * a.brow, brow + (int64_t)kp0 * 1024, bytes, bbar);
}

// One step of any format: exact f32 dequantisation rounded to f16 (hi + lo weights when split),
// activations hi + lo, or Q8_K codes (qi) whose piece sums are scaled by the rows' d.
template <int NT>
__device__ __forceinline__ void generic_step(const Layout& L, int kp, const uint8_t* wsl, int mt, int g, int c4,
                                             const uint8_t* brow, int bnt, bool split, bool qi, const DxAt& dx,
                                             float* acc) {
    float t[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) t[nt][0] = t[nt][1] = t[nt][2] = t[nt][3] = 0.f;
    const int64_t prb = piece_row_bytes(L, kp);
    const int64_t kleft = L.k - (int64_t)kp * PIECE_K;
    const int klen = (int)(kleft < PIECE_K ? kleft : PIECE_K);
    const bool active = 64 * c4 < klen;  // this thread's 64 columns exist in the piece
    const int rA = 16 * mt + g, rB = rA + 8;
    const HTables none{nullptr, nullptr, nullptr};
#pragma unroll 1
    for (int ss = 0; ss < 4; ++ss) {
        uint32_t af[4][4], al[4][4];
        if (!active) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                af[kk][0] = af[kk][1] = af[kk][2] = af[kk][3] = 0u;
                al[kk][0] = al[kk][1] = al[kk][2] = al[kk][3] = 0u;
            }
        } else {
            float v0[16], v1[16];
            const int kofs = 64 * c4 + 16 * ss;
            dec16_exact<false>(L.fmt, wsl, rA, prb, kofs, v0, none);
            dec16_exact<false>(L.fmt, wsl, rB, prb, kofs, v1, none);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {  // hh = 0: columns 4kk, 4kk+1; 1: 4kk+2, 4kk+3
                    const int i = 4 * kk + 2 * hh;
                    const __half2 x0 = __floats2half2_rn(v0[i], v0[i + 1]);
                    const __half2 x1 = __floats2half2_rn(v1[i], v1[i + 1]);
                    af[kk][2 * hh] = h22u(x0);
                    af[kk][2 * hh + 1] = h22u(x1);
                    const float2 f0 = __half22float2(x0), f1 = __half22float2(x1);
                    al[kk][2 * hh] = h22u(__floats2half2_rn(__fsub_rn(v0[i], f0.x), __fsub_rn(v0[i + 1], f0.y)));
                    al[kk][2 * hh + 1] = h22u(__floats2half2_rn(__fsub_rn(v1[i], f1.x), __fsub_rn(v1[i + 1], f1.y)));
                }
            }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            uint32_t hb[8], lb[8];
            load_b(brow + nt * bnt, ss, !qi, hb, lb);
            float* d = qi ? t[nt] : acc + nt * 4;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                mma_16816(d, af[kk], hb[2 * kk], hb[2 * kk + 1]);
                if (!qi) mma_16816(d, af[kk], lb[2 * kk], lb[2 * kk + 1]);
                if (split) mma_16816(d, al[kk], hb[2 * kk], hb[2 * kk + 1]);
            }
        }
    }
    if (qi)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[nt * 4 + i] = __fmaf_rn(t[nt][i], dx_of(dx, nt, bnt, i), acc[nt * 4 + i]);
}

template <int FMT, int KS, int NT>
__global__ void __launch_bounds__(GEMV_THREADS, 1) k_gemv(GemvArgs a) {
    using C = Cfg<KS>;
    static_assert(KS == 1 || NT == 1, "n-tiles per pass only without K-slices");
    extern __shared__ __align__(128) uint8_t smem[];
    // two rings: weight slots (released as soon as the warps hold their bytes in registers, on
    // the fast path) and activation slots with the step header (released after the math)
    uint64_t* full_w = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty_w = full_w + 8;
    uint64_t* full_b = full_w + 16;
    uint64_t* empty_b = full_w + 24;
    uint8_t* tbl = smem + BAR_BYTES;
    float* red = reinterpret_cast<float*>(smem + BAR_BYTES + Tbl<FMT>::BYTES);
    uint8_t* wslots = smem + BAR_BYTES + Tbl<FMT>::BYTES + RED_FLOATS * 4 + RING_BYTES;
    uint8_t* bslots = wslots + a.nst * a.wslot_bytes;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < a.nst; ++s) {
            mbar_init(&full_w[s], 1);
            mbar_init(&empty_w[s], NCW);
            mbar_init(&full_b[s], 1);
            mbar_init(&empty_b[s], NCW);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp >= NCW) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(PROD_REGS));
        // ---------------- producers: all four walk the same sequence of steps; producer warp pw
        // fills the slots s with s % NPW == pw, so every slot has one writer, which has issued the
        // slot's previous step itself (its empty barriers are never more than a phase behind), and
        // each producer has several step-times to issue one step
        const int pw = warp - NCW;
        PRing* ring = reinterpret_cast<PRing*>(smem + BAR_BYTES + Tbl<FMT>::BYTES + RED_FLOATS * 4) + pw;
        pdl_wait();  // the piles and activation rows of the kernels before
        const uint32_t n_used = *a.n_used;
        int s = 0;        // slot of step q (q mod nst in both rings)
        uint32_t ph = 0;  // parity of the current round of the rings
        int64_t q = 0;
        for (int64_t base = 0;; base += PBATCH) {
            Item mine;
            const bool ok = lane < PBATCH &&
                            get_item<KS>(a, (uint32_t)(blockIdx.x + (base + lane) * gridDim.x), n_used, &mine);
            if (ok) {
                ring->it[lane] = mine;
                if (a.tokcap <= RING_TOK) {
                    const uint32_t n0 = pass_tokens(mine, mine.pass0, a.tokcap);
                    for (uint32_t t = 0; t < n0; ++t)
                        pass_rows(a, mine, mine.pass0, t, &ring->arow[lane][t], &ring->orow[lane][t]);
                }
            }
            const uint32_t okm = __ballot_sync(0xffffffffu, ok);
            __syncwarp();
            const int nitems = __popc(okm);  // items are consecutive: the valid ones come first
            for (int li = 0; li < nitems; ++li) {
                const Item it = ring->it[li];
                const GemvJob& jb = a.job[it.job];
                const CopyPlan cp = plan_copies<KS>(a, it, lane);
                const int64_t prb = jb.m.L.kp_row_bytes, lprb = jb.m.L.last_kp_row_bytes;
                for (int pass = it.pass0; pass < it.pass0 + it.passes; ++pass) {
                    const uint32_t ntok = pass_tokens(it, pass, a.tokcap);
                    uint32_t arow = 0, orow = 0;
                    if ((uint32_t)lane < ntok) {
                        if (pass == it.pass0 && a.tokcap <= RING_TOK) {
                            arow = ring->arow[li][lane];
                            orow = ring->orow[li][lane];
                        } else {
                            pass_rows(a, it, pass, lane, &arow, &orow);
                        }
                    }
                    const uint8_t* brow = jb.b + (int64_t)arow * jb.bstride;
                    for (int sk = 0; sk < it.nsk; ++sk) {
                        if (s % NPW == pw) {
                            if (q >= a.nst && !mbar_wait(&empty_w[s], ph ^ 1u, a.err)) return;
                            issue_weights<KS>(a, it, cp, prb, lprb, sk, wslots + s * a.wslot_bytes, &full_w[s], lane);
                            if (q >= a.nst && !mbar_wait(&empty_b[s], ph ^ 1u, a.err)) return;
                            uint8_t* bslot = bslots + s * a.bslot_bytes;
                            StepHdr* h = reinterpret_cast<StepHdr*>(bslot);
                            if (lane == 0) {
                                const int flags = (sk == 0 ? HF_PASS_START : 0) | (sk == it.nsk - 1 ? HF_PASS_END : 0) |
                                                  (jb.split ? HF_SPLIT : 0) | (jb.qint ? HF_QINT : 0) |
                                                  (jb.m.L.fmt << 8);
                                uint4* hv = reinterpret_cast<uint4*>(h);
                                hv[0] = make_uint4((uint32_t)it.job, (uint32_t)flags, (uint32_t)(sk * KS), (uint32_t)it.n_kp);
                                hv[1] = make_uint4((uint32_t)it.rows, ntok, (uint32_t)(it.rt * jb.rows), (uint32_t)jb.m.L.n);
                                h->out = jb.out;
                                h->ostride = (int)jb.ostride;
                                h->e = it.e;
                                h->bias = jb.bias;
                            }
                            if ((uint32_t)lane < ntok) h->orow[lane] = orow;
                            __syncwarp();
                            issue_acts<KS>(a, it, sk, ntok, brow, bslot, &full_b[s], lane);
                        }
                        ++q;
                        if (++s == a.nst) {
                            s = 0;
                            ph ^= 1u;
                        }
                    }
                }
            }
            __syncwarp();  // the ring is refilled by the next batch
            if (okm != (1u << PBATCH) - 1u) break;
        }
        if (s % NPW == pw) {  // the end marker, after the last step
            if (q >= a.nst && !mbar_wait(&empty_b[s], ph ^ 1u, a.err)) return;
            if (lane == 0) {
                reinterpret_cast<StepHdr*>(bslots + s * a.bslot_bytes)->job = -1;
                mbar_arrive(&full_b[s]);
            }
        }
        return;
    }

    // ---------------- consumers
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(CONS_REGS));
    if (FMT != 0) {
        build_tables<FMT, NCW * 32>(tbl, tid);  // (static tables only: runs while the kernel before ends)
        asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
    }
    pdl_wait();  // before the first write of an output row an earlier kernel may still read
    const uint8_t* tl = tbl + tbl_lane(FMT, lane);
    const int mt = warp % C::MT, ks = warp / C::MT;
    const int g = lane >> 2, c4 = lane & 3;
    // this thread's activation row (slot g of n-tile 0; with one n-tile, passes of fewer than 8
    // slots read row 0 past their capacity), its chunk of this K-slice; n-tile nt is bnt further
    const int bnt = 8 * a.brow;
    const int brow_off = HDR_BYTES + (NT == 1 && g >= a.tokcap ? 0 : g) * a.brow + ks * 1024 + 16 * c4;
    // the rows of this thread's output columns 2 c4 and 2 c4 + 1 (Q8_K scales), row 0 past capacity
    const int dx0_off = HDR_BYTES + (2 * c4 < a.tokcap ? 2 * c4 : 0) * a.brow + ks * 1024 + 512;
    const int dx1_off = HDR_BYTES + (2 * c4 + 1 < a.tokcap ? 2 * c4 + 1 : 0) * a.brow + ks * 1024 + 512;
    float acc[4 * NT];
#pragma unroll
    for (int i = 0; i < 4 * NT; ++i) acc[i] = 0.f;
    int s = 0;
    uint32_t ph = 0;
    for (;;) {
        if (!mbar_wait(&full_b[s], ph, a.err)) return;
        const uint8_t* bslot = bslots + s * a.bslot_bytes;
        const StepHdr* h = reinterpret_cast<const StepHdr*>(bslot);
        const uint4 h0 = reinterpret_cast<const uint4*>(h)[0], h1 = reinterpret_cast<const uint4*>(h)[1];
        const int jobi = (int)h0.x;
        if (jobi < 0) return;
        const int flags = (int)h0.y, fmt = (flags >> 8) & 0xFF;
        const bool pass_start = flags & HF_PASS_START, pass_end = flags & HF_PASS_END, lo = flags & HF_SPLIT;
        const bool qi = flags & HF_QINT;
        const int kp = (int)h0.z + ks, n_kp = (int)h0.w;
        const int rows = (int)h1.x;
        const uint32_t ntok = h1.y;
        if (pass_start) {
#pragma unroll
            for (int i = 0; i < 4 * NT; ++i) acc[i] = 0.f;
        }
        const bool active = kp < n_kp && 16 * mt < rows;
        const uint8_t* wsl = wslots + s * a.wslot_bytes + ks * a.slot_bytes;
        const uint8_t* brow = bslot + brow_off;
        if (!mbar_wait(&full_w[s], ph, a.err)) return;
        if (FMT != 0 && FMT != F_MXFP4 && fmt == FMT && !lo && !qi) {
            FastIn in;
            if (active) fast_load<FMT>(wsl, mt, g, c4, in);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_w[s]);  // the weights go back before the math
            if (active) fast_compute<FMT, NT>(in, tl, brow, bnt, false, acc);
        } else {
            if (active) {
                const Layout& L = a.job[jobi].m.L;
                const DxAt dx{bslot + dx0_off, bslot + dx1_off};
                // (late release; IQ4_XS weights above 2048 are not exact in f16, so its products
                // that must carry ~22 bits take the exact path; MXFP4 weights are exact, and their
                // products always take the activations' lo parts too, as Q8_0-rounded activations
                // are not exact in f16; a row's last MXFP4 piece of fewer than 8 blocks is stored
                // row after row: one of 2 blocks (K = 64 mod 256, as 2880) has its own loader,
                // longer ones take the exact path)
                const bool mx_tail = FMT == F_MXFP4 && kp + 1 == L.n_kp && L.last_kp_row_bytes != L.kp_row_bytes;
                if (FMT != 0 && L.fmt == FMT && !qi && (FMT != F_IQ4_XS || !lo) &&
                    (!mx_tail || L.last_kp_row_bytes == 2 * 17)) {
                    FastIn in;
                    if (mx_tail) fast_load_mx_tail(wsl, L.last_kp_row_bytes, mt, g, c4, in);
                    else fast_load<FMT>(wsl, mt, g, c4, in);
                    fast_compute<FMT, NT>(in, tl, brow, bnt, lo || FMT == F_MXFP4, acc);
                }
                else if (L.fmt == F_Q4_K && L.kp_row_bytes == 144) q4k_step<NT>(wsl, mt, g, c4, brow, bnt, lo, qi, dx, acc);
                else generic_step<NT>(L, kp, wsl, mt, g, c4, brow, bnt, lo, qi, dx, acc);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_w[s]);
        }
        // what the pass's epilogue needs, taken out of the slot before the slot is handed back (after
        // the math, so these registers are not held through it)
        uint4 h2 = make_uint4(0, 0, 0, 0), h3 = h2;
        uint2 orw[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) orw[nt] = make_uint2(0, 0);
        if (pass_end) {
            h2 = reinterpret_cast<const uint4*>(h)[2];
            h3 = reinterpret_cast<const uint4*>(h)[3];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) orw[nt] = *reinterpret_cast<const uint2*>(&h->orow[8 * nt + 2 * c4]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_b[s]);
        if (++s == a.nst) {
            s = 0;
            ph ^= 1u;
        }
        if (KS > 1 && pass_end) {
            // K-slices 1..KS-1 hand their partial sums to slice 0 (summed in slice order)
            if (ks > 0) {
                float* rb = red + ((ks - 1) * C::MT + mt) * 128;
#pragma unroll
                for (int i = 0; i < 4; ++i) rb[lane * 4 + i] = acc[i];
            }
            asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
            if (ks == 0)
                for (int k2 = 1; k2 < KS; ++k2) {
                    const float* rb = red + ((k2 - 1) * C::MT + mt) * 128;
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc[i] = __fadd_rn(acc[i], rb[lane * 4 + i]);
                }
            asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
        }
        if (pass_end && ks == 0 && 16 * mt < rows) {
            // header words 2 and 3: out, ostride, e; bias
            float* out = reinterpret_cast<float*>(((uint64_t)h2.y << 32) | h2.x);
            const int64_t ostride = (int)h2.z;
            const uint32_t e = h2.w;
            const float* bias = reinterpret_cast<const float*>(((uint64_t)h3.y << 32) | h3.x);
            const int feat0 = (int)h1.z, n = (int)h1.w;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t slot = 8 * nt + 2 * c4 + (i & 1);
                    if (slot < ntok) {
                        const int64_t feat = feat0 + 16 * mt + g + ((i >> 1) ? 8 : 0);
                        const int64_t orow = (i & 1) ? orw[nt].y : orw[nt].x;
                        float v = acc[nt * 4 + i];
                        if (bias) v = __fadd_rn(v, bias[(int64_t)e * n + feat]);
                        out[orow * ostride + feat] = v;
                    }
                }
        }
    }
}

// ---------------------------------------------------------------- host side
static int tbl_bytes(int fmt) {
    switch (fmt) {
        case F_IQ2_S: return Tbl<F_IQ2_S>::BYTES;
        case F_IQ3_S: return Tbl<F_IQ3_S>::BYTES;
        case F_IQ2_XXS: return Tbl<F_IQ2_XXS>::BYTES;
        case F_IQ3_XXS: return Tbl<F_IQ3_XXS>::BYTES;
        case F_IQ4_XS: return Tbl<F_IQ4_XS>::BYTES;
        case F_MXFP4: return Tbl<F_MXFP4>::BYTES;
        default: return 0;
    }
}
// Routed formats with a fast path in k_gemv.
static bool fast_fmt(int fmt) {
    return fmt == F_IQ2_S || fmt == F_IQ3_S || fmt == F_IQ2_XXS || fmt == F_IQ3_XXS || fmt == F_IQ4_XS ||
           fmt == F_MXFP4;
}

// Stage sizes of a launch with routed format fmt (0: none), ks K-slices and a.tokcap picks per
// pass: the weight bytes of a K-slice (a routed tile of the fast format at full height, every job
// at full height when there is no fast format, and at least 16 rows of every other job; jobs of
// other formats get the rows that fit), the activation row stride (the hi halves only when one
// K-slice is copied and no job reads the lo parts), and how many stages fit in shared memory.
// Returns the stage count (below 2: the configuration does not fit).
static int size_stages(GemvArgs& a, int fmt, int ks, int64_t experts_est, int64_t* items, int* smem) {
    const int64_t R = 16 * (NCW / ks);
    int64_t slot = 0;
    bool hi_only = ks == 1;
    for (int j = 0; j < a.njobs; ++j) {
        const GemvJob& jb = a.job[j];
        const Layout& L = jb.m.L;
        const int64_t want = (fmt == 0 || L.fmt == fmt) ? R : 16;
        const int64_t b = pad16(want * L.kp_row_bytes);
        if (b > slot) slot = b;
        // which products read the activations' lo halves: the exact path of any format, and
        // split products, unless the rows hold Q8_K codes
        const bool fast = fmt != 0 && L.fmt == fmt, q4 = L.fmt == F_Q4_K && L.kp_row_bytes == 144;
        if (!jb.qint && (jb.split || !(fast || q4) || L.fmt == F_MXFP4)) hi_only = false;
    }
    a.slot_bytes = (int)slot;
    *items = 0;
    const int64_t sp = (a.s_count + a.tokcap - 1) / a.tokcap;
    for (int j = 0; j < a.njobs; ++j) {
        GemvJob& jb = a.job[j];
        int64_t rows = slot / jb.m.L.kp_row_bytes / 16 * 16;
        if (rows > R) rows = R;
        jb.rows = (int)rows;
        const int64_t t = (jb.m.L.n + rows - 1) / rows;
        *items += jb.shared ? t * sp : t * experts_est;
    }
    // rows of a slot 64 bytes past a multiple of 128, so the 8 rows one load instruction touches
    // fall in different banks
    a.bhi = hi_only ? 1 : 0;
    a.brow = (hi_only ? 512 : ks * 1024) + 64;
    a.wslot_bytes = (int)((ks * slot + 127) & ~(int64_t)127);
    a.bslot_bytes = (int)((HDR_BYTES + (int64_t)a.tokcap * a.brow + 127) & ~(int64_t)127);
    const int fixed = BAR_BYTES + tbl_bytes(fmt) + RED_FLOATS * 4 + RING_BYTES;
    int nst = (SMEM_LIMIT - fixed) / (a.wslot_bytes + a.bslot_bytes);
    if (nst > 8) nst = 8;
    a.nst = nst;
    *smem = fixed + nst * (a.wslot_bytes + a.bslot_bytes);
    return nst;
}

template <int FMT, int KS, int NT>
static int launch_fk(const GemvArgs& a, int64_t items, int smem, int device, int sm_count, cudaStream_t st) {
    constexpr int fi = FMT == 0           ? 0
                       : FMT == F_IQ2_S     ? 1
                       : FMT == F_IQ3_S     ? 2
                       : FMT == F_IQ2_XXS   ? 3
                       : FMT == F_IQ3_XXS   ? 4
                       : FMT == F_IQ4_XS    ? 5
                                            : 6;
    constexpr int ki = (KS == 1 ? 0 : KS == 2 ? 1 : KS == 4 ? 2 : 3) + (NT == 2 ? 4 : NT == 4 ? 5 : 0);
    // the register split assumes the launch allocates LAUNCH_REGS per thread (allocation is in
    // steps of 8): a kernel compiled with fewer would make the consumers' increase wait forever
    static int regs_ok[7][6] = {{0}};
    if (!regs_ok[fi][ki]) {
        cudaFuncAttributes fa;
        cudaError_t e = cudaFuncGetAttributes(&fa, k_gemv<FMT, KS, NT>);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes(k_gemv)");
        if ((fa.numRegs + 7) / 8 * 8 != LAUNCH_REGS)
            return fail(CWX_EUNSUPPORTED, "k_gemv compiled with %d registers, the register split needs %d",
                        fa.numRegs, LAUNCH_REGS);
        regs_ok[fi][ki] = 1;
    }
    static int attr_set[64][7][6] = {{{0}}};
    if (device < 0 || device >= 64 || attr_set[device][fi][ki] < smem) {
        cudaError_t e = cudaFuncSetAttribute(k_gemv<FMT, KS, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(k_gemv)");
        if (device >= 0 && device < 64) attr_set[device][fi][ki] = smem;
    }
    int64_t grid = sm_count;
    if (grid > items) grid = items;
    if (grid < 1) return CWX_OK;
    cudaError_t e = launch_pdl(k_gemv<FMT, KS, NT>, dim3((unsigned)grid), dim3(GEMV_THREADS), smem, st, a);
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_gemv");
}

template <int FMT>
static int launch_f(const GemvArgs& a, int ks, int nt, int64_t items, int smem, int device, int sm_count,
                    cudaStream_t st) {
    if (nt == 4) return launch_fk<FMT, 1, 4>(a, items, smem, device, sm_count, st);
    if (nt == 2) return launch_fk<FMT, 1, 2>(a, items, smem, device, sm_count, st);
    switch (ks) {
        case 1: return launch_fk<FMT, 1, 1>(a, items, smem, device, sm_count, st);
        case 2: return launch_fk<FMT, 2, 1>(a, items, smem, device, sm_count, st);
        case 4: return launch_fk<FMT, 4, 1>(a, items, smem, device, sm_count, st);
        default: return launch_fk<FMT, 8, 1>(a, items, smem, device, sm_count, st);
    }
}

static int launch_fmt(int fmt, const GemvArgs& a, int ks, int nt, int64_t items, int smem, int device, int sm_count,
                      cudaStream_t st) {
    switch (fmt) {
        case F_IQ2_S: return launch_f<F_IQ2_S>(a, ks, nt, items, smem, device, sm_count, st);
        case F_IQ3_S: return launch_f<F_IQ3_S>(a, ks, nt, items, smem, device, sm_count, st);
        case F_IQ2_XXS: return launch_f<F_IQ2_XXS>(a, ks, nt, items, smem, device, sm_count, st);
        case F_IQ3_XXS: return launch_f<F_IQ3_XXS>(a, ks, nt, items, smem, device, sm_count, st);
        case F_IQ4_XS: return launch_f<F_IQ4_XS>(a, ks, nt, items, smem, device, sm_count, st);
        case F_MXFP4: return launch_f<F_MXFP4>(a, ks, nt, items, smem, device, sm_count, st);
        default: return launch_f<0>(a, ks, nt, items, smem, device, sm_count, st);
    }
}

int launch_gemv(const GemvArgs& in, int64_t experts_est, int device, int sm_count, cudaStream_t st) {
    GemvArgs a = in;
    // the routed format, when every routed job shares one IQ format
    int fmt = -1, n_kp = 1 << 30;
    int64_t rows = 0;
    for (int j = 0; j < a.njobs; ++j) {
        const Layout& L = a.job[j].m.L;
        if (a.job[j].shared) continue;
        fmt = fmt == -1 ? L.fmt : (fmt == L.fmt ? fmt : 0);
        if (L.n_kp < n_kp) n_kp = L.n_kp;
        rows += L.n;
    }
    if (!fast_fmt(fmt)) fmt = 0;
    for (int j = 0; j < a.njobs; ++j)  // a bank only the exact path reads correctly
        if (a.job[j].m.L.fmt == fmt && a.job[j].exact) fmt = 0;
    int64_t items = 0;
    int smem = 0;
    // large piles (on average 24 or 10 picks and more): 32 or 16 picks per pass (4 or 2 n-tiles of
    // 8 per decoded weight fragment), one K-slice, when two stages of that fit
    for (int nt = 4; nt >= 2; nt /= 2)
        if (a.pile_est >= (nt == 4 ? 24 : 10) && a.tok_est > 8) {
            a.tokcap = 8 * nt;
            if (size_stages(a, fmt, 1, experts_est, &items, &smem) >= 2) {
                return launch_fmt(fmt, a, 1, nt, items, smem, device, sm_count, st);
            }
        }
    // otherwise passes of the expected largest pile, a power of two up to 8
    int tc = 1;
    while (tc < 8 && tc < a.tok_est) tc *= 2;
    a.tokcap = tc;
    // K-slices: the smallest split (up to the pieces per row, and 8 staged activation pieces per
    // stage) whose items still fill the GPU twice
    int ks = 1;
    if (rows > 0)
        while (ks < 8 && ks * 2 <= n_kp && ks * 2 * tc <= 8) {
            const int64_t r = 16 * (NCW / ks);
            const int64_t it = experts_est * ((rows + r - 1) / r);
            if (it >= 2 * sm_count) break;
            ks *= 2;
        }
    if (size_stages(a, fmt, ks, experts_est, &items, &smem) < 2)
        return fail(CWX_EUNSUPPORTED, "expert pieces too large for shared memory");
    return launch_fmt(fmt, a, ks, 1, items, smem, device, sm_count, st);
}

}  // namespace cwx
