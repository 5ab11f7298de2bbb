// Shared definitions of the cwx CUDA library: formats, the tiled bank layout, error state and
// the inline PTX used by the kernels (bulk copies, mbarriers, ldmatrix, mma).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cwx.h"

namespace cwx {

// ---------------------------------------------------------------- formats (GGUF type ids)
enum Fmt : int {
    F_Q8_0 = CWX_TYPE_Q8_0,
    F_Q4_K = CWX_TYPE_Q4_K,
    F_Q6_K = CWX_TYPE_Q6_K,
    F_IQ3_S = CWX_TYPE_IQ3_S,
    F_IQ2_S = CWX_TYPE_IQ2_S,
    F_MXFP4 = CWX_TYPE_MXFP4,
    F_IQ2_XXS = CWX_TYPE_IQ2_XXS,
    F_IQ3_XXS = CWX_TYPE_IQ3_XXS,
    F_IQ4_XS = CWX_TYPE_IQ4_XS,
};

__host__ __device__ inline int fmt_block_elems(int t) {
    switch (t) {
        case F_Q8_0: case F_MXFP4: return 32;
        case F_Q4_K: case F_Q6_K: case F_IQ2_S: case F_IQ3_S: case F_IQ2_XXS: case F_IQ3_XXS: case F_IQ4_XS:
            return 256;
        default: return 0;
    }
}
__host__ __device__ inline int fmt_block_bytes(int t) {
    switch (t) {
        case F_Q8_0: return 34;
        case F_MXFP4: return 17;
        case F_Q4_K: return 144;
        case F_Q6_K: return 210;
        case F_IQ2_S: return 82;
        case F_IQ3_S: return 110;
        case F_IQ2_XXS: return 66;
        case F_IQ3_XXS: return 98;
        case F_IQ4_XS: return 136;
        default: return 0;
    }
}

// Activation mode of a matrix product: which input the weights are multiplied with.
enum ActMode : int {
    AM_F32 = 0,   // f32 activations (Metal semantics; the only mode of the IQ formats)
    AM_Q8_K = 1,  // activations quantised to Q8_K per 256 (candle CPU VecDotType of K-quants)
    AM_Q8_0 = 2,  // activations quantised to Q8_0 per 32 (candle CPU VecDotType of Q8_0, MXFP4)
};
__host__ __device__ inline int act_mode_for(int fmt, int policy) {
    if (policy == CWX_ACT_MODE_F32) return AM_F32;
    switch (fmt) {
        case F_Q4_K: case F_Q6_K: return AM_Q8_K;
        case F_Q8_0: case F_MXFP4: return AM_Q8_0;
        default: return AM_F32;
    }
}

// ---------------------------------------------------------------- tiled bank layout
// A bank (E experts x n rows x k columns) is stored expert-major; inside an expert, 64-row tiles;
// inside a tile, K-pieces of up to 256 columns; inside a piece, the tile's rows one after the
// other, each row's quant blocks of that K range. A piece is one contiguous run of bytes padded
// to 16, so one bulk copy brings a (64 rows x 256 K) slab into shared memory. The quant blocks
// themselves are the GGUF bytes, unchanged.
constexpr int TILE_ROWS = 64;
constexpr int PIECE_K = 256;

__host__ __device__ inline int64_t pad16(int64_t x) { return (x + 15) & ~(int64_t)15; }

struct Layout {
    int fmt;
    int64_t n, k, n_experts;
    int64_t row_bytes;     // GGUF bytes of one row
    int n_kp;              // K-pieces per row
    int64_t kp_row_bytes;  // bytes of one row inside a full piece (256 K)
    int64_t last_kp_row_bytes;
    int64_t full_tile_bytes;
    int64_t expert_bytes;  // tiled bytes of one expert, padded to 256
};

__host__ __device__ inline int64_t piece_row_bytes(const Layout& L, int kp) {
    return kp == L.n_kp - 1 ? L.last_kp_row_bytes : L.kp_row_bytes;
}
__host__ __device__ inline int tile_rows(const Layout& L, int64_t rt) {
    int64_t r = L.n - rt * TILE_ROWS;
    return (int)(r < TILE_ROWS ? r : TILE_ROWS);
}
// Offset of piece (rt, kp) inside an expert, and its size.
__host__ __device__ inline int64_t piece_offset(const Layout& L, int64_t rt, int kp) {
    int rows = tile_rows(L, rt);
    int64_t off = rt * L.full_tile_bytes;
    int64_t full = pad16((int64_t)rows * L.kp_row_bytes);
    return off + (int64_t)kp * full;
}
__host__ __device__ inline int64_t piece_bytes(const Layout& L, int64_t rt, int kp) {
    return pad16((int64_t)tile_rows(L, rt) * piece_row_bytes(L, kp));
}

inline bool make_layout(int fmt, int64_t n, int64_t k, int64_t e, Layout* L) {
    int be = fmt_block_elems(fmt), bb = fmt_block_bytes(fmt);
    if (be == 0 || n <= 0 || k <= 0 || e <= 0 || k % be) return false;
    L->fmt = fmt;
    L->n = n;
    L->k = k;
    L->n_experts = e;
    L->row_bytes = k / be * bb;
    L->n_kp = (int)((k + PIECE_K - 1) / PIECE_K);
    L->kp_row_bytes = (int64_t)(PIECE_K < k ? PIECE_K : k) / be * bb;
    int64_t last_k = k - (int64_t)(L->n_kp - 1) * PIECE_K;
    L->last_kp_row_bytes = last_k / be * bb;
    L->full_tile_bytes = 0;
    for (int kp = 0; kp < L->n_kp; ++kp)
        L->full_tile_bytes += pad16((int64_t)TILE_ROWS * (kp == L->n_kp - 1 ? L->last_kp_row_bytes : L->kp_row_bytes));
    int64_t full_tiles = n / TILE_ROWS;
    int64_t eb = full_tiles * L->full_tile_bytes;
    if (n % TILE_ROWS) {
        int rows = (int)(n % TILE_ROWS);
        for (int kp = 0; kp < L->n_kp; ++kp)
            eb += pad16((int64_t)rows * (kp == L->n_kp - 1 ? L->last_kp_row_bytes : L->kp_row_bytes));
    }
    L->expert_bytes = (eb + 255) & ~(int64_t)255;
    return true;
}
// Note for partial tiles: every piece of a tile has the same padded size except the tail piece,
// so piece_offset() is exact for full pieces before the tail; tiles are laid out back to back.

// IQ2_S and IQ3_S pieces (one 256-column block per row) are stored as groups of 16 rows, each
// group field by field, so that what one thread of the grouped products reads (a row's fields
// for 64 consecutive columns, c4 = which 64) is one aligned vector. Same bytes, reordered; other
// formats keep whole rows.
//   IQ2_S group (16 x 82 = 1312 B): per (row, c4) a 16-byte record [qs 8 B | signs 8 B] at
//     (row*4 + c4)*16; per (row, c4) a 4-byte record [qh 2 B | scales 2 B] at 1024 + (row*4+c4)*4;
//     d at 1280 + row*2.
//   IQ3_S group (16 x 110 = 1760 B): qs at row*64, signs at 1024 + row*32, qh at 1536 + row*8,
//     scales at 1664 + row*4, d at 1728 + row*2.
//   IQ2_XXS group (16 x 66 = 1056 B): per (row, c4) a 16-byte record = GGUF bytes 2 + 16 c4 ..
//     (grid entries and signs/scale words of the two 32-column blocks) at (row*4 + c4)*16; d at
//     1024 + row*2.
//   IQ3_XXS group (16 x 98 = 1568 B): per (row, c4) the 16 grid-entry bytes (GGUF 2 + 16 c4 ..) at
//     (row*4 + c4)*16 and the two signs/scale words (GGUF 66 + 8 c4 ..) at 1024 + (row*4 + c4)*8;
//     d at 1536 + row*2.
//   IQ4_XS group (16 x 136 = 2176 B): per (row, c4) the 32 nibble bytes (GGUF 8 + 32 c4 ..) at
//     (row*4 + c4)*32; per row [d | scales_h | scales_l] (GGUF 0 .. 7) at 2048 + row*8.
//   MXFP4 group (16 x 136 = 2176 B; a piece row is 8 GGUF blocks of 17 bytes, e then 16 nibble
//     bytes): per (row, c4) the nibble bytes of blocks 2 c4 and 2 c4 + 1 at (row*4 + c4)*32; per
//     row the 8 scale bytes e at 2048 + row*8.
// GGUF blocks: IQ2_S = d(2) qs(32) signs(32) qh(8) scales(8); IQ3_S = d(2) qs(64) qh(8) signs(32)
// scales(4); IQ2_XXS = d(2) 8 x [entries(4) signs/scale(4)]; IQ3_XXS = d(2) entries(64)
// signs/scale(32); IQ4_XS = d(2) scales_h(2) scales_l(4) qs(128).
__host__ __device__ inline bool fmt_soa(int fmt) {
    return fmt == F_IQ2_S || fmt == F_IQ3_S || fmt == F_IQ2_XXS || fmt == F_IQ3_XXS || fmt == F_IQ4_XS ||
           fmt == F_MXFP4;
}

// Whether a piece whose rows are prb bytes is stored in 16-row groups: every piece of the IQ
// formats; the whole 256-column pieces of MXFP4 (a row's last piece of 2 to 7 blocks stays row
// after row).
__host__ __device__ inline bool soa_piece(int fmt, int64_t prb) {
    return fmt_soa(fmt) && (fmt != F_MXFP4 || prb == 8 * 17);
}

// Offset inside a 16-row group of byte b of the GGUF block of row rg (0..15).
__host__ __device__ inline int soa_offset(int fmt, int rg, int b) {
    if (fmt == F_IQ2_XXS) {
        if (b < 2) return 1024 + rg * 2 + b;
        const int j = b - 2;
        return (rg * 4 + (j >> 4)) * 16 + (j & 15);
    }
    if (fmt == F_IQ3_XXS) {
        if (b < 2) return 1536 + rg * 2 + b;
        if (b < 66) { const int j = b - 2; return (rg * 4 + (j >> 4)) * 16 + (j & 15); }
        const int j = b - 66;
        return 1024 + (rg * 4 + (j >> 3)) * 8 + (j & 7);
    }
    if (fmt == F_MXFP4) {
        const int blk = b / 17, o = b % 17;
        if (o == 0) return 2048 + rg * 8 + blk;
        return (rg * 4 + (blk >> 1)) * 32 + (blk & 1) * 16 + (o - 1);
    }
    if (fmt == F_IQ4_XS) {
        if (b < 8) return 2048 + rg * 8 + b;
        const int j = b - 8;
        return (rg * 4 + (j >> 5)) * 32 + (j & 31);
    }
    if (fmt == F_IQ2_S) {
        if (b < 2) return 1280 + rg * 2 + b;
        if (b < 34) { const int j = b - 2; return (rg * 4 + (j >> 3)) * 16 + (j & 7); }
        if (b < 66) { const int j = b - 34; return (rg * 4 + (j >> 3)) * 16 + 8 + (j & 7); }
        if (b < 74) { const int j = b - 66; return 1024 + (rg * 4 + (j >> 1)) * 4 + (j & 1); }
        const int j = b - 74;
        return 1024 + (rg * 4 + (j >> 1)) * 4 + 2 + (j & 1);
    }
    if (b < 2) return 1728 + rg * 2 + b;
    if (b < 66) return rg * 64 + (b - 2);
    if (b < 74) return 1536 + rg * 8 + (b - 66);
    if (b < 106) return 1024 + rg * 32 + (b - 74);
    return 1664 + rg * 4 + (b - 106);
}

// Byte b of row rr (row inside its 64-row tile rt) of piece kp -> offset inside the expert.
__host__ __device__ inline int64_t tiled_offset(const Layout& L, int64_t rt, int64_t rr, int kp, int64_t b) {
    const int64_t prb = piece_row_bytes(L, kp);
    const int64_t base = piece_offset(L, rt, kp);
    if (!soa_piece(L.fmt, prb)) return base + rr * prb + b;
    return base + (rr / 16) * 16 * prb + soa_offset(L.fmt, (int)(rr % 16), (int)b);
}

}  // namespace cwx

struct cwx_bank {
    int device;
    cwx::Layout L;
    uint8_t* d;  // tiled bytes, E * expert_bytes
    int64_t bytes_per_expert_gguf;
    // MXFP4: some row's 256-column piece (or 2-block tail piece) has block scales more than 2^24
    // apart, beyond the f16 range of the grouped products' fast path (its launches take the exact
    // path)
    int mx_wide;
    // MXFP4: every block scale e lies in [104, 140], so every weight (code times 2^(e - 128)) is
    // exact in f16 and the tensor-core products can take the bank
    int mx_f16;
};

struct cwx_ctx {
    int device;
    int sm_count;
    uint8_t* ws;  // workspace
    size_t ws_bytes;
    int* d_err;   // device error word (first error code wins); d_err + 8: grid barrier words of the fused decode layer
    int* h_err;   // pinned mirror
    uint16_t* d_iq3s_map;  // encoder maps for synthetic banks (built on first use)
    uint16_t* d_iq2s_map;
    uint16_t* d_iq3xxs_map;
    uint16_t* d_iq2xxs_map;
    int profiling;     // record per-phase events (cwx_ctx_set_profiling)
    void* prof;        // recorded (phase, start, end) events
    int64_t launches;  // kernel launches issued through this context
    int mma_min_pile;  // average picks per expert from which IQ layers take the tensor-core products (0: never)
    int fused_max_tokens;  // batches up to this size take the fused decode layer when it applies (0: never)
    cudaStream_t side;  // forked work inside a layer (created on first use)
    cudaEvent_t ev_fork, ev_join;
};

namespace cwx {

// ---------------------------------------------------------------- error reporting
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
// Grows the context workspace to at least `bytes` (refused while `st` is capturing a graph).
int ensure_ws(cwx_ctx* ctx, size_t bytes, cudaStream_t st);

#define CWX_CUDA(call)                                 \
    do {                                               \
        cudaError_t _e = (call);                       \
        if (_e != cudaSuccess) return cuda_fail(_e, #call); \
    } while (0)

// Device error codes written to cwx_ctx::d_err.
enum DevErr : int { DE_OK = 0, DE_TIMEOUT = 1, DE_BAD_ID = 2, DE_SHAPE = 3 };

__device__ inline void dev_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// ---------------------------------------------------------------- programmatic dependent launch
// The layer's kernels run back to back on one stream; each is launched with programmatic stream
// serialisation (launch_pdl), so its launch is processed, and its blocks scheduled as the blocks
// of the kernel before exit, without the gap of a full grid-to-grid dependency. Every such kernel
// calls pdl_wait() before it reads anything an earlier kernel wrote or writes anything an earlier
// kernel reads (the wait returns once the preceding grid has completed and its writes are
// visible; in a kernel launched without the attribute it returns at once). Work before the wait
// touches only shared memory, kernel parameters and tables that no kernel writes. No kernel
// signals its dependents early (griddepcontrol.launch_dependents): dependents parked on the SMs
// beside a running grid measured 9 % slower prefill layers and no faster decode.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------- PTX helpers
__device__ inline uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ inline void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ inline void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ inline void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait on an mbarrier phase. Returns false (and records DE_TIMEOUT) when the phase has
// not completed within `limit_ns` of wall-clock time (try_wait may suspend the thread, so the
// bound is on time, not on polls): a lost copy ends the kernel instead of hanging the GPU.
__device__ inline bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, uint64_t limit_ns = 2000000000ull) {
    const uint32_t a = smem_u32(bar);
    {  // already complete: a plain test costs a fraction of a suspending try_wait
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        // the suspend-time hint lets a waiting warp sleep until the phase completes (or 20 us
        // pass) instead of spinning on issue slots that the working warps of its SM need
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(parity), "r"(20000u)
            : "memory");
        if (done) return true;
        if (i == 0) t0 = globaltimer_ns();
        else if ((i & 63) == 0 && globaltimer_ns() - t0 > limit_ns) break;
    }
    dev_error(err, DE_TIMEOUT);
    return false;
}

__device__ inline void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 1-D bulk copy global -> shared, completion signalled on `bar` (bytes and addresses 16-aligned).
__device__ inline void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ inline void ldmatrix_x4(uint32_t* r, const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

// D += A (16x16 f16, row) * B (16x8 f16, col), f32 accumulate.
__device__ inline void mma_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ inline uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// f32 -> (hi, lo) f16 pair with hi + lo = x to about 2^-22 relative.
__device__ inline void split_f16(float x, __half* hi, __half* lo) {
    __half h = __float2half_rn(x);
    *hi = h;
    *lo = __float2half_rn(__fsub_rn(x, __half2float(h)));
}

}  // namespace cwx
