// Grouped expert products for large piles (prefill) on the 5th-generation tensor cores.
//
//   reference  MoeMatvec on prefill-sized batches (crates/engine/src/experts.rs:2183-2309), which
//              ends in kernel_mul_mm_idg_* (crates/engine/src/mv_id.rs:220-384,
//              vendor/candle-metal-kernels/src/metal_src/quantized.metal:7868-7911): per expert, the
//              picks routed to it times the expert's dequantised matrix.
//
// One persistent CTA per SM walks work items (used expert, row tile of 128 outputs, column tile of
// up to 256 picks). Per item the CTA streams the tile's quantised pieces (256 columns) into shared
// memory with bulk copies, decodes them 64 columns at a time into f16 A tiles, gathers the picks'
// activation rows (f16) into B tiles with cp.async, and one thread issues tcgen05.mma
// (M = 128, N = the tile's picks rounded up to 16, K = 16 per instruction) into a TMEM
// accumulator. Two accumulators (TMEM columns 0-255 and 256-511) let the epilogue of one item run
// while the next one multiplies.
//
// Operand layout (both K-major, 128-byte swizzle): a tile row holds 64 f16 (128 bytes), rows are
// 128 bytes apart, 16-byte chunk c of row r sits at chunk position c ^ (r % 8), and 8-row groups
// are 1024 bytes apart (the smem descriptor's stride byte offset). The MMA for columns
// 16 kk .. 16 kk + 15 of a stage starts 32 kk bytes into the tile.
//
// Weights: IQ2_S / IQ3_S / IQ2_XXS / IQ3_XXS codebook values times sign times (2 s + 1), times 1/8
// (IQ2_S, IQ2_XXS) or 1/4 (IQ3_XXS), are exact in f16 (at most 11 significant bits); one f16
// multiply by the block scale d rounds each weight once, so the A tiles hold the exact dequantised
// weight rounded to f16. (Scaling d by 1/8 first would not be exact: typical d are near the f16
// subnormal range.) IQ4_XS: (d * (ls - 32)) * level in f32 rounded to f16 once, as the
// reference's Metal matrix kernels store it.
//
// Two forms of a launch:
//   fused gate/up: A rows 0-63 are gate rows f0 .. f0+63, rows 64-127 the up rows of the same
//     features; the epilogue writes h = silu(gate) * up as f16 rows (one per pick), the B operand
//     of the down products;
//   plain: A rows are 128 consecutive rows of one matrix; the epilogue writes f32 rows per pick.
//
// Roles (22 warps): 0-3 epilogue (TMEM lanes 32w .. 32w+31), 4 MMA issue and TMEM allocation,
// 5 quantised-piece copies, 6-9 activation gathers, 10-21 decode. Every wait is bounded; a role
// that gives up records DE_TIMEOUT and leaves its loop, and the CTA still meets at the final
// barrier, where the TMEM is freed.
#include "cwx_common.cuh"
#include "decode.cuh"
#include "kernels.cuh"

namespace cwx {

namespace mm {

constexpr int NS = 3;             // operand stages (64 columns each)
constexpr int NQ = 2;             // quantised-piece stages (256 columns each)
constexpr int NMAX = 256;         // picks per column tile
constexpr int A_BYTES = 128 * 128;
constexpr int B_BYTES = NMAX * 128;
constexpr int Q_BYTES = 128 * 144;  // 128 rows of the largest piece (Q4_K)
constexpr int XCH_BYTES = 32 * 64 * 4;
constexpr int THREADS = 22 * 32;
constexpr int W_MMA = 4, W_QCOPY = 5, W_GATHER = 6, N_GATHER = 4, W_DEC = 10, N_DEC = 12;
constexpr int DEC_CHUNKS = 128 * 8;                                   // 16-byte A chunks per stage
constexpr int DEC_PER = (DEC_CHUNKS + N_DEC * 32 - 1) / (N_DEC * 32);  // per decoder thread
constexpr int GATHER_PER = NMAX * 8 / (N_GATHER * 32);                 // B chunks per gather thread
constexpr int TMEM_COLS = 512;

// Codebook as f16 values: IQ2_S and IQ2_XXS 8 per entry, two copies (entry e of copy j at
// e*32 + j*16, the copy picked by the lane's parity, so fewer lanes of a wavefront meet on a bank);
// IQ3_S and IQ3_XXS 4 per entry, four copies (e*32 + j*8); the 16 IQ4_XS levels as f32, one copy
// per lane (level n of copy j at n*128 + j*4); MXFP4: nibble pair p -> the f16 pair of codes
// (twice the e2m1 values, the reference's kvalues_mxfp4), 16 copies (p*64 + j*4, j = lane % 16).
template <int FMT>
struct Tab {
    static constexpr int BYTES = FMT == F_IQ2_S ? 1024 * 32
                                 : FMT == F_IQ3_S ? 512 * 32
                                 : (FMT == F_IQ2_XXS || FMT == F_IQ3_XXS) ? 256 * 32
                                 : FMT == F_IQ4_XS ? 16 * 128
                                 : FMT == F_MXFP4  ? 256 * 64
                                                   : 0;
};

// Pipeline geometry: three operand stages of B tiles for NMAX picks; with hi + lo activations
// (LO) two stages, each B stage holding the hi and the lo tile of NMAX picks.
template <bool LO>
struct Geo {
    static constexpr int NSS = LO ? 2 : NS;                              // operand stages
    static constexpr int B_STAGE = (LO ? 2 : 1) * B_BYTES;              // bytes of a B stage
    static constexpr int GP = (LO ? 2 : 1) * NMAX * 8 / (N_GATHER * 32);  // B chunks per gather thread
};

// shared memory: barriers, then 1024-aligned A and B stages, quantised stages, codebook, exchange
template <int FMT, bool LO>
struct Smem {
    static constexpr int BAR = 0;
    static constexpr int A = 1024;
    static constexpr int B = A + Geo<LO>::NSS * A_BYTES;
    static constexpr int Q = B + Geo<LO>::NSS * Geo<LO>::B_STAGE;
    static constexpr int TAB = Q + NQ * Q_BYTES;
    static constexpr int XCH = TAB + Tab<FMT>::BYTES;
    static constexpr int TOTAL = XCH + XCH_BYTES;
    static_assert(TOTAL + 1024 <= 227 * 1024, "k_mma: shared memory above a CTA's 227 KB");
};

struct Bars {
    uint64_t full_q[NQ], empty_q[NQ];
    uint64_t full_a[NS], full_b[NS], empty_s[NS];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t mma_done;
    uint32_t tmem;
};
static_assert(sizeof(Bars) <= 1024, "barrier block");

// ---------------------------------------------------------------- tcgen05 / async-copy PTX
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
// One lane of the (converged) warp.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n .reg .b32 r;\n .reg .pred p;\n elect.sync r|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(pred));
    return pred != 0;
}
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, f16 inputs, f32 accumulate; acc = 0 overwrites D.
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
// The mbarrier completes once every tcgen05 operation this thread issued before it has finished.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 32 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// Arrives on bar once this thread's earlier cp.async copies have landed (counts toward the
// barrier's expected arrivals).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc(const void* p) {
    const uint32_t a = smem_u32(p);
    return (uint64_t)((a >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: f32 accumulator, f16 A and B, both K-major, M = 128, N.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// ---------------------------------------------------------------- work items
// Items in order: per used expert, per column tile of NMAX picks, per row tile.
struct Iter {
    uint32_t u = 0xFFFFFFFFu;  // current used expert (none loaded yet)
    uint32_t base = 0;         // items before expert u
    uint32_t n_items = 0;      // items of expert u
    uint32_t e = 0, first = 0, count = 0;
};
struct MItem {
    uint32_t e, first, n0, ntok;
    int mt;
};

// nmax: picks per column tile (NMAX, or NMAX / 2 when the B tiles carry hi and lo parts).
__device__ __forceinline__ bool next_item(const MmaArgs& a, Iter& st, uint32_t i, uint32_t n_used, MItem* o,
                                          uint32_t nmax) {
    while (st.u == 0xFFFFFFFFu || i >= st.base + st.n_items) {
        if (st.u != 0xFFFFFFFFu) st.base += st.n_items;
        st.u = st.u == 0xFFFFFFFFu ? 0 : st.u + 1;
        if (st.u >= n_used) return false;
        st.e = a.used3[3 * st.u];
        st.first = a.used3[3 * st.u + 1];
        st.count = a.used3[3 * st.u + 2];
        st.n_items = (st.count + nmax - 1) / nmax * (uint32_t)a.mtiles;
    }
    const uint32_t local = i - st.base;
    const uint32_t nt = local / (uint32_t)a.mtiles;
    o->mt = (int)(local % (uint32_t)a.mtiles);
    o->e = st.e;
    o->first = st.first;
    o->n0 = nt * nmax;
    const uint32_t left = st.count - o->n0;
    o->ntok = left < nmax ? left : nmax;
    return true;
}

// Source of A rows 0-63 (half 0) and 64-127 (half 1) of row tile mt, piece kp.
__device__ __forceinline__ const uint8_t* half_src(const MmaArgs& a, int half, uint32_t e, int mt, int kp) {
    const MatRef& m = half == 0 || !a.fused ? a.a0 : a.a1;
    const int64_t t = a.fused ? mt : 2 * mt + half;
    const Layout& L = m.L;
    return m.base + (int64_t)e * L.expert_bytes + t * L.full_tile_bytes + (int64_t)kp * pad16(64 * L.kp_row_bytes);
}

// ---------------------------------------------------------------- decode
// 8 consecutive weights (chunk gi of the 64-column slice c4) of row r of a staged piece, as f16
// (exact dequantised value rounded once), 16 bytes.
__device__ __forceinline__ uint32_t u_h2(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 h2_u(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ uint32_t sgn_pair(uint32_t s8, int q, uint32_t g) {
    const uint32_t m = s8 * ((1u << (15 - q)) + (1u << (30 - q)));
    return (m & 0x80008000u) ^ g;
}
// n in 0..15 -> (2n + 1) as an f16 pair, exact.
__device__ __forceinline__ __half2 odd_h2(uint32_t n) {
    return __hsub2(h2_u(n * 0x00020002u + 0x64016401u), __floats2half2_rn(1024.f, 1024.f));
}

// 2^(e - 128) as an f16 pair (e in [104, 140]: a normal or subnormal f16, exact).
__device__ __forceinline__ __half2 mx_scale_h2(uint32_t e) {
    const int s = (int)e - 128;
    const uint32_t bits = s >= -14 ? (uint32_t)(s + 15) << 10 : 1u << (s + 24);
    return h2_u(bits | (bits << 16));
}

// prb: bytes of a staged row of this piece (MXFP4's last piece of 2 to 7 blocks is row-major).
template <int FMT>
__device__ __forceinline__ uint4 dec_chunk(const uint8_t* q, int r, int c4, int gi, const uint8_t* tab, int prb) {
    if (FMT == F_MXFP4) {
        // chunk gi: block 2 c4 + gi / 4, its columns 8 (gi % 4) ..: the low (gi % 4 < 2) or high
        // nibbles of bytes 8 (gi % 2) .. + 7; y = code * 2^(e - 128) (the reference's
        // dequantize: kvalues_mxfp4 times e8m0_to_fp32_half), exact in f16 for the banks that
        // take this path (cwx_bank::mx_f16)
        uint2 b;
        uint32_t e;
        if (prb == 136) {
            const uint8_t* grp = q + (r >> 4) * (16 * 136);
            const int rg = r & 15;
            b = *reinterpret_cast<const uint2*>(grp + (rg * 4 + c4) * 32 + 16 * (gi >> 2) + 8 * (gi & 1));
            e = grp[2048 + rg * 8 + 2 * c4 + (gi >> 2)];
        } else {  // GGUF blocks of 17 bytes, row after row
            const uint8_t* blk = q + r * prb + 17 * (2 * c4 + (gi >> 2));
            e = blk[0];
            const uint8_t* nb = blk + 1 + 8 * (gi & 1);
            b.x = (uint32_t)nb[0] | ((uint32_t)nb[1] << 8) | ((uint32_t)nb[2] << 16) | ((uint32_t)nb[3] << 24);
            b.y = (uint32_t)nb[4] | ((uint32_t)nb[5] << 8) | ((uint32_t)nb[6] << 16) | ((uint32_t)nb[7] << 24);
        }
        const __half2 sc = mx_scale_h2(e);
        const int sh = (gi & 2) ? 4 : 0;
        uint32_t w[4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t y = ((h ? b.y : b.x) >> sh) & 0x0F0F0F0Fu;
            const uint32_t z = y | (y >> 4);  // byte 0: nibbles 0, 1; byte 2: nibbles 2, 3
            const uint32_t p0 = *reinterpret_cast<const uint32_t*>(tab + ((z & 0xFFu) << 6));
            const uint32_t p1 = *reinterpret_cast<const uint32_t*>(tab + (((z >> 16) & 0xFFu) << 6));
            w[2 * h] = u_h2(__hmul2(h2_u(p0), sc));
            w[2 * h + 1] = u_h2(__hmul2(h2_u(p1), sc));
        }
        return make_uint4(w[0], w[1], w[2], w[3]);
    } else if (FMT == F_Q4_K) {
        // y = d * sc * q - dmin * m per 32-column sub-block (candle's to_float, each operation
        // rounded as there), then rounded to f16; sub-block 2 c4 + (gi >= 4) holds the low
        // (gi < 4) or high nibbles of bytes 32 c4 + 8 (gi % 4) .. + 7
        const uint8_t* row = q + r * 144;
        const float d = h2f_bits(*reinterpret_cast<const uint16_t*>(row));
        const float dmin = h2f_bits(*reinterpret_cast<const uint16_t*>(row + 2));
        int sc, mn;
        get_scale_min_k4(2 * c4 + (gi >> 2), row + 4, &sc, &mn);
        const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
        const uint2 b = *reinterpret_cast<const uint2*>(row + 16 + 32 * c4 + 8 * (gi & 3));
        const uint32_t sh = gi >= 4 ? 4 : 0;
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t byte = ((j < 4 ? b.x : b.y) >> (8 * (j & 3))) & 0xFFu;
            v[j] = __fsub_rn(__fmul_rn(d1, (float)((byte >> sh) & 0xFu)), m1);
        }
        uint4 o;
        o.x = u_h2(__floats2half2_rn(v[0], v[1]));
        o.y = u_h2(__floats2half2_rn(v[2], v[3]));
        o.z = u_h2(__floats2half2_rn(v[4], v[5]));
        o.w = u_h2(__floats2half2_rn(v[6], v[7]));
        return o;
    } else if (FMT == F_IQ4_XS) {
        // chunk gi: block gi / 4 of the slice, its columns 8 (gi % 4) ..: the low (gi % 4 < 2) or
        // high nibbles of bytes 8 (gi % 2) .. + 7; y = (d * (ls - 32)) * level in f32 (the
        // reference's dequantize_iq4_xs), rounded to f16 once
        const uint8_t* grp = q + (r >> 4) * (16 * 136);
        const int rg = r & 15;
        const uint2 M = *reinterpret_cast<const uint2*>(grp + 2048 + rg * 8);
        const int ib = 2 * c4 + (gi >> 2);
        const int ls = (int)(((M.y >> (4 * ib)) & 15u) | (((M.x >> (16 + 2 * ib)) & 3u) << 4));
        const float ds = __fmul_rn(h2f_bits((uint16_t)(M.x & 0xFFFFu)), (float)(ls - 32));
        const uint2 b = *reinterpret_cast<const uint2*>(grp + (rg * 4 + c4) * 32 + 16 * (gi >> 2) + 8 * (gi & 1));
        const int sh = (gi & 2) ? 4 : 0;
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t n = (((j < 4 ? b.x : b.y) >> (8 * (j & 3) + sh)) & 15u);
            v[j] = __fmul_rn(ds, *reinterpret_cast<const float*>(tab + n * 128));
        }
        uint4 o;
        o.x = u_h2(__floats2half2_rn(v[0], v[1]));
        o.y = u_h2(__floats2half2_rn(v[2], v[3]));
        o.z = u_h2(__floats2half2_rn(v[4], v[5]));
        o.w = u_h2(__floats2half2_rn(v[6], v[7]));
        return o;
    } else if (FMT == F_IQ2_XXS) {
        // record (r, c4) = [entries | signs/scale] of the slice's two 32-column blocks; chunk gi is
        // group gi % 4 of block gi / 4
        const uint8_t* grp = q + (r >> 4) * (16 * 66);
        const int rg = r & 15;
        const uint4 Q = *reinterpret_cast<const uint4*>(grp + (rg * 4 + c4) * 16);
        const __half2 d2 = __half2half2(__ushort_as_half(*reinterpret_cast<const uint16_t*>(grp + 1024 + 2 * rg)));
        const uint32_t qw = gi < 4 ? Q.x : Q.z, aux = gi < 4 ? Q.y : Q.w;
        const uint32_t b = __byte_perm(qw, 0u, 0x4440 | (gi & 3));
        const uint4 G = *reinterpret_cast<const uint4*>(tab + b * 32);
        const uint32_t s7 = (aux >> (7 * (gi & 3))) & 127u;
        const uint32_t s8 = s7 | ((__popc(s7) & 1u) << 7);
        const __half2 od = __hmul2(odd_h2(aux >> 28), __floats2half2_rn(0.125f, 0.125f));
        uint4 o;
        o.x = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 0, G.x)), od), d2));
        o.y = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 2, G.y)), od), d2));
        o.z = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 4, G.z)), od), d2));
        o.w = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 6, G.w)), od), d2));
        return o;
    } else if (FMT == F_IQ3_XXS) {
        // entries 2 gi, 2 gi + 1 of the slice's 16 (two per 8 columns); signs/scale word of block gi / 4
        const uint8_t* grp = q + (r >> 4) * (16 * 98);
        const int rg = r & 15;
        const uint16_t e2 = *reinterpret_cast<const uint16_t*>(grp + (rg * 4 + c4) * 16 + 2 * gi);
        const uint32_t aux = *reinterpret_cast<const uint32_t*>(grp + 1024 + (rg * 4 + c4) * 8 + 4 * (gi >> 2));
        const __half2 d2 = __half2half2(__ushort_as_half(*reinterpret_cast<const uint16_t*>(grp + 1536 + 2 * rg)));
        const uint32_t s7 = (aux >> (7 * (gi & 3))) & 127u;
        const uint32_t s8 = s7 | ((__popc(s7) & 1u) << 7);
        const __half2 od = __hmul2(odd_h2(aux >> 28), __floats2half2_rn(0.25f, 0.25f));
        const uint2 G0 = *reinterpret_cast<const uint2*>(tab + (e2 & 0xFFu) * 32);
        const uint2 G1 = *reinterpret_cast<const uint2*>(tab + (e2 >> 8) * 32);
        uint4 o;
        o.x = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 0, G0.x)), od), d2));
        o.y = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 2, G0.y)), od), d2));
        o.z = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 4, G1.x)), od), d2));
        o.w = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 6, G1.y)), od), d2));
        return o;
    } else if (FMT == F_IQ2_S) {
        const uint8_t* grp = q + (r >> 4) * (16 * 82);
        const int rg = r & 15;
        const uint4 Q = *reinterpret_cast<const uint4*>(grp + (rg * 4 + c4) * 16);
        const uint32_t H = *reinterpret_cast<const uint32_t*>(grp + 1024 + (rg * 4 + c4) * 4);
        const __half2 d2 = __half2half2(__ushort_as_half(*reinterpret_cast<const uint16_t*>(grp + 1280 + 2 * rg)));
        const uint32_t qw = gi < 4 ? Q.x : Q.y, sw = gi < 4 ? Q.z : Q.w;
        const uint32_t b = __byte_perm(qw, 0u, 0x4440 | (gi & 3));
        const uint32_t idx = b | (((H >> (2 * gi)) & 3u) << 8);
        const uint4 G = *reinterpret_cast<const uint4*>(tab + idx * 32);
        const uint32_t s8 = __byte_perm(sw, 0u, 0x4440 | (gi & 3));
        const __half2 od = __hmul2(odd_h2((H >> (16 + 4 * (gi >> 1))) & 0xFu), __floats2half2_rn(0.125f, 0.125f));
        uint4 o;
        o.x = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 0, G.x)), od), d2));
        o.y = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 2, G.y)), od), d2));
        o.z = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 4, G.z)), od), d2));
        o.w = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 6, G.w)), od), d2));
        return o;
    } else {
        const uint8_t* grp = q + (r >> 4) * (16 * 110);
        const int rg = r & 15;
        const uint16_t qs2 = *reinterpret_cast<const uint16_t*>(grp + rg * 64 + 16 * c4 + 2 * gi);
        const uint8_t s8 = grp[1024 + rg * 32 + 8 * c4 + gi];
        const uint16_t qh = *reinterpret_cast<const uint16_t*>(grp + 1536 + rg * 8 + 2 * c4);
        const uint8_t sc = grp[1664 + rg * 4 + c4];
        const __half2 d2 = __half2half2(__ushort_as_half(*reinterpret_cast<const uint16_t*>(grp + 1728 + 2 * rg)));
        const __half2 od = odd_h2((sc >> (4 * (gi >> 2))) & 0xFu);
        const uint32_t i0 = (qs2 & 0xFFu) | (((qh >> (2 * gi)) & 1u) << 8);
        const uint32_t i1 = (qs2 >> 8) | (((qh >> (2 * gi + 1)) & 1u) << 8);
        const uint2 G0 = *reinterpret_cast<const uint2*>(tab + i0 * 32);
        const uint2 G1 = *reinterpret_cast<const uint2*>(tab + i1 * 32);
        uint4 o;
        o.x = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 0, G0.x)), od), d2));
        o.y = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 2, G0.y)), od), d2));
        o.z = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 4, G1.x)), od), d2));
        o.w = u_h2(__hmul2(__hmul2(h2_u(sgn_pair(s8, 6, G1.y)), od), d2));
        return o;
    }
}

__device__ __forceinline__ float silu(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

// 64-column stages of piece kp (a tail piece of MXFP4 may hold fewer than four).
__device__ __forceinline__ int piece_stages(const Layout& L, int kp) {
    return kp < L.n_kp - 1 ? 4 : (int)((L.k - (int64_t)PIECE_K * (L.n_kp - 1)) / 64);
}
// Whether half 1 (A rows 64-127) of row tile mt exists: always for fused gate/up; for a plain
// launch, unless the matrix ends with half a tile.
__device__ __forceinline__ bool half1_exists(const MmaArgs& a, int mt) {
    return a.fused || (int64_t)(2 * mt + 1) * 64 < a.a0.L.n;
}

}  // namespace mm

// LO: the activations come as f16 hi and lo parts (a.b, a.blo; x = hi + lo exactly for the
// Q8_0-rounded rows of the candle policy): each B stage holds both tiles (two stages instead of
// three), and every A tile meets both, so the products carry f32-level activations.
template <int FMT, bool LO>
__global__ void __launch_bounds__(mm::THREADS, 1) k_mma(MmaArgs a) {
    using namespace mm;
    using G = Geo<LO>;
    using S = Smem<FMT, LO>;
    constexpr uint32_t TN = NMAX;       // picks per column tile
    constexpr int LO_OFF = NMAX * 128;  // the lo tile inside a B stage
    constexpr int NS = G::NSS;          // (shadows mm::NS)
    constexpr int B_BYTES = G::B_STAGE;
    constexpr int GATHER_PER = G::GP;
    extern __shared__ uint8_t smem_raw[];
    // 1024-aligned base (the swizzled operand tiles need it)
    uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
    Bars* bars = reinterpret_cast<Bars*>(smem + S::BAR);
    uint8_t* sa = smem + S::A;
    uint8_t* sb = smem + S::B;
    uint8_t* sq = smem + S::Q;
    uint8_t* tab = smem + S::TAB;
    float* xch = reinterpret_cast<float*>(smem + S::XCH);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < NQ; ++i) {
            mbar_init(&bars->full_q[i], 1);
            mbar_init(&bars->empty_q[i], N_DEC);
        }
        for (int i = 0; i < NS; ++i) {
            mbar_init(&bars->full_a[i], N_DEC);
            mbar_init(&bars->full_b[i], N_GATHER * 32);
            mbar_init(&bars->empty_s[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars->acc_full[i], 1);
            mbar_init(&bars->acc_empty[i], 4);
        }
        mbar_init(&bars->mma_done, 1);
        fence_mbar_init();
    }
    if (warp == W_MMA) {
        tmem_alloc(&bars->tmem, TMEM_COLS);
        tmem_relinquish();
    }
    if (warp >= W_DEC) {  // the codebook as f16 values: IQ2_S 8 per entry, IQ3_S 4
        const int t = tid - W_DEC * 32;
        if (FMT == F_Q4_K) {
            // no codebook
        } else if (FMT == F_IQ4_XS) {
            for (int e = t; e < 16 * 32; e += N_DEC * 32)
                *reinterpret_cast<float*>(tab + (e >> 5) * 128 + (e & 31) * 4) = (float)cwx_iq4nl(e >> 5);
        } else if (FMT == F_MXFP4) {
            const int8_t kv[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
            for (int e = t; e < 256 * 16; e += N_DEC * 32) {
                const int pr = e >> 4;
                *reinterpret_cast<uint32_t*>(tab + pr * 64 + (e & 15) * 4) =
                    u_h2(__floats2half2_rn((float)kv[pr & 15], (float)kv[pr >> 4]));
            }
        } else if (FMT == F_IQ2_S || FMT == F_IQ2_XXS) {
            for (int e = t; e < (FMT == F_IQ2_S ? 1024 : 256); e += N_DEC * 32) {
                const uint64_t v = cwx_iq2s_expand(FMT == F_IQ2_S ? d_iq2s_codes[e] : d_iq2xxs_codes[e]);
                uint4 o;
                o.x = u_h2(__floats2half2_rn((float)(v & 0xFF), (float)((v >> 8) & 0xFF)));
                o.y = u_h2(__floats2half2_rn((float)((v >> 16) & 0xFF), (float)((v >> 24) & 0xFF)));
                o.z = u_h2(__floats2half2_rn((float)((v >> 32) & 0xFF), (float)((v >> 40) & 0xFF)));
                o.w = u_h2(__floats2half2_rn((float)((v >> 48) & 0xFF), (float)(v >> 56)));
                *reinterpret_cast<uint4*>(tab + e * 32) = o;
                *reinterpret_cast<uint4*>(tab + e * 32 + 16) = o;
            }
        } else {
            for (int e = t; e < (FMT == F_IQ3_S ? 512 : 256); e += N_DEC * 32) {
                const uint32_t v = FMT == F_IQ3_S ? cwx_iq3s_expand(d_iq3s_codes[e]) : cwx_iq3xxs_expand(d_iq3xxs_codes[e]);
                const uint2 o = make_uint2(u_h2(__floats2half2_rn((float)(v & 0xFF), (float)((v >> 8) & 0xFF))),
                                           u_h2(__floats2half2_rn((float)((v >> 16) & 0xFF), (float)(v >> 24))));
#pragma unroll
                for (int j = 0; j < 4; ++j) *reinterpret_cast<uint2*>(tab + e * 32 + j * 8) = o;
            }
        }
    }
    tc_before();
    __syncthreads();
    tc_after();
    const uint32_t tmem = bars->tmem;
    const uint32_t n_used = *a.n_used;
    const int n_kp = a.a0.L.n_kp;
    const int nks = 4 * (n_kp - 1) + piece_stages(a.a0.L, n_kp - 1);  // 64-column stages per item

    if (warp == W_MMA) {
        // ---------------- MMA issue: the whole warp walks the stages (the descriptors stay
        // warp-uniform), one elected lane issues the MMAs and commits
        Iter it;
        MItem m;
        uint32_t c = 0;  // stage counter
        bool ok = true;
        int li = 0;
        const bool leader = elect_one();
        for (uint32_t i = blockIdx.x; ok && next_item(a, it, i, n_used, &m, TN); i += gridDim.x, ++li) {
            const int buf = li & 1;
            const uint32_t use = (uint32_t)li >> 1;
            if (use > 0 && !mbar_wait(&bars->acc_empty[buf], (use - 1) & 1, a.err)) {
                ok = false;
                break;
            }
            tc_after();
            const int npad = ((int)m.ntok + 15) & ~15;
            const uint32_t idesc = idesc_f16(npad);
            const uint32_t d = tmem + (uint32_t)buf * 256;
            for (int ks = 0; ks < nks; ++ks, ++c) {
                const int s = (int)(c % NS);
                const uint32_t ph = (c / NS) & 1;
                if (!mbar_wait(&bars->full_a[s], ph, a.err) || !mbar_wait(&bars->full_b[s], ph, a.err)) {
                    ok = false;
                    break;
                }
                tc_after();
                fence_async_smem();  // the gathered activations were written by cp.async
                const uint64_t ad = sdesc(sa + s * A_BYTES), bd = sdesc(sb + s * B_BYTES);
                if (leader) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {  // +32 bytes = +2 in the descriptor's address field
                        tc_mma(d, ad + 2 * kk, bd + 2 * kk, idesc, (ks | kk) != 0);
                        if (LO) tc_mma(d, ad + 2 * kk, sdesc(sb + s * B_BYTES + LO_OFF) + 2 * kk, idesc, 1);
                    }
                    tc_commit(&bars->empty_s[s]);
                }
                __syncwarp();
            }
            if (!ok) break;
            if (leader) tc_commit(&bars->acc_full[buf]);
            __syncwarp();
        }
        // every MMA issued has finished before the TMEM is freed
        if (leader) tc_commit(&bars->mma_done);
        __syncwarp();
        mbar_wait(&bars->mma_done, 0, a.err);
    } else if (warp == W_QCOPY) {
        // ---------------- quantised pieces: two 64-row halves per piece, one bulk copy each
        Iter it;
        MItem m;
        uint32_t p = 0;
        bool ok = true;
        for (uint32_t i = blockIdx.x; ok && next_item(a, it, i, n_used, &m, TN); i += gridDim.x) {
            for (int kp = 0; kp < n_kp; ++kp, ++p) {
                const int s = (int)(p % NQ);
                const uint32_t use = p / NQ;
                if (use > 0 && !mbar_wait(&bars->empty_q[s], (use - 1) & 1, a.err)) {
                    ok = false;
                    break;
                }
                // (64 rows of a piece: a multiple of 16 bytes)
                const int64_t hb0 = 64 * piece_row_bytes(a.a0.L, kp);
                const int64_t hb1 = half1_exists(a, m.mt) ? 64 * piece_row_bytes((a.fused ? a.a1 : a.a0).L, kp) : 0;
                if (lane == 0) mbar_expect_tx(&bars->full_q[s], (uint32_t)(hb0 + hb1));
                __syncwarp();
                uint8_t* dst = sq + s * Q_BYTES;
                if (lane == 0) bulk_g2s(dst, half_src(a, 0, m.e, m.mt, kp), (uint32_t)hb0, &bars->full_q[s]);
                if (lane == 1 && hb1) bulk_g2s(dst + hb0, half_src(a, 1, m.e, m.mt, kp), (uint32_t)hb1, &bars->full_q[s]);
            }
        }
        // the copies in flight land before the CTA ends
        for (uint32_t q = p > NQ ? p - NQ : 0; q < p; ++q) mbar_wait(&bars->full_q[q % NQ], (q / NQ) & 1, a.err);
    } else if (warp >= W_GATHER && warp < W_GATHER + N_GATHER) {
        // ---------------- activation rows: chunk i = t + 128 j (j < 16) of a stage is row i / 8,
        // 16-byte chunk i % 8 (so 8 threads read one row's 128 contiguous bytes)
        const int t = tid - W_GATHER * 32;
        Iter it;
        MItem m;
        uint32_t c = 0;
        bool ok = true;
        for (uint32_t i = blockIdx.x; ok && next_item(a, it, i, n_used, &m, TN); i += gridDim.x) {
            // chunk slot j: pick (t / 8) + 16 j (LO: + 16 (j % 16), from the hi rows for j < 16 and
            // the lo rows above; the row of slot j + 16 is the row of slot j)
            constexpr int NP = LO ? GATHER_PER / 2 : GATHER_PER;  // picks per gather thread
            int row[NP];
#pragma unroll
            for (int j = 0; j < NP; ++j) {
                const uint32_t n = (uint32_t)(t >> 3) + 16 * j;
                if (n < m.ntok) {
                    const uint32_t pk = a.pairs[m.first + m.n0 + n];
                    row[j] = (int)(a.rowmap ? a.rowmap[pk] : pk / (uint32_t)a.bdiv);
                } else {
                    row[j] = -1;
                }
            }
            for (int ks = 0; ks < nks; ++ks, ++c) {
                const int s = (int)(c % NS);
                const uint32_t use = c / NS;
                if (lane == 0 && use > 0 && !mbar_wait(&bars->empty_s[s], (use - 1) & 1, a.err)) ok = false;
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                uint8_t* bt = sb + s * B_BYTES;
                const int64_t co = 16 * (t & 7) + (int64_t)ks * 128;
#pragma unroll
                for (int j = 0; j < GATHER_PER; ++j) {
                    const bool lo = LO && j >= NP;
                    const int jj = lo ? j - NP : j;
                    const int n = (t >> 3) + 16 * jj, ch = t & 7;
                    if (row[jj] >= 0)
                        cp_async16(bt + (lo ? LO_OFF : 0) + n * 128 + ((ch ^ (n & 7)) << 4),
                                   (lo ? a.blo : a.b) + co + (int64_t)row[jj] * a.bstride);
                }
                cp_async_arrive(&bars->full_b[s]);
            }
        }
        cp_async_wait_all();
    } else if (warp >= W_DEC) {
        // ---------------- decode: the decoder threads share a stage's 128 rows x 8 chunks
        const int t = tid - W_DEC * 32;
        // this lane's copy of the table
        const uint8_t* tl = tab + ((FMT == F_IQ2_S || FMT == F_IQ2_XXS) ? (lane & 1) * 16
                                   : FMT == F_IQ4_XS                   ? lane * 4
                                   : FMT == F_MXFP4                    ? (lane & 15) * 4
                                                                       : (lane & 3) * 8);
        Iter it;
        MItem m;
        uint32_t c = 0, p = 0;
        bool ok = true;
        for (uint32_t i = blockIdx.x; ok && next_item(a, it, i, n_used, &m, TN); i += gridDim.x) {
            for (int kp = 0; kp < n_kp && ok; ++kp, ++p) {
                const int qs = (int)(p % NQ);
                if (!mbar_wait(&bars->full_q[qs], (p / NQ) & 1, a.err)) {
                    ok = false;
                    break;
                }
                const uint8_t* q = sq + qs * Q_BYTES;
                const int prb = (int)piece_row_bytes(a.a0.L, kp);
                const int rows = half1_exists(a, m.mt) ? 128 : 64;  // (the rows of a missing half stay unwritten:
                                                                   // their outputs are never read)
                const int nst = piece_stages(a.a0.L, kp);
                for (int c4 = 0; c4 < nst; ++c4, ++c) {
                    const int s = (int)(c % NS);
                    const uint32_t use = c / NS;
                    if (lane == 0 && use > 0 && !mbar_wait(&bars->empty_s[s], (use - 1) & 1, a.err)) ok = false;
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) break;
                    uint8_t* at = sa + s * A_BYTES;
#pragma unroll
                    for (int j = 0; j < DEC_PER; ++j) {
                        const int ci = t + N_DEC * 32 * j;  // chunk: row ci / 8, 16-byte chunk ci % 8
                        if (ci < DEC_CHUNKS && (ci >> 3) < rows) {
                            const int r = ci >> 3, gi = ci & 7;
                            const uint4 w = dec_chunk<FMT>(q, r, c4, gi, tl, prb);
                            *reinterpret_cast<uint4*>(at + r * 128 + ((gi ^ (r & 7)) << 4)) = w;
                        }
                    }
                    fence_async_smem();  // the tensor cores read the tile through the async proxy
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bars->full_a[s]);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->empty_q[qs]);
            }
        }
    } else {
        // ---------------- epilogue (warps 0-3: TMEM lanes 32 w .. 32 w + 31 = A rows)
        Iter it;
        MItem m;
        int li = 0;
        for (uint32_t i = blockIdx.x; next_item(a, it, i, n_used, &m, TN); i += gridDim.x, ++li) {
            const int buf = li & 1;
            if (!mbar_wait(&bars->acc_full[buf], ((uint32_t)li >> 1) & 1, a.err)) break;
            tc_after();
            const uint32_t* pk = a.pairs + m.first + m.n0;
            const int nch = ((int)m.ntok + 31) >> 5;
            for (int cc = 0; cc < nch; ++cc) {
                uint32_t r[32];
                tc_ld32(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(buf * 256 + cc * 32), r);
                tc_wait_ld();
                if (a.fused) {
                    // Lanes 0-63 hold gate rows, 64-127 the up rows of the same 64 features. The
                    // four warps split the chunk's 32 picks: warps 0-1 take picks 0-15 (their
                    // up values from warps 2-3 through shared memory), warps 2-3 picks 16-31 (their
                    // gate values from warps 0-1). A warp's 32 features are one Q8_0 block of each
                    // pick's h row.
                    const int hf = warp & 1;
                    const bool gate_side = warp < 2;
                    float* give = xch + (gate_side ? 0 : 1024);
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj)
                        give[jj * 64 + hf * 32 + lane] = __uint_as_float(gate_side ? r[16 + jj] : r[jj]);
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                    const float* take = xch + (gate_side ? 1024 : 0);
                    const int64_t f = (int64_t)m.mt * 64 + hf * 32 + lane;
                    const int64_t fb = (int64_t)m.e * a.a0.L.n + f;  // expert bias index
                    const float gb = a.gate_b ? a.gate_b[fb] : 0.f, ub = a.up_b ? a.up_b[fb] : 0.f;
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const int col = cc * 32 + (gate_side ? jj : 16 + jj);
                        if (col < (int)m.ntok) {  // (the same for the whole warp)
                            const float mine = __uint_as_float(gate_side ? r[jj] : r[16 + jj]);
                            const float other = take[jj * 64 + hf * 32 + lane];
                            const float g = gate_side ? mine : other, u = gate_side ? other : mine;
                            float h;
                            if (a.act == CWX_ACT_SILU) {
                                h = __fmul_rn(silu(g), u);
                            } else {  // gpt-oss clamped SwiGLU, as k_prep (act.cu)
                                float gv = a.gate_b ? __fadd_rn(g, gb) : g, uv = a.up_b ? __fadd_rn(u, ub) : u;
                                gv = fminf(gv, a.limit);
                                uv = fminf(fmaxf(uv, -a.limit), a.limit);
                                const float z = __fmul_rn(gv, a.alpha);
                                const float sg = __fdiv_rn(1.0f, __fadd_rn(expf(-z), 1.0f));
                                h = __fmul_rn(__fadd_rn(uv, 1.0f), __fmul_rn(gv, sg));
                            }
                            if (a.h_q80) {  // BlockQ8_0::from_float over the warp's block, as pack_words
                                float am = fabsf(h);
                                for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
                                const float d = __fdiv_rn(am, 127.f);
                                const float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
                                const float qv = fminf(fmaxf(roundf(__fmul_rn(h, id)), -128.f), 127.f);
                                h = __fmul_rn(qv, __half2float(__float2half_rn(d)));
                            }
                            a.hout[(int64_t)pk[col] * a.ostride + f] = __float2half_rn(h);
                        }
                    }
                    asm volatile("bar.sync 1, 128;" ::: "memory");
                } else {
                    const int64_t f = (int64_t)m.mt * 128 + warp * 32 + lane;
                    if (f < a.a0.L.n) {  // (the rows of a missing half tile are not outputs)
                        const float bv = a.bias ? a.bias[(int64_t)m.e * a.a0.L.n + f] : 0.f;
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const int col = cc * 32 + j;
                            float v = __uint_as_float(r[j]);
                            if (a.bias) v = __fadd_rn(v, bv);
                            if (col < (int)m.ntok) a.out[(int64_t)pk[col] * a.ostride + f] = v;
                        }
                    }
                }
            }
            tc_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->acc_empty[buf]);
        }
    }
    tc_before();
    __syncthreads();
    tc_after();
    if (warp == W_MMA) tmem_dealloc(tmem, TMEM_COLS);
}

// x (R, K) f32 -> f16 rows (the activation rows of the fused gate/up products).
__global__ void __launch_bounds__(256) k_f16rows(const float* __restrict__ x, int64_t n, __half* __restrict__ y) {
    const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i + 3 < n) {
        const float4 v = *reinterpret_cast<const float4*>(x + i);
        *reinterpret_cast<__half2*>(y + i) = __floats2half2_rn(v.x, v.y);
        *reinterpret_cast<__half2*>(y + i + 2) = __floats2half2_rn(v.z, v.w);
    } else {
        for (int64_t j = i; j < n; ++j) y[j] = __float2half_rn(x[j]);
    }
}

int launch_f16rows(const float* x, int64_t n, __half* y, cudaStream_t st) {
    if (n <= 0) return CWX_OK;
    const int64_t blocks = (n / 4 + 255) / 256 + 1;
    k_f16rows<<<(unsigned)blocks, 256, 0, st>>>(x, n, y);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_f16rows");
}

// x (R, K) f32 -> f16 rows through Q8_0 per 32 columns (BlockQ8_0::from_float, as pack_words):
// one warp per block, lane j holding column j.
// The value q * d (d rounded to f16, q <= 127: at most 18 significant bits) is exactly hi + lo.
__global__ void __launch_bounds__(256) k_f16rows_q80(const float* __restrict__ x, int64_t n, __half* __restrict__ y,
                                                     __half* __restrict__ ylo) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const float v = i < n ? x[i] : 0.f;
    float am = fabsf(v);
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const float d = __fdiv_rn(am, 127.f);
    const float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
    const float qv = fminf(fmaxf(roundf(__fmul_rn(v, id)), -128.f), 127.f);
    const float w = __fmul_rn(qv, __half2float(__float2half_rn(d)));
    const __half h = __float2half_rn(w);
    if (i < n) {
        y[i] = h;
        if (ylo) ylo[i] = __float2half_rn(__fsub_rn(w, __half2float(h)));
    }
}

int launch_f16rows_q80(const float* x, int64_t n, __half* y, __half* ylo, cudaStream_t st) {
    if (n <= 0) return CWX_OK;
    if (n % 32) return fail(CWX_EINVAL, "Q8_0 rows: %lld values is not a whole number of blocks", (long long)n);
    k_f16rows_q80<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, n, y, ylo);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_f16rows_q80");
}

// Formats the tensor-core products decode.
bool mma_format(int fmt) {
    return fmt == F_IQ2_S || fmt == F_IQ3_S || fmt == F_IQ2_XXS || fmt == F_IQ3_XXS || fmt == F_IQ4_XS || fmt == F_Q4_K ||
           fmt == F_MXFP4;
}

// Which launches can take the tensor-core path: weights of those formats in full 64-row tiles
// (a plain launch may end with half of its 128-row tile), whole 256-column pieces or (MXFP4) a
// tail piece of whole 64-column stages, gate and up of one format and shape.
bool mma_supports(const MmaArgs& a) {
    const Layout& L = a.a0.L;
    if (!mma_format(L.fmt)) return false;
    if (L.k % (L.fmt == F_MXFP4 ? 64 : PIECE_K) || L.n % 64) return false;
    if (a.fused) {
        const Layout& U = a.a1.L;
        if (U.fmt != L.fmt || U.n != L.n || U.k != L.k) return false;
    }
    if (a.bstride % 16 || ((uintptr_t)a.b & 15)) return false;
    if (a.blo && (L.fmt != F_MXFP4 || ((uintptr_t)a.blo & 15))) return false;  // (hi + lo: the MXFP4 kernel)
    return true;
}

template <int FMT, bool LO = false>
static int launch_mma_f(const MmaArgs& a, int device, int sm_count, cudaStream_t st) {
    constexpr int fi = FMT == F_IQ2_S    ? 0
                       : FMT == F_IQ3_S  ? 1
                       : FMT == F_IQ2_XXS ? 2
                       : FMT == F_IQ3_XXS ? 3
                       : FMT == F_IQ4_XS ? 4
                       : FMT == F_MXFP4  ? 6
                                         : 5;
    const int smem = mm::Smem<FMT, LO>::TOTAL + 1024;
    static int attr_set[64][8] = {{0}};
    const int slot = LO ? 7 : fi;
    if (device < 0 || device >= 64 || !attr_set[device][slot]) {
        cudaError_t e = cudaFuncSetAttribute(k_mma<FMT, LO>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(k_mma)");
        if (device >= 0 && device < 64) attr_set[device][slot] = 1;
    }
    const unsigned grid = (unsigned)(sm_count > 0 ? sm_count : 1);
    k_mma<FMT, LO><<<grid, mm::THREADS, smem, st>>>(a);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_mma");
}

int launch_mma(const MmaArgs& in, int device, int sm_count, cudaStream_t st) {
    MmaArgs a = in;
    if (!mma_supports(a)) return fail(CWX_EUNSUPPORTED, "tensor-core expert products: unsupported layout");
    a.mtiles = (int)(a.fused ? a.a0.L.n / 64 : (a.a0.L.n + 127) / 128);
    switch (a.a0.L.fmt) {
        case F_IQ2_S: return launch_mma_f<F_IQ2_S>(a, device, sm_count, st);
        case F_IQ3_S: return launch_mma_f<F_IQ3_S>(a, device, sm_count, st);
        case F_IQ2_XXS: return launch_mma_f<F_IQ2_XXS>(a, device, sm_count, st);
        case F_IQ3_XXS: return launch_mma_f<F_IQ3_XXS>(a, device, sm_count, st);
        case F_IQ4_XS: return launch_mma_f<F_IQ4_XS>(a, device, sm_count, st);
        case F_MXFP4:
            return a.blo ? launch_mma_f<F_MXFP4, true>(a, device, sm_count, st)
                         : launch_mma_f<F_MXFP4, false>(a, device, sm_count, st);
        default: return launch_mma_f<F_Q4_K>(a, device, sm_count, st);
    }
}

// The shared expert as one pile holding every token: pairs = 0 .. T-1, used list {(0, 0, T)}.
__global__ void k_all_tokens(uint32_t* pairs, int T, uint32_t* used3, uint32_t* n_used) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < T) pairs[i] = (uint32_t)i;
    if (i == 0) {
        used3[0] = 0;
        used3[1] = 0;
        used3[2] = (uint32_t)T;
        *n_used = T > 0 ? 1u : 0u;
    }
}

int launch_all_tokens(uint32_t* pairs, int T, uint32_t* used3, uint32_t* n_used, cudaStream_t st) {
    k_all_tokens<<<(T + 255) / 256 + (T == 0), 256, 0, st>>>(pairs, T, used3, n_used);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_all_tokens");
}

}  // namespace cwx
