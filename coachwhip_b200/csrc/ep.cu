// Expert parallelism: the per-rank steps around the two all-to-all exchanges.
//
//   reference  experts are sharded across devices by expert (one exchange each way); the reference
//              itself runs one device, so the layer's semantics are StreamedMoe::forward
//              (crates/engine/src/experts.rs:2539-2614): out[t] = sum over picks of w * expert(x[t]).
//
// Units: a token sends its row once to every rank that owns at least one of its picks (a unit =
// (token, destination rank)), with one record per pick (the unit's index in the message, the
// expert's index on the destination, the pick's weight). Units of a destination are in token
// order, a unit's records in pick order. The destination runs the picks, sums each unit's
// weighted rows in pick order and sends one row per unit back; the source adds its units' rows in
// rank order. With top-k picks over W ranks a token sends min(k, W)-ish rows instead of k.
#include "cwx_common.cuh"
#include "kernels.cuh"

namespace cwx {

// Slot of expert e: rank slot / epr, local index slot % epr (the placement when there is one; a
// slot out of range falls back to e, so no record can leave the valid ranks and experts).
__device__ __forceinline__ uint32_t ep_slot(const int32_t* place, uint32_t e, int E) {
    if (!place) return e;
    const uint32_t s = (uint32_t)place[e];
    return s < (uint32_t)E ? s : e;
}

// Picks of each token per destination rank: cnt[t * W + d].
__global__ void k_ep_count(const uint32_t* __restrict__ ids, int T, int K, int epr, int W,
                           const int32_t* __restrict__ place, int E, int32_t* __restrict__ cnt) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    for (int d = 0; d < W; ++d) cnt[(int64_t)t * W + d] = 0;
    for (int j = 0; j < K; ++j) {
        const int d = (int)(ep_slot(place, ids[(int64_t)t * K + j], E) / (uint32_t)epr);
        cnt[(int64_t)t * W + d] += 1;
    }
}

// Per destination d (one block each): exclusive scans over the tokens of [cnt > 0] (unit
// position) and of cnt (first record), and the totals.
__global__ void __launch_bounds__(1024) k_ep_scan(const int32_t* __restrict__ cnt, int T, int W,
                                                  int32_t* __restrict__ upos, int32_t* __restrict__ pbase,
                                                  int32_t* __restrict__ tot /* (W, 2): units, picks */) {
    __shared__ int32_t su[32], sp[32];
    __shared__ int32_t carry_u, carry_p;
    const int d = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) carry_u = carry_p = 0;
    __syncthreads();
    for (int t0 = 0; t0 < T; t0 += 1024) {
        const int t = t0 + tid;
        const int c = t < T ? cnt[(int64_t)t * W + d] : 0;
        int u = c > 0, p = c;
        // inclusive warp scans
        for (int o = 1; o < 32; o <<= 1) {
            const int uu = __shfl_up_sync(0xffffffffu, u, o), pp = __shfl_up_sync(0xffffffffu, p, o);
            if (lane >= o) {
                u += uu;
                p += pp;
            }
        }
        if (lane == 31) {
            su[warp] = u;
            sp[warp] = p;
        }
        __syncthreads();
        if (warp == 0) {
            int a = su[lane], b = sp[lane];
            for (int o = 1; o < 32; o <<= 1) {
                const int aa = __shfl_up_sync(0xffffffffu, a, o), bb = __shfl_up_sync(0xffffffffu, b, o);
                if (lane >= o) {
                    a += aa;
                    b += bb;
                }
            }
            su[lane] = a;
            sp[lane] = b;
        }
        __syncthreads();
        const int wu = warp ? su[warp - 1] : 0, wp = warp ? sp[warp - 1] : 0;
        if (t < T) {
            upos[(int64_t)t * W + d] = c > 0 ? carry_u + wu + u - 1 : -1;
            pbase[(int64_t)t * W + d] = carry_p + wp + p - c;
        }
        __syncthreads();
        if (tid == 0) {
            carry_u += su[31];
            carry_p += sp[31];
        }
        __syncthreads();
    }
    if (tid == 0) {
        tot[2 * d] = carry_u;
        tot[2 * d + 1] = carry_p;
    }
}

// One block per token: its row to each destination it has picks on (f32, or f16 when the
// destination's products take f16 activations), and its pick records. upos becomes the unit's
// index in the whole send buffer (destination offsets added).
// With cap > 0 (the fixed-capacity layout of the library's own exchange) destination d's units
// start at row d * cap and its records at d * cap_rec, whatever the other destinations hold.
template <bool F16>
__global__ void __launch_bounds__(256) k_ep_pack_units(const float* __restrict__ x, int T, int H, int K, int W,
                                                       int epr, const int32_t* __restrict__ place, int E,
                                                       const uint32_t* __restrict__ ids,
                                                       const float* __restrict__ w, int32_t* __restrict__ upos,
                                                       const int32_t* __restrict__ pbase,
                                                       const int32_t* __restrict__ tot, void* __restrict__ send_rows,
                                                       int32_t* __restrict__ send_picks, int cap, int cap_rec) {
    const int t = blockIdx.x;
    __shared__ int32_t uoff[64], poff[64];
    if (threadIdx.x == 0) {
        int32_t a = 0, b = 0;
        for (int d = 0; d < W; ++d) {
            uoff[d] = cap > 0 ? d * cap : a;
            poff[d] = cap > 0 ? d * cap_rec : b;
            a += tot[2 * d];
            b += tot[2 * d + 1];
        }
    }
    __syncthreads();
    const float* src = x + (int64_t)t * H;
    for (int d = 0; d < W; ++d) {
        const int32_t u = upos[(int64_t)t * W + d];
        if (u < 0) continue;
        const int64_t g = (int64_t)uoff[d] + u;
        if (F16) {
            __half* dst = reinterpret_cast<__half*>(send_rows) + g * H;
            for (int c = threadIdx.x * 2; c < H; c += blockDim.x * 2)
                *reinterpret_cast<__half2*>(dst + c) = __floats2half2_rn(src[c], src[c + 1]);
        } else {
            float* dst = reinterpret_cast<float*>(send_rows) + g * H;
            for (int c = threadIdx.x * 4; c < H; c += blockDim.x * 4)
                *reinterpret_cast<float4*>(dst + c) = *reinterpret_cast<const float4*>(src + c);
        }
        if (threadIdx.x == 0) {
            int32_t r = poff[d] + pbase[(int64_t)t * W + d];
            for (int j = 0; j < K; ++j) {
                const uint32_t e = ep_slot(place, ids[(int64_t)t * K + j], E);
                if ((int)(e / (uint32_t)epr) != d) continue;
                send_picks[3 * (int64_t)r] = u;  // unit index within the message to d
                send_picks[3 * (int64_t)r + 1] = (int32_t)(e % (uint32_t)epr);
                send_picks[3 * (int64_t)r + 2] = __float_as_int(w[(int64_t)t * K + j]);
                ++r;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0)  // the unit's index in the whole send buffer, for the combine
        for (int d = 0; d < W; ++d) {
            const int32_t u = upos[(int64_t)t * W + d];
            if (u >= 0) upos[(int64_t)t * W + d] = uoff[d] + u;
        }
}

// Receiver: records of source s occupy [pstart[s], pstart[s+1]); their units start at ustart[s].
// rowmap[p] = the pick's row (unit) in the received buffer, eid[p], wgt[p]; first[u] = the unit's
// first record (units are contiguous runs of records).
__global__ void k_ep_recv(const int32_t* __restrict__ picks, int64_t P, EpOffsets off, uint32_t* __restrict__ rowmap,
                          uint32_t* __restrict__ eid, float* __restrict__ wgt, int32_t* __restrict__ first) {
    const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= P) return;
    int s = 0;
    while (s + 1 < off.n && p >= off.pstart[s + 1]) ++s;
    const uint32_t u = (uint32_t)(picks[3 * p] + off.ustart[s]);
    rowmap[p] = u;
    eid[p] = (uint32_t)picks[3 * p + 1];
    wgt[p] = __int_as_float(picks[3 * p + 2]);
    // a unit's records are a run inside its source's segment
    if (p == off.pstart[s] || picks[3 * (p - 1)] != picks[3 * p]) first[u] = (int32_t)p;
}

// Receiver, fixed-capacity layout: source s's records in slots [s * cap_rec, s * cap_rec + n_s)
// and its units in rows [s * cap, s * cap + u_s), the counts (u_s, n_s) in rcnt[2s], rcnt[2s + 1].
// The records are packed into picks 0 .. P-1 in source order (P = the sum of the n_s, written to
// n_picks): rowmap[p] = the unit's row, eid, wgt; each valid unit row r gets its run of records
// [first[r], end[r]).
__global__ void k_ep_recv_cap(const int32_t* __restrict__ picks, const int32_t* __restrict__ rcnt, int W, int cap,
                              int cap_rec, uint32_t* __restrict__ rowmap, uint32_t* __restrict__ eid,
                              float* __restrict__ wgt, int32_t* __restrict__ first, int32_t* __restrict__ end,
                              int32_t* __restrict__ n_picks) {
    const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (q == 0) {
        int32_t tot = 0;
        for (int s = 0; s < W; ++s) tot += rcnt[2 * s + 1];
        *n_picks = tot;
    }
    if (q >= (int64_t)W * cap_rec) return;
    const int s = (int)(q / cap_rec), i = (int)(q % cap_rec);
    const int32_t ns = rcnt[2 * s + 1];
    if (i >= ns) return;
    int64_t p = i;
    for (int r = 0; r < s; ++r) p += rcnt[2 * r + 1];
    const int32_t u = picks[3 * q];
    const uint32_t row = (uint32_t)((int64_t)s * cap + u);
    rowmap[p] = row;
    eid[p] = (uint32_t)picks[3 * q + 1];
    wgt[p] = __int_as_float(picks[3 * q + 2]);
    if (i == 0 || picks[3 * (q - 1)] != u) first[row] = (int32_t)p;
    if (i == ns - 1 || picks[3 * (q + 1)] != u) end[row] = (int32_t)(p + 1);
}

// Fixed-capacity unit sums: row r = s * cap + u is a unit when u < rcnt[2s]; its sum is written in
// place (other rows are left as they are: nothing reads them).
__global__ void __launch_bounds__(256) k_ep_unit_sum_cap(const float* __restrict__ y, const float* __restrict__ wgt,
                                                         const int32_t* __restrict__ first,
                                                         const int32_t* __restrict__ end,
                                                         const int32_t* __restrict__ rcnt, int cap, int H,
                                                         float* __restrict__ yu) {
    const int64_t r = blockIdx.x;
    const int s = (int)(r / cap), u = (int)(r % cap);
    if (u >= rcnt[2 * s]) return;
    const int64_t p0 = first[r], p1 = end[r];
    for (int c = threadIdx.x; c < H; c += blockDim.x) {
        float acc = 0.f;
        for (int64_t p = p0; p < p1; ++p) acc = __fadd_rn(acc, __fmul_rn(y[p * H + c], wgt[p]));
        yu[r * H + c] = acc;
    }
}

// yu[u] = sum over the unit's records p in order of wgt[p] * y[p].
__global__ void __launch_bounds__(256) k_ep_unit_sum(const float* __restrict__ y, const float* __restrict__ wgt,
                                                     const int32_t* __restrict__ first, int64_t U, int64_t P, int H,
                                                     float* __restrict__ yu) {
    const int64_t u = blockIdx.x;
    const int64_t p0 = first[u], p1 = u + 1 < U ? first[u + 1] : P;
    for (int c = threadIdx.x; c < H; c += blockDim.x) {
        float acc = 0.f;
        for (int64_t p = p0; p < p1; ++p) acc = __fadd_rn(acc, __fmul_rn(y[p * H + c], wgt[p]));
        yu[u * H + c] = acc;
    }
}

// out[t] = sum over destination ranks in order of the returned unit rows + sgate * shared + residual.
__global__ void __launch_bounds__(256) k_ep_combine(const float* __restrict__ back, const int32_t* __restrict__ unit,
                                                    int T, int W, int H, const float* __restrict__ shared,
                                                    const float* __restrict__ sgate,
                                                    const float* __restrict__ residual, float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * H) return;
    const int64_t t = i / H, c = i % H;
    float acc = 0.f;
    for (int d = 0; d < W; ++d) {
        const int32_t u = unit[t * W + d];
        if (u >= 0) acc = __fadd_rn(acc, back[(int64_t)u * H + c]);
    }
    if (shared) acc = __fadd_rn(acc, __fmul_rn(shared[t * H + c], sgate[t]));
    if (residual) acc = __fadd_rn(acc, residual[i]);
    out[i] = acc;
}

__global__ void k_f16_to_f32(const __half* __restrict__ x, int64_t n, float* __restrict__ y) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __half2float(x[i]);
}

static int launched(const char* what) {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, what);
}

int launch_ep_units(const float* x, int T, int H, int K, int W, int epr, const int32_t* place, int E,
                    const uint32_t* ids, const float* w, int32_t* cnt, int32_t* upos, int32_t* pbase, int32_t* tot,
                    bool f16, void* send_rows, int32_t* send_picks, cudaStream_t st, int cap, int cap_rec) {
    if (W > 64) return fail(CWX_EUNSUPPORTED, "expert parallelism over more than 64 ranks");
    if (T == 0) {
        CWX_CUDA(cudaMemsetAsync(tot, 0, (size_t)2 * W * 4, st));
        return CWX_OK;
    }
    k_ep_count<<<(T + 255) / 256, 256, 0, st>>>(ids, T, K, epr, W, place, E, cnt);
    k_ep_scan<<<W, 1024, 0, st>>>(cnt, T, W, upos, pbase, tot);
    if (f16)
        k_ep_pack_units<true><<<T, 256, 0, st>>>(x, T, H, K, W, epr, place, E, ids, w, upos, pbase, tot, send_rows, send_picks,
                                                 cap, cap_rec);
    else
        k_ep_pack_units<false><<<T, 256, 0, st>>>(x, T, H, K, W, epr, place, E, ids, w, upos, pbase, tot, send_rows, send_picks,
                                                  cap, cap_rec);
    return launched("expert-parallel dispatch kernels");
}

int launch_f16_to_f32(const __half* x, int64_t n, float* y, cudaStream_t st) {
    if (n == 0) return CWX_OK;
    k_f16_to_f32<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, n, y);
    return launched("k_f16_to_f32");
}

int launch_ep_recv(const int32_t* picks, int64_t P, const EpOffsets& off, uint32_t* rowmap, uint32_t* eid,
                   float* wgt, int32_t* first, cudaStream_t st) {
    if (P == 0) return CWX_OK;
    k_ep_recv<<<(unsigned)((P + 255) / 256), 256, 0, st>>>(picks, P, off, rowmap, eid, wgt, first);
    return launched("k_ep_recv");
}

int launch_ep_recv_cap(const int32_t* picks, const int32_t* rcnt, int W, int cap, int cap_rec, uint32_t* rowmap,
                       uint32_t* eid, float* wgt, int32_t* first, int32_t* end, int32_t* n_picks, cudaStream_t st) {
    const int64_t n = (int64_t)W * cap_rec;
    const unsigned blocks = (unsigned)(n > 0 ? (n + 255) / 256 : 1);
    k_ep_recv_cap<<<blocks, 256, 0, st>>>(picks, rcnt, W, cap, cap_rec, rowmap, eid, wgt, first, end, n_picks);
    return launched("k_ep_recv_cap");
}

int launch_ep_unit_sum_cap(const float* y, const float* wgt, const int32_t* first, const int32_t* end,
                           const int32_t* rcnt, int W, int cap, int H, float* yu, cudaStream_t st) {
    if ((int64_t)W * cap == 0) return CWX_OK;
    k_ep_unit_sum_cap<<<(unsigned)((int64_t)W * cap), 256, 0, st>>>(y, wgt, first, end, rcnt, cap, H, yu);
    return launched("k_ep_unit_sum_cap");
}

int launch_ep_unit_sum(const float* y, const float* wgt, const int32_t* first, int64_t U, int64_t P, int H, float* yu,
                       cudaStream_t st) {
    if (U == 0) return CWX_OK;
    k_ep_unit_sum<<<(unsigned)U, 256, 0, st>>>(y, wgt, first, U, P, H, yu);
    return launched("k_ep_unit_sum");
}

int launch_ep_combine(const float* back, const int32_t* unit, int T, int W, int H, const float* shared,
                      const float* sgate, const float* residual, float* out, cudaStream_t st) {
    if (T == 0) return CWX_OK;
    const int64_t n = (int64_t)T * H;
    k_ep_combine<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(back, unit, T, W, H, shared, sgate, residual, out);
    return launched("k_ep_combine");
}

}  // namespace cwx
