// Expert parallelism: the per-rank steps around the two all-to-all exchanges.
//
//   reference  experts are sharded across devices by the SURVEY's EP design; the reference itself
//              runs one device, so the layer's semantics are StreamedMoe::forward
//              (crates/engine/src/experts.rs:2539-2614) and cw_pile's grouping (fuse_kernel.rs:180-202).
//
// Dispatch: the local tokens' picks, in pile order (grouped by expert, ascending pick index inside
// an expert), are also grouped by destination rank, because rank d owns the contiguous experts
// [d*epr, (d+1)*epr). One block per pick copies its token's row; the expert id is rewritten to
// the expert's index on the destination rank.
// Combine: the rows coming back arrive in the same pile order; inv maps a pick to its row.
#include "cwx_common.cuh"
#include "kernels.cuh"

namespace cwx {

__global__ void __launch_bounds__(256) k_ep_pack(const float* __restrict__ x, int H, int K,
                                                 const uint32_t* __restrict__ ids, const uint32_t* __restrict__ pairs,
                                                 int epr, float* __restrict__ send_rows,
                                                 uint32_t* __restrict__ send_eids) {
    const int64_t pos = blockIdx.x;
    const uint32_t p = pairs[pos];
    const int64_t t = p / (uint32_t)K;
    if (threadIdx.x == 0) send_eids[pos] = ids[p] % (uint32_t)epr;
    const float* src = x + t * H;
    float* dst = send_rows + pos * H;
    if ((H & 3) == 0) {
        for (int c = threadIdx.x * 4; c < H; c += blockDim.x * 4)
            *reinterpret_cast<float4*>(dst + c) = *reinterpret_cast<const float4*>(src + c);
    } else {
        for (int c = threadIdx.x; c < H; c += blockDim.x) dst[c] = src[c];
    }
}

__global__ void k_ep_counts(const uint32_t* __restrict__ heads, int E, int epr, int world, int32_t* __restrict__ counts) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= world) return;
    int64_t c = 0;
    for (int e = d * epr; e < (d + 1) * epr && e < E; ++e) c += heads[3 * e + 2];
    counts[d] = (int32_t)c;
}

__global__ void k_inverse(const uint32_t* __restrict__ pairs, int64_t n, uint32_t* __restrict__ inv) {
    const int64_t pos = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (pos < n) inv[pairs[pos]] = (uint32_t)pos;
}

int launch_ep_pack(const float* x, int H, int K, const uint32_t* ids, const uint32_t* pairs, int64_t n, int epr,
                   float* send_rows, uint32_t* send_eids, cudaStream_t st) {
    if (n == 0) return CWX_OK;
    k_ep_pack<<<(unsigned)n, 256, 0, st>>>(x, H, K, ids, pairs, epr, send_rows, send_eids);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_ep_pack");
}

int launch_ep_counts(const uint32_t* heads, int E, int epr, int world, int32_t* counts, cudaStream_t st) {
    k_ep_counts<<<(world + 127) / 128, 128, 0, st>>>(heads, E, epr, world, counts);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_ep_counts");
}

int launch_inverse(const uint32_t* pairs, int64_t n, uint32_t* inv, cudaStream_t st) {
    if (n == 0) return CWX_OK;
    k_inverse<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(pairs, n, inv);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CWX_OK : cuda_fail(e, "k_inverse");
}

}  // namespace cwx
