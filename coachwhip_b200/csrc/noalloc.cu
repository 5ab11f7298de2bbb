// cwx_permute_noalloc: the expert piles of cwx_permute for callers that must not allocate.
//
// cwx_permute keeps its scratch (per-tile expert counts, the used-expert list) in the context
// workspace, which grows on demand with cudaMalloc. Some callers cannot allow that: an engine
// that owns all device memory through its own pool and forbids hidden device allocations, a
// latency-critical loop in which cudaMalloc's implicit device synchronisation is not acceptable,
// or a caller without a cwx_ctx. This entry point runs the same kernels with the scratch in one
// fixed device array of this library (1 MiB per device), so a call makes no allocation at all:
// no cudaMalloc, no cudaFree, no allocating library call.
//
// Limits and rules:
//   - scratch words needed = ceil(tokens*top_k / 1024) * n_experts + 3 * n_experts + 8 must be
//     <= CWX_NOALLOC_SCRATCH_WORDS (262144), and n_experts <= 4096; larger calls are refused with
//     CWX_EINVAL before any device work.
//   - the array is shared by every call on a device, so calls on one device must not overlap:
//     issue them on one stream, or order the streams. Two calls in flight at once race.
//   - runs on the caller's current device; `stream` must belong to it.
//   - the first call on a device looks up the array's address (cudaGetSymbolAddress); make that
//     first call outside stream capture.
//   - only the error word must start at zero; each call clears it on its stream before the
//     kernels. The count and list words are fully rewritten by every call.
#include <mutex>

#include "cwx_common.cuh"
#include "kernels.cuh"

namespace cwx {

constexpr size_t NOALLOC_WORDS = CWX_NOALLOC_SCRATCH_WORDS;  // 1 MiB of uint32 per device
static_assert(NOALLOC_WORDS == 262144, "the header documents a 1 MiB scratch array");
constexpr int NOALLOC_MAX_EXPERTS = 4096;

static __device__ __align__(256) uint32_t g_noalloc_scratch[NOALLOC_WORDS];

static std::mutex g_noalloc_mu;
static uint32_t* g_noalloc_ptr[128];

static int noalloc_scratch(int device, uint32_t** out) {
    if (device < 0 || device >= 128) return fail(CWX_EINVAL, "cwx_permute_noalloc: device %d out of range", device);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cwx_permute_noalloc: cudaGetSymbolAddress");
        if (!p) return fail(CWX_ECUDA, "cwx_permute_noalloc: null scratch address");
        g_noalloc_ptr[device] = (uint32_t*)p;
    }
    *out = g_noalloc_ptr[device];
    return CWX_OK;
}

}  // namespace cwx

using namespace cwx;

extern "C" int cwx_permute_noalloc(const uint32_t* ids, int32_t T, int32_t K, int32_t E, uint32_t* pairs,
                                   uint32_t* heads, int32_t* dev_status, void* stream) {
    if ((!ids && T) || !heads || (!pairs && T)) return fail(CWX_EINVAL, "cwx_permute_noalloc: null argument");
    if (T < 0 || K < 1 || E < 1) return fail(CWX_EINVAL, "cwx_permute_noalloc: bad sizes");
    if (E > NOALLOC_MAX_EXPERTS)
        return fail(CWX_EINVAL, "cwx_permute_noalloc: n_experts=%d above the limit of %d", E, NOALLOC_MAX_EXPERTS);
    const int64_t n = (int64_t)T * K;
    const int64_t ntiles = n > 0 ? (n + 1023) / 1024 : 1;
    const size_t need = (size_t)ntiles * E + (size_t)3 * E + 8;
    if (need > NOALLOC_WORDS)
        return fail(CWX_EINVAL,
                    "cwx_permute_noalloc: tokens*top_k=%lld with n_experts=%d needs %zu scratch words, above the "
                    "fixed %zu; use cwx_permute",
                    (long long)n, E, need, NOALLOC_WORDS);
    int dev = 0;
    CWX_CUDA(cudaGetDevice(&dev));
    uint32_t* s = nullptr;
    int rc = noalloc_scratch(dev, &s);
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    // layout: [0] error word, [4] used-expert count, [8, 8+3E) used list, then the tile counts
    int* err = reinterpret_cast<int*>(s);
    uint32_t* n_used = s + 4;
    uint32_t* used3 = s + 8;
    uint32_t* counts = s + 8 + (size_t)3 * E;
    CWX_CUDA(cudaMemsetAsync(err, 0, 4, st));
    rc = launch_permute(ids, n, E, pairs, heads, used3, n_used, counts, err, st);
    if (rc) return rc;
    if (dev_status) CWX_CUDA(cudaMemcpyAsync(dev_status, err, 4, cudaMemcpyDeviceToDevice, st));
    return CWX_OK;
}
