// The C ABI: contexts, workspace, error reporting, profiling, and the orchestration of one MoE
// layer.
//
// cwx_moe_forward is the resident branch of StreamedMoe::forward
// (crates/engine/src/experts.rs:2562-2614) plus SharedExpert::forward
// (crates/engine/src/model_next.rs:731-741): router logits, route, piles, gate/up products, the
// activation, down products, weighted combine, shared expert, optional residual
// (model_next.rs:1437). Everything is stream-ordered; nothing synchronises.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <vector>

#include "cwx_common.cuh"
#include "kernels.cuh"

namespace cwx {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? CWX_ENOMEM : CWX_ECUDA;
}

// Bump allocator over the context workspace.
struct Carve {
    uint8_t* base;
    size_t off;
    template <typename T>
    T* take(size_t count) {
        off = (off + 255) & ~(size_t)255;
        T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
        off += count * sizeof(T);
        return p;
    }
};

int ensure_ws(cwx_ctx* ctx, size_t bytes, cudaStream_t st) {
    if (bytes <= ctx->ws_bytes) return CWX_OK;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cap);
    if (cap != cudaStreamCaptureStatusNone)
        return fail(CWX_EINVAL, "workspace too small during stream capture: call cwx_ctx_reserve first");
    const size_t nb = ((bytes + (1 << 20) - 1) >> 20) << 20;  // 1 MB rounding, as the reference arena does
    if (ctx->ws) {
        cudaError_t e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return cuda_fail(e, "workspace grow");
        cudaFree(ctx->ws);
        ctx->ws = nullptr;
        ctx->ws_bytes = 0;
    }
    CWX_CUDA(cudaMalloc(&ctx->ws, nb));
    ctx->ws_bytes = nb;
    return CWX_OK;
}

// ---------------------------------------------------------------- profiling
struct ProfEvent {
    int phase;
    cudaEvent_t a, b;
};
using ProfLog = std::vector<ProfEvent>;

// Inside stream capture the events are recorded as graph nodes (cudaEventRecordExternal), so each
// replay of the graph records them again.
static void record_event(cudaEvent_t e, cudaStream_t st) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cap);
    if (cap == cudaStreamCaptureStatusActive) cudaEventRecordWithFlags(e, st, cudaEventRecordExternal);
    else cudaEventRecord(e, st);
}

// Event pair around one phase of a call (no-op unless profiling is on).
struct PhaseTimer {
    cwx_ctx* c;
    cudaStream_t st;
    int phase;
    cudaEvent_t a = nullptr;
    PhaseTimer(cwx_ctx* c_, cudaStream_t s_, int ph) : c(c_), st(s_), phase(ph) {
        if (!c->profiling) return;
        if (cudaEventCreate(&a) == cudaSuccess) record_event(a, st);
        else a = nullptr;
    }
    void end() {
        if (!a) return;
        cudaEvent_t b;
        if (cudaEventCreate(&b) == cudaSuccess) {
            record_event(b, st);
            static_cast<ProfLog*>(c->prof)->push_back({phase, a, b});
        } else {
            cudaEventDestroy(a);
        }
        a = nullptr;
    }
};

// ---------------------------------------------------------------- layer plan
static int act_mode_of(const cwx_bank* b, int policy) { return act_mode_for(b->L.fmt, policy); }

struct LayerPlan {
    int H, E, K, I, Is, T;
    int mgu, msgu, md, msd;  // activation modes
    float* logits;
    float* sgate;
    uint32_t* ids;
    float* w;
    uint32_t* heads;
    uint32_t* pairs;
    uint32_t* used3;
    uint32_t* n_used;
    uint32_t* perm;
    uint8_t* xpk[3];         // packed activation rows of x per activation mode
    float *g, *u, *gs, *us;  // gate / up outputs (routed by pick, shared by token)
    uint8_t *hpk, *hspk;     // packed hidden rows (routed, shared)
    float* y;
    float* ys;
    int64_t xrows;     // rows of x (T, unless an expert-parallel call maps picks to received rows)
    const uint32_t* rowmap;  // when set: activation row of pick p = rowmap[p]
    int mma;           // routed products on the tensor cores (IQ banks, large piles)
    int sh_mma;        // the shared expert on the tensor cores too (f32 activations)
    __half* x16;       // (T, H) f16 rows of x
    __half* x16lo;     // (T, H) their lo parts (MXFP4 under the Q8_0 policy), or null
    __half* h16;       // (n, I) f16 hidden rows per pick
    __half* hs16;      // (T, Is) f16 hidden rows of the shared expert
    uint32_t* spairs;  // the shared expert's pile (every token) and used list
    uint32_t* sused3;
    uint32_t* snused;
    size_t bytes;
};

// IQ formats: f32 activations under every policy (the reference runs them on Metal only), decoded
// by both product kernels.
static bool iq_format(int f) {
    return f == F_IQ2_S || f == F_IQ3_S || f == F_IQ2_XXS || f == F_IQ3_XXS || f == F_IQ4_XS;
}

// The shared expert joins the tensor-core products when its activations are f32 (no Q8 codes,
// whose per-piece scale a TMEM accumulator cannot apply) and its banks are a supported format.
static bool shared_mma_ok(const cwx_moe_layer* L) {
    if (!L->sh_gate) return false;
    const Layout &g = L->sh_gate->L, &u = L->sh_up->L, &d = L->sh_down->L;
    auto fmt_ok = [](int f) { return iq_format(f) || f == F_Q4_K; };
    if (!fmt_ok(g.fmt) || !fmt_ok(d.fmt) || g.fmt != u.fmt) return false;
    if (act_mode_of(L->sh_gate, L->act_mode) != AM_F32 || act_mode_of(L->sh_down, L->act_mode) != AM_F32)
        return false;
    return g.n % 256 == 0 && L->hidden % 256 == 0;
}

// Whether a layer's routed products run on the tensor cores: IQ banks (f32 activations under
// every policy), Q4_K under the f32 policy, MXFP4 banks whose weights are exact in f16 (f32, or
// Q8_0 rounded activations); SiLU or the clamped SwiGLU; piles large enough on average.
static bool mma_layer(const cwx_ctx* c, const cwx_moe_layer* L, int T) {
    if (!c || c->mma_min_pile <= 0) return false;
    if (L->act != CWX_ACT_SILU && L->act != CWX_ACT_CLAMPED_SWIGLU) return false;
    const int64_t pile = ((int64_t)T * L->top_k + L->n_experts - 1) / L->n_experts;
    if (pile < c->mma_min_pile) return false;
    const cwx_bank* bs[3] = {L->gate, L->up, L->down};
    for (const cwx_bank* b : bs) {
        const int f = b->L.fmt;
        // Q4_K only with f32 activations (its Q8_K codes carry a per-piece, per-token scale)
        if (!iq_format(f) && !(f == F_Q4_K && act_mode_of(b, L->act_mode) == AM_F32) && !(f == F_MXFP4 && b->mx_f16))
            return false;
    }
    if (L->gate->L.fmt != L->up->L.fmt) return false;
    // whole 256-column pieces, or (MXFP4) a tail of whole 64-column stages; 64-row tiles
    const int kq = L->gate->L.fmt == F_MXFP4 ? 64 : 256, kd = L->down->L.fmt == F_MXFP4 ? 64 : 256;
    return L->hidden % kq == 0 && L->inter % kd == 0 && L->hidden % 64 == 0 && L->inter % 64 == 0;
}

static int validate_layer(const cwx_moe_layer* L) {
    if (!L) return fail(CWX_EINVAL, "cwx_moe_forward: null layer");
    if (!L->router_w || !L->gate || !L->up || !L->down) return fail(CWX_EINVAL, "cwx_moe_forward: missing router or expert bank");
    if (L->top_k < 1 || L->top_k > 16 || L->top_k > L->n_experts)
        return fail(CWX_EINVAL, "cwx_moe_forward: top_k %d out of range (1..16, <= experts)", L->top_k);
    if (L->n_experts < 1 || L->n_experts > 1024) return fail(CWX_EUNSUPPORTED, "cwx_moe_forward: %d experts (max 1024)", L->n_experts);
    const Layout &g = L->gate->L, &u = L->up->L, &d = L->down->L;
    if (g.n != L->inter || g.k != L->hidden || u.n != L->inter || u.k != L->hidden || d.n != L->hidden || d.k != L->inter)
        return fail(CWX_EINVAL, "cwx_moe_forward: bank shapes do not match hidden=%d inter=%d", L->hidden, L->inter);
    if (g.n_experts != L->n_experts || u.n_experts != L->n_experts || d.n_experts != L->n_experts)
        return fail(CWX_EINVAL, "cwx_moe_forward: banks hold a different number of experts than %d", L->n_experts);
    if (L->hidden % 64 || L->inter % 64) return fail(CWX_EUNSUPPORTED, "cwx_moe_forward: hidden and inter must be multiples of 64");
    if (act_mode_of(L->gate, L->act_mode) != act_mode_of(L->up, L->act_mode))
        return fail(CWX_EUNSUPPORTED, "cwx_moe_forward: gate and up need different activation quantisation");
    if (L->sh_gate || L->sh_up || L->sh_down) {
        if (!L->sh_gate || !L->sh_up || !L->sh_down || !L->sh_gate_inp)
            return fail(CWX_EINVAL, "cwx_moe_forward: incomplete shared expert");
        const Layout &sg = L->sh_gate->L, &su = L->sh_up->L, &sd = L->sh_down->L;
        if (sg.k != L->hidden || su.k != L->hidden || sg.n != su.n || sd.n != L->hidden || sd.k != sg.n ||
            sg.n_experts != 1 || su.n_experts != 1 || sd.n_experts != 1)
            return fail(CWX_EINVAL, "cwx_moe_forward: shared expert shapes do not match");
        if (sg.n % 64) return fail(CWX_EUNSUPPORTED, "cwx_moe_forward: shared inter must be a multiple of 64");
        if (act_mode_of(L->sh_gate, L->act_mode) != act_mode_of(L->sh_up, L->act_mode))
            return fail(CWX_EUNSUPPORTED, "cwx_moe_forward: shared gate and up need different activation quantisation");
    }
    if (L->act != CWX_ACT_SILU && L->act != CWX_ACT_CLAMPED_SWIGLU) return fail(CWX_EINVAL, "cwx_moe_forward: unknown act %d", L->act);
    return CWX_OK;
}

static void plan_layer(const cwx_moe_layer* L, int T, int mma, uint8_t* base, LayerPlan* p) {
    p->H = L->hidden;
    p->E = L->n_experts;
    p->K = L->top_k;
    p->I = L->inter;
    p->Is = L->sh_gate ? (int)L->sh_gate->L.n : 0;
    p->T = T;
    p->xrows = T;
    p->rowmap = nullptr;
    p->mgu = act_mode_of(L->gate, L->act_mode);
    p->md = act_mode_of(L->down, L->act_mode);
    p->msgu = L->sh_gate ? act_mode_of(L->sh_gate, L->act_mode) : -1;
    p->msd = L->sh_down ? act_mode_of(L->sh_down, L->act_mode) : -1;
    const int64_t n = (int64_t)T * p->K;
    Carve c{base, 0};
    p->logits = c.take<float>((size_t)T * p->E);
    p->sgate = c.take<float>((size_t)T + 1);
    p->ids = c.take<uint32_t>((size_t)n + 1);
    p->w = c.take<float>((size_t)n + 1);
    p->heads = c.take<uint32_t>((size_t)3 * p->E);
    p->pairs = c.take<uint32_t>((size_t)n + 1);
    p->used3 = c.take<uint32_t>((size_t)3 * p->E);
    p->n_used = c.take<uint32_t>(4);
    p->perm = c.take<uint32_t>(perm_scratch_bytes(n, p->E) / 4);
    const int sh_mma = mma && shared_mma_ok(L) ? 1 : 0;
    for (int m = 0; m < 3; ++m) {
        const bool need = (m == p->mgu && !mma) || (m == p->msgu && !sh_mma);
        p->xpk[m] = need ? c.take<uint8_t>((size_t)(T * packed_row_bytes(p->H))) : nullptr;
    }
    const size_t nr = mma ? 0 : (size_t)n;  // the tensor-core products write h directly
    p->g = c.take<float>(nr * p->I);
    p->u = c.take<float>(nr * p->I);
    const size_t ns = sh_mma ? 0 : (size_t)T;  // the tensor-core shared expert writes h directly
    p->gs = c.take<float>(ns * p->Is);
    p->us = c.take<float>(ns * p->Is);
    p->hpk = c.take<uint8_t>((size_t)(nr * packed_row_bytes(p->I)));
    p->hspk = c.take<uint8_t>((size_t)(ns * packed_row_bytes(p->Is)));
    p->y = c.take<float>((size_t)n * p->H);
    p->ys = c.take<float>((size_t)T * p->H);
    p->mma = mma;
    p->sh_mma = sh_mma;
    p->x16 = mma ? c.take<__half>((size_t)T * p->H) : nullptr;
    p->x16lo = mma && p->mgu == AM_Q8_0 ? c.take<__half>((size_t)T * p->H) : nullptr;
    p->h16 = mma ? c.take<__half>((size_t)n * p->I) : nullptr;
    p->hs16 = sh_mma ? c.take<__half>((size_t)T * p->Is) : nullptr;
    p->spairs = sh_mma ? c.take<uint32_t>((size_t)T + 1) : nullptr;
    p->sused3 = sh_mma ? c.take<uint32_t>(4) : nullptr;
    p->snused = sh_mma ? c.take<uint32_t>(4) : nullptr;
    p->bytes = c.off + 256;
}

static MatRef mref(const cwx_bank* b) { return MatRef{b ? b->d : nullptr, b ? b->L : Layout{}}; }

static GemvJob job(const cwx_bank* b, int shared, const uint8_t* act, int mode, int64_t k, int bdiv, float* out,
                   int64_t ostride, int split, const float* bias) {
    GemvJob j;
    j.m = mref(b);
    j.qint = mode == AM_Q8_K;
    j.shared = shared;
    j.b = act;
    j.bstride = packed_row_bytes(k);
    j.bdiv = bdiv;
    j.rowmap = nullptr;
    j.out = out;
    j.ostride = ostride;
    j.split = split;
    j.bias = bias;
    j.exact = b && b->mx_wide;
    return j;
}

static PrepArgs prep(const float* src, const float* up, int64_t R, int64_t K, int mode, uint8_t* out) {
    PrepArgs a;
    memset(&a, 0, sizeof a);
    a.src = src;
    a.up = up;
    a.R = R;
    a.K = K;
    a.mode = mode;
    a.act = CWX_ACT_SILU;
    a.out = out;
    return a;
}

}  // namespace cwx

using namespace cwx;

extern "C" const char* cwx_last_error(void) { return g_err; }
extern "C" int cwx_version(void) { return 1; }

extern "C" int cwx_ctx_create(int device, cwx_ctx** out) {
    if (!out) return fail(CWX_EINVAL, "cwx_ctx_create: null output pointer");
    *out = nullptr;
    int ndev = 0;
    CWX_CUDA(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return fail(CWX_EINVAL, "cwx_ctx_create: device %d of %d", device, ndev);
    CWX_CUDA(cudaSetDevice(device));
    cwx_ctx* c = new cwx_ctx();
    memset(c, 0, sizeof *c);
    c->device = device;
    c->mma_min_pile = 32;
    c->fused_max_tokens = DL_MAX_T;
    c->prof = new ProfLog();
    cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device);
    cudaError_t e = cudaMalloc(&c->d_err, 64);
    if (e == cudaSuccess) e = cudaMemset(c->d_err, 0, 64);
    if (e != cudaSuccess) {
        delete static_cast<ProfLog*>(c->prof);
        delete c;
        return cuda_fail(e, "cwx_ctx_create");
    }
    *out = c;
    return CWX_OK;
}

extern "C" int cwx_ctx_reset_profile(cwx_ctx* c) {
    if (!c) return fail(CWX_EINVAL, "cwx_ctx_reset_profile: null context");
    ProfLog* log = static_cast<ProfLog*>(c->prof);
    if (!log) return CWX_OK;
    cudaSetDevice(c->device);
    for (const ProfEvent& e : *log) {
        cudaEventDestroy(e.a);
        cudaEventDestroy(e.b);
    }
    log->clear();
    return CWX_OK;
}

extern "C" int cwx_ctx_destroy(cwx_ctx* c) {
    if (!c) return CWX_OK;
    cudaSetDevice(c->device);
    if (c->ws) cudaFree(c->ws);
    if (c->d_err) cudaFree(c->d_err);
    if (c->d_iq3s_map) cudaFree(c->d_iq3s_map);
    if (c->d_iq2s_map) cudaFree(c->d_iq2s_map);
    if (c->d_iq3xxs_map) cudaFree(c->d_iq3xxs_map);
    if (c->d_iq2xxs_map) cudaFree(c->d_iq2xxs_map);
    if (c->side) cudaStreamDestroy(c->side);
    if (c->ev_fork) cudaEventDestroy(c->ev_fork);
    if (c->ev_join) cudaEventDestroy(c->ev_join);
    cwx_ctx_reset_profile(c);
    delete static_cast<ProfLog*>(c->prof);
    delete c;
    return CWX_OK;
}

extern "C" int cwx_ctx_set_mma_min_pile(cwx_ctx* c, int min_pile) {
    if (!c) return fail(CWX_EINVAL, "cwx_ctx_set_mma_min_pile: null context");
    if (min_pile < 0) return fail(CWX_EINVAL, "cwx_ctx_set_mma_min_pile: %d is negative", min_pile);
    c->mma_min_pile = min_pile;
    return CWX_OK;
}

extern "C" int cwx_ctx_set_fused_decode(cwx_ctx* c, int max_tokens) {
    if (!c) return fail(CWX_EINVAL, "cwx_ctx_set_fused_decode: null context");
    if (max_tokens < 0) return fail(CWX_EINVAL, "cwx_ctx_set_fused_decode: %d is negative", max_tokens);
    c->fused_max_tokens = max_tokens;
    return CWX_OK;
}

extern "C" int cwx_ctx_set_profiling(cwx_ctx* c, int enabled) {
    if (!c) return fail(CWX_EINVAL, "cwx_ctx_set_profiling: null context");
    c->profiling = enabled ? 1 : 0;
    return CWX_OK;
}

extern "C" int cwx_ctx_read_profile(cwx_ctx* c, double* ms, int64_t* count) {
    if (!c) return fail(CWX_EINVAL, "cwx_ctx_read_profile: null context");
    CWX_CUDA(cudaSetDevice(c->device));
    CWX_CUDA(cudaDeviceSynchronize());
    for (const ProfEvent& e : *static_cast<ProfLog*>(c->prof)) {
        float t = 0.f;
        CWX_CUDA(cudaEventElapsedTime(&t, e.a, e.b));
        if (ms) ms[e.phase] += t;
        if (count) count[e.phase] += 1;
    }
    return CWX_OK;
}

extern "C" int64_t cwx_ctx_launches(const cwx_ctx* c) { return c ? c->launches : 0; }

extern "C" int cwx_ctx_status(cwx_ctx* c, void* stream) {
    if (!c) return fail(CWX_EINVAL, "cwx_ctx_status: null context");
    CWX_CUDA(cudaSetDevice(c->device));
    CWX_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    int h = 0;
    CWX_CUDA(cudaMemcpy(&h, c->d_err, 4, cudaMemcpyDeviceToHost));
    if (h == DE_OK) return CWX_OK;
    CWX_CUDA(cudaMemset(c->d_err, 0, 64));  // (a timed-out grid barrier leaves its counter off step)
    if (h == DE_TIMEOUT) return fail(CWX_ETIMEOUT, "a device-side wait gave up (bulk copy did not complete)");
    if (h == DE_BAD_ID) return fail(CWX_EDEVICE, "an expert id was out of range");
    if (h == DE_SHAPE) return fail(CWX_EDEVICE, "a length read on the device was out of range (attention cache row)");
    return fail(CWX_EDEVICE, "device error %d", h);
}

// One bounded wait on an mbarrier that nothing completes (the failure path of every kernel's
// waits): the wait gives up after limit_ns, records DE_TIMEOUT and the kernel returns.
__global__ void k_wait_check(int* err, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_wait(&bar, 0, err, limit_ns);
    }
}

extern "C" int cwx_ctx_check_wait(cwx_ctx* c, int32_t limit_us, void* stream) {
    if (!c) return fail(CWX_EINVAL, "cwx_ctx_check_wait: null context");
    if (limit_us < 1 || limit_us > 1000000) return fail(CWX_EINVAL, "cwx_ctx_check_wait: limit %d us", limit_us);
    CWX_CUDA(cudaSetDevice(c->device));
    k_wait_check<<<1, 32, 0, (cudaStream_t)stream>>>(c->d_err, (uint64_t)limit_us * 1000);
    CWX_CUDA(cudaGetLastError());
    c->launches += 1;
    return CWX_OK;
}

extern "C" int cwx_ctx_reserve(cwx_ctx* c, const void* layer, int32_t tokens) {
    if (!c || !layer) return fail(CWX_EINVAL, "cwx_ctx_reserve: null argument");
    const cwx_moe_layer* L = (const cwx_moe_layer*)layer;
    int rc = validate_layer(L);
    if (rc) return rc;
    CWX_CUDA(cudaSetDevice(c->device));
    // the larger of the two plans (tensor-core products or not), so any batch up to `tokens` fits
    LayerPlan p, q;
    plan_layer(L, tokens, 0, nullptr, &p);
    plan_layer(L, tokens, mma_layer(c, L, tokens) ? 1 : 0, nullptr, &q);
    return ensure_ws(c, p.bytes > q.bytes ? p.bytes : q.bytes, 0);
}

extern "C" int cwx_route(cwx_ctx* c, const float* logits, int32_t T, int32_t E, int32_t K, int32_t norm, uint32_t* ids,
                         float* w, void* stream) {
    if (!c || (!logits && T) || (!ids && T) || (!w && T)) return fail(CWX_EINVAL, "cwx_route: null argument");
    if (T < 0 || E < 1 || E > 1024) return fail(CWX_EINVAL, "cwx_route: %d experts (1..1024)", E);
    if (K < 1 || K > 16 || K > E) return fail(CWX_EINVAL, "cwx_route: top_k %d (1..16, <= experts)", K);
    CWX_CUDA(cudaSetDevice(c->device));
    c->launches += T > 0 ? 1 : 0;
    return launch_route(logits, T, E, K, norm, ids, w, nullptr, nullptr, 0, nullptr, (cudaStream_t)stream);
}

extern "C" int cwx_permute(cwx_ctx* c, const uint32_t* ids, int32_t T, int32_t K, int32_t E, uint32_t* pairs,
                           uint32_t* heads, void* stream) {
    if (!c || (!ids && T) || !heads || (!pairs && T)) return fail(CWX_EINVAL, "cwx_permute: null argument");
    if (T < 0 || K < 1 || E < 1 || E > 12288) return fail(CWX_EINVAL, "cwx_permute: bad sizes");
    CWX_CUDA(cudaSetDevice(c->device));
    cudaStream_t st = (cudaStream_t)stream;
    const int64_t n = (int64_t)T * K;
    Carve cv{nullptr, 0};
    cv.take<uint32_t>((size_t)3 * E);
    cv.take<uint32_t>(4);
    cv.take<uint32_t>(perm_scratch_bytes(n, E) / 4);
    int rc = ensure_ws(c, cv.off + 256, st);
    if (rc) return rc;
    Carve w{c->ws, 0};
    uint32_t* used3 = w.take<uint32_t>((size_t)3 * E);
    uint32_t* n_used = w.take<uint32_t>(4);
    uint32_t* scratch = w.take<uint32_t>(perm_scratch_bytes(n, E) / 4);
    c->launches += perm_launches(n, E);
    return launch_permute(ids, n, E, pairs, heads, used3, n_used, scratch, c->d_err, st);
}

extern "C" int cwx_expert_matmul(cwx_ctx* c, const cwx_bank* bank, const float* x, int32_t rows_per_expert,
                                 const uint32_t* ids, int32_t tokens, int32_t nei0, int32_t act_mode, float* out,
                                 void* stream) {
    if (!c || !bank || (tokens && (!x || !ids || !out))) return fail(CWX_EINVAL, "cwx_expert_matmul: null argument");
    if (tokens < 0 || nei0 < 1) return fail(CWX_EINVAL, "cwx_expert_matmul: bad sizes tokens=%d nei0=%d", tokens, nei0);
    if (bank->L.k % 64 || bank->L.n % 16)
        return fail(CWX_EUNSUPPORTED, "cwx_expert_matmul: k must be a multiple of 64 and n of 16 (k=%lld n=%lld)",
                    (long long)bank->L.k, (long long)bank->L.n);
    if (bank->L.n_experts > 12288) return fail(CWX_EUNSUPPORTED, "cwx_expert_matmul: too many experts");
    if (tokens == 0) return CWX_OK;
    CWX_CUDA(cudaSetDevice(c->device));
    cudaStream_t st = (cudaStream_t)stream;
    const int E = (int)bank->L.n_experts;
    const int64_t n = (int64_t)tokens * nei0;
    const int64_t xrows = rows_per_expert ? n : tokens;
    const int64_t K = bank->L.k;
    const int mode = act_mode_of(bank, act_mode);
    Carve cv{nullptr, 0};
    cv.take<uint32_t>((size_t)n);
    cv.take<uint32_t>((size_t)3 * E);
    cv.take<uint32_t>((size_t)3 * E);
    cv.take<uint32_t>(4);
    cv.take<uint32_t>(perm_scratch_bytes(n, E) / 4);
    cv.take<uint8_t>((size_t)(xrows * packed_row_bytes(K)));
    int rc = ensure_ws(c, cv.off + 256, st);
    if (rc) return rc;
    Carve w{c->ws, 0};
    uint32_t* pairs = w.take<uint32_t>((size_t)n);
    uint32_t* heads = w.take<uint32_t>((size_t)3 * E);
    uint32_t* used3 = w.take<uint32_t>((size_t)3 * E);
    uint32_t* n_used = w.take<uint32_t>(4);
    uint32_t* scratch = w.take<uint32_t>(perm_scratch_bytes(n, E) / 4);
    uint8_t* xpk = w.take<uint8_t>((size_t)(xrows * packed_row_bytes(K)));
    if ((rc = launch_permute(ids, n, E, pairs, heads, used3, n_used, scratch, c->d_err, st))) return rc;
    if ((rc = launch_prep(prep(x, nullptr, xrows, K, mode, xpk), st))) return rc;
    GemvArgs a;
    memset(&a, 0, sizeof a);
    a.njobs = 1;
    a.job[0] = job(bank, 0, xpk, mode, K, rows_per_expert ? 1 : nei0, out, bank->L.n, 0, nullptr);
    a.pairs = pairs;
    a.used3 = used3;
    a.n_used = n_used;
    a.tok_est = tokens;
    a.pile_est = (int)((n + E - 1) / E);
    a.err = c->d_err;
    c->launches += perm_launches(n, E) + 2;
    return launch_gemv(a, n < E ? n : E, c->device, c->sm_count, st);
}

// Gate/up, activation and down products on the grouped mma.sync products (every format, any
// batch; the shared expert in the same launches).
// x's packed activation rows in every mode the layer's products take (one launch).
static int prep_x(cwx_ctx* c, const cwx_moe_args* A, const LayerPlan& p, cudaStream_t st) {
    PhaseTimer t(c, st, CWX_PHASE_PREP);
    PrepArgs px[2];
    int nx = 0;
    for (int m = 0; m < 3; ++m)
        if (p.xpk[m]) px[nx++] = prep(A->x, nullptr, p.xrows, p.H, m, p.xpk[m]);
    int rc = launch_prep2(px, nx, st);
    if (rc) return rc;
    c->launches += 1;
    t.end();
    return CWX_OK;
}

// The context's side stream and its fork/join events (created on first use, on the context's
// device); work forked onto it is captured into a graph like the main stream's.
static int ctx_side(cwx_ctx* c) {
    if (c->side) return CWX_OK;
    CWX_CUDA(cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking));
    CWX_CUDA(cudaEventCreateWithFlags(&c->ev_fork, cudaEventDisableTiming));
    CWX_CUDA(cudaEventCreateWithFlags(&c->ev_join, cudaEventDisableTiming));
    return CWX_OK;
}

// prepped: x's rows were already packed (forked alongside the routing).
static int moe_gemv(cwx_ctx* c, const cwx_moe_layer* L, const cwx_moe_args* A, const LayerPlan& p, cudaStream_t st,
                    bool prepped = false) {
    const int T = p.T, H = p.H, E = p.E, K = p.K, I = p.I, Is = p.Is;
    const int64_t n = (int64_t)T * K;
    const bool shared = L->sh_gate != nullptr;
    int rc;
    const int64_t used_max = n < E ? n : E;
    if (!prepped && (rc = prep_x(c, A, p, st))) return rc;
    // gate and up: routed piles and the shared expert, four matrix jobs in one launch. A product
    // whose result is re-quantised downstream (the down matrix takes Q8 activations) carries its
    // weights to ~22 bits, so the hidden state matches the CPU path closely enough that its Q8
    // codes do not flip at rounding boundaries.
    {
        GemvArgs a;
        memset(&a, 0, sizeof a);
        const int split_r = p.md != AM_F32, split_s = shared && p.msd != AM_F32;
        a.job[a.njobs++] = job(L->gate, 0, p.xpk[p.mgu], p.mgu, H, K, p.g, I, split_r, nullptr);
        a.job[a.njobs++] = job(L->up, 0, p.xpk[p.mgu], p.mgu, H, K, p.u, I, split_r, nullptr);
        a.job[0].rowmap = a.job[1].rowmap = p.rowmap;
        if (shared) {
            a.job[a.njobs++] = job(L->sh_gate, 1, p.xpk[p.msgu], p.msgu, H, 1, p.gs, Is, split_s, nullptr);
            a.job[a.njobs++] = job(L->sh_up, 1, p.xpk[p.msgu], p.msgu, H, 1, p.us, Is, split_s, nullptr);
        }
        a.pairs = p.pairs;
        a.used3 = p.used3;
        a.n_used = p.n_used;
        a.s_count = T;
        a.tok_est = T;
        a.pile_est = (int)((n + E - 1) / E);
        a.err = c->d_err;
        PhaseTimer t(c, st, CWX_PHASE_GATE_UP);
        if ((rc = launch_gemv(a, used_max, c->device, c->sm_count, st))) return rc;
        t.end();
    }
    {
        PhaseTimer t(c, st, CWX_PHASE_PREP);
        PrepArgs pa = prep(p.g, p.u, n, I, p.md, p.hpk);
        pa.act = L->act;
        pa.alpha = L->alpha;
        pa.limit = L->limit;
        pa.gate_b = L->gate_b;
        pa.up_b = L->up_b;
        pa.ids = p.ids;
        PrepArgs ph[2] = {pa, shared ? prep(p.gs, p.us, T, Is, p.msd, p.hspk) : PrepArgs{}};
        if ((rc = launch_prep2(ph, shared ? 2 : 1, st))) return rc;
        t.end();
    }
    c->launches += 2;
    {
        GemvArgs d;
        memset(&d, 0, sizeof d);
        d.job[d.njobs++] = job(L->down, 0, p.hpk, p.md, I, 1, p.y, H, 0,
                               L->act == CWX_ACT_CLAMPED_SWIGLU ? L->down_b : nullptr);
        if (shared) d.job[d.njobs++] = job(L->sh_down, 1, p.hspk, p.msd, Is, 1, p.ys, H, 0, nullptr);
        d.pairs = p.pairs;
        d.used3 = p.used3;
        d.n_used = p.n_used;
        d.s_count = T;
        d.tok_est = T;
        d.pile_est = (int)((n + E - 1) / E);
        d.err = c->d_err;
        PhaseTimer t(c, st, CWX_PHASE_DOWN);
        if ((rc = launch_gemv(d, used_max, c->device, c->sm_count, st))) return rc;
        t.end();
    }
    c->launches += 1;
    return CWX_OK;
}

// The shared expert's products alone (the routed ones run on the tensor cores).
static int shared_gemv(cwx_ctx* c, const cwx_moe_layer* L, const LayerPlan& p, int down, cudaStream_t st) {
    const int T = p.T, H = p.H, Is = p.Is;
    GemvArgs a;
    memset(&a, 0, sizeof a);
    const int split_s = p.msd != AM_F32;
    if (!down) {
        a.job[a.njobs++] = job(L->sh_gate, 1, p.xpk[p.msgu], p.msgu, H, 1, p.gs, Is, split_s, nullptr);
        a.job[a.njobs++] = job(L->sh_up, 1, p.xpk[p.msgu], p.msgu, H, 1, p.us, Is, split_s, nullptr);
    } else {
        a.job[a.njobs++] = job(L->sh_down, 1, p.hspk, p.msd, Is, 1, p.ys, H, 0, nullptr);
    }
    a.pairs = p.pairs;
    a.used3 = p.used3;
    a.n_used = p.n_used;
    a.s_count = T;
    a.tok_est = T;
    a.pile_est = T;
    a.err = c->d_err;
    return launch_gemv(a, 0, c->device, c->sm_count, st);
}

// Routed products on the tensor cores (mma.cu): x as f16 rows; fused gate/up writing h = silu(g)
// * u as f16 rows per pick; down from those rows. The shared expert stays on the mma.sync
// products, one launch per stage.
static int moe_mma(cwx_ctx* c, const cwx_moe_layer* L, const cwx_moe_args* A, const LayerPlan& p, cudaStream_t st) {
    const int T = p.T, H = p.H, K = p.K, I = p.I, Is = p.Is;
    const bool shared = L->sh_gate != nullptr;
    int rc;
    {
        PhaseTimer t(c, st, CWX_PHASE_PREP);
        // (Q8_0 policy, MXFP4: the rows through Q8_0 first, as the reference's vec_dot_type, kept
        // exactly as hi + lo: h goes through Q8_0 again, whose rounding an f16-only product would
        // flip for some elements)
        if ((rc = p.mgu == AM_Q8_0 ? launch_f16rows_q80(A->x, p.xrows * H, p.x16, p.x16lo, st)
                                   : launch_f16rows(A->x, p.xrows * H, p.x16, st)))
            return rc;
        c->launches += 1;
        if (shared && !p.sh_mma) {
            if ((rc = launch_prep(prep(A->x, nullptr, T, H, p.msgu, p.xpk[p.msgu]), st))) return rc;
            c->launches += 1;
        }
        if (p.sh_mma) {
            if ((rc = launch_all_tokens(p.spairs, T, p.sused3, p.snused, st))) return rc;
            c->launches += 1;
        }
        t.end();
    }
    MmaArgs m;
    memset(&m, 0, sizeof m);
    m.pairs = p.pairs;
    m.used3 = p.used3;
    m.n_used = p.n_used;
    m.err = c->d_err;
    {
        PhaseTimer t(c, st, CWX_PHASE_GATE_UP);
        MmaArgs g = m;
        g.a0 = mref(L->gate);
        g.a1 = mref(L->up);
        g.fused = 1;
        g.b = reinterpret_cast<const uint8_t*>(p.x16);
        g.blo = reinterpret_cast<const uint8_t*>(p.x16lo);
        g.bstride = (int64_t)H * 2;
        g.bdiv = K;
        g.rowmap = p.rowmap;
        g.brows = p.xrows;
        g.hout = p.h16;
        g.ostride = I;
        g.act = L->act;
        g.alpha = L->alpha;
        g.limit = L->limit;
        if (L->act == CWX_ACT_CLAMPED_SWIGLU) {
            g.gate_b = L->gate_b;
            g.up_b = L->up_b;
        }
        g.h_q80 = p.md == AM_Q8_0;
        if ((rc = launch_mma(g, c->device, c->sm_count, st))) return rc;
        c->launches += 1;
        if (p.sh_mma) {
            MmaArgs sg = g;
            sg.a0 = mref(L->sh_gate);
            sg.a1 = mref(L->sh_up);
            sg.pairs = p.spairs;
            sg.used3 = p.sused3;
            sg.n_used = p.snused;
            sg.bdiv = 1;
            sg.hout = p.hs16;
            sg.ostride = Is;
            sg.blo = nullptr;
            sg.act = CWX_ACT_SILU;
            sg.gate_b = sg.up_b = nullptr;
            sg.h_q80 = 0;
            if ((rc = launch_mma(sg, c->device, c->sm_count, st))) return rc;
            c->launches += 1;
        } else if (shared) {
            if ((rc = shared_gemv(c, L, p, 0, st))) return rc;
            c->launches += 1;
        }
        t.end();
    }
    if (shared && !p.sh_mma) {
        PhaseTimer t(c, st, CWX_PHASE_PREP);
        if ((rc = launch_prep(prep(p.gs, p.us, T, Is, p.msd, p.hspk), st))) return rc;
        c->launches += 1;
        t.end();
    }
    {
        PhaseTimer t(c, st, CWX_PHASE_DOWN);
        MmaArgs d = m;
        d.a0 = mref(L->down);
        d.fused = 0;
        d.b = reinterpret_cast<const uint8_t*>(p.h16);
        d.blo = nullptr;
        d.bstride = (int64_t)I * 2;
        d.brows = (int64_t)T * K;
        d.bdiv = 1;
        d.out = p.y;
        d.ostride = H;
        d.bias = L->act == CWX_ACT_CLAMPED_SWIGLU ? L->down_b : nullptr;
        if ((rc = launch_mma(d, c->device, c->sm_count, st))) return rc;
        c->launches += 1;
        if (p.sh_mma) {
            MmaArgs sd = d;
            sd.a0 = mref(L->sh_down);
            sd.pairs = p.spairs;
            sd.used3 = p.sused3;
            sd.n_used = p.snused;
            sd.b = reinterpret_cast<const uint8_t*>(p.hs16);
            sd.bstride = (int64_t)Is * 2;
            sd.brows = T;
            sd.out = p.ys;
            sd.ostride = H;
            sd.bias = nullptr;
            if ((rc = launch_mma(sd, c->device, c->sm_count, st))) return rc;
            c->launches += 1;
        } else if (shared) {
            if ((rc = shared_gemv(c, L, p, 1, st))) return rc;
            c->launches += 1;
        }
        t.end();
    }
    return CWX_OK;
}

// Whether a call takes the fused decode layer (decode_layer.cu): a small batch of a layer whose
// banks and shapes it handles.
static bool fused_layer(const cwx_ctx* c, const cwx_moe_layer* L, const cwx_moe_args* A, int T) {
    if (c->fused_max_tokens <= 0 || T < 1 || T > c->fused_max_tokens || T > DL_MAX_T) return false;
    if ((int64_t)T * L->top_k > DL_MAX_PICKS || L->act != CWX_ACT_SILU) return false;
    if (L->n_experts > DL_MAX_E || L->hidden % 256 || L->hidden > DL_MAX_H || L->inter % 256 ||
        L->inter > DL_MAX_I)
        return false;
    if (L->gate->L.fmt != L->up->L.fmt || !decode_fused_formats(L->gate->L.fmt, L->down->L.fmt)) return false;
    if ((((uintptr_t)A->x) | ((uintptr_t)L->router_w)) & 15) return false;
    if (L->sh_gate) {
        const Layout &g = L->sh_gate->L, &u = L->sh_up->L, &d = L->sh_down->L;
        if (g.fmt != F_Q4_K || u.fmt != F_Q4_K || d.fmt != F_Q4_K || g.n % 256 || g.n > DL_MAX_I) return false;
        if (act_mode_of(L->sh_gate, L->act_mode) != act_mode_of(L->sh_down, L->act_mode)) return false;
    }
    return true;
}

// The whole layer in one launch of the fused decode layer.
static int moe_fused(cwx_ctx* c, const cwx_moe_layer* L, const cwx_moe_args* A, cudaStream_t st) {
    const int T = A->tokens, H = L->hidden, E = L->n_experts, K = L->top_k, I = L->inter;
    const int Is = L->sh_gate ? (int)L->sh_gate->L.n : 0;
    const bool qint = L->sh_gate && act_mode_of(L->sh_gate, L->act_mode) == AM_Q8_K;
    (void)H;
    Carve sz{nullptr, 0};
    for (int pass = 0; pass < 2; ++pass) {
        if (pass) {
            int rc = ensure_ws(c, sz.off + 256, st);
            if (rc) return rc;
        }
        Carve w{pass ? c->ws : nullptr, 0};
        DecodeArgs a;
        memset(&a, 0, sizeof a);
        a.logits = w.take<float>((size_t)T * (E + 1));  // + the shared expert's gates
        a.hpk = w.take<uint8_t>((size_t)((int64_t)T * K * (I / 256) * 512));
        a.hs = Is ? w.take<float>((size_t)T * Is) : nullptr;
        if (!pass) {
            sz = w;
            continue;
        }
        a.x = A->x;
        a.residual = A->residual;
        a.out = A->out;
        a.norm_w = A->norm_w;
        a.norm_eps = A->norm_eps;
        a.norm_out = A->norm_out;
        a.norm_vec = ((((uintptr_t)A->out) | ((uintptr_t)A->norm_w) | ((uintptr_t)A->norm_out)) & 15) == 0;
        a.T = T;
        a.H = H;
        a.E = E;
        a.K = K;
        a.I = I;
        a.Is = Is;
        a.norm = L->norm_topk_prob;
        a.router_w = L->router_w;
        a.router_b = L->router_b;
        a.gate = mref(L->gate);
        a.up = mref(L->up);
        a.down = mref(L->down);
        if (L->sh_gate) {
            a.sg = mref(L->sh_gate);
            a.su = mref(L->sh_up);
            a.sd = mref(L->sh_down);
            a.sg_inp = L->sh_gate_inp;
        }
        a.sh_qint = qint ? 1 : 0;
        a.err = c->d_err;
        a.bar = reinterpret_cast<unsigned long long*>(c->d_err + 8);
        a.ids_out = A->ids_out;
        a.w_out = A->weights_out;
        a.pairs_out = A->pairs_out;
        a.heads_out = A->heads_out;
        PhaseTimer t(c, st, CWX_PHASE_DECODE_FUSED);
        int rc = launch_decode_layer(a, c->device, c->sm_count, st);
        if (rc) return rc;
        t.end();
        c->launches += 1;
    }
    return CWX_OK;
}

extern "C" int cwx_moe_forward(cwx_ctx* c, const cwx_moe_layer* L, const cwx_moe_args* A, void* stream) {
    if (!c || !A) return fail(CWX_EINVAL, "cwx_moe_forward: null argument");
    int rc = validate_layer(L);
    if (rc) return rc;
    const int T = A->tokens;
    if (T < 0) return fail(CWX_EINVAL, "cwx_moe_forward: tokens %d", T);
    if (T == 0) return CWX_OK;
    if (!A->x || !A->out) return fail(CWX_EINVAL, "cwx_moe_forward: null x or out");
    if (A->norm_w && (!A->norm_out || A->norm_out == A->out || A->norm_out == A->x || A->norm_out == A->residual))
        return fail(CWX_EINVAL, "cwx_moe_forward: norm_w needs a norm_out buffer of its own");
    CWX_CUDA(cudaSetDevice(c->device));
    cudaStream_t st = (cudaStream_t)stream;
    if (fused_layer(c, L, A, T)) return moe_fused(c, L, A, st);
    LayerPlan p;
    const int mma = mma_layer(c, L, T) ? 1 : 0;
    plan_layer(L, T, mma, nullptr, &p);
    if ((rc = ensure_ws(c, p.bytes, st))) return rc;
    plan_layer(L, T, mma, c->ws, &p);
    const int H = p.H, E = p.E, K = p.K;
    const int64_t n = (int64_t)T * K;
    const bool shared = L->sh_gate != nullptr;

    // x's activation rows depend only on x: packed on the side stream while the routing runs
    const bool fork = !p.mma;
    if (fork) {
        if ((rc = ctx_side(c))) return rc;
        CWX_CUDA(cudaEventRecord(c->ev_fork, st));
        CWX_CUDA(cudaStreamWaitEvent(c->side, c->ev_fork, 0));
        if ((rc = prep_x(c, A, p, c->side))) return rc;
        CWX_CUDA(cudaEventRecord(c->ev_join, c->side));
    }
    {
        PhaseTimer t(c, st, CWX_PHASE_ROUTER);
        if ((rc = launch_router(A->x, L->router_w, L->router_b, T, H, E, p.logits, st))) return rc;
        t.end();
    }
    {
        PhaseTimer t(c, st, CWX_PHASE_ROUTE);
        if ((rc = launch_route(p.logits, T, E, K, L->norm_topk_prob, p.ids, p.w, A->x,
                               shared ? L->sh_gate_inp : nullptr, H, shared ? p.sgate : nullptr, st)))
            return rc;
        t.end();
    }
    {
        PhaseTimer t(c, st, CWX_PHASE_PILES);
        if ((rc = launch_permute(p.ids, n, E, p.pairs, p.heads, p.used3, p.n_used, p.perm, c->d_err, st))) return rc;
        t.end();
    }
    c->launches += 2 + perm_launches(n, E);
    if (fork) CWX_CUDA(cudaStreamWaitEvent(st, c->ev_join, 0));
    if (p.mma) {
        if ((rc = moe_mma(c, L, A, p, st))) return rc;
    } else {
        if ((rc = moe_gemv(c, L, A, p, st, fork))) return rc;
    }
    {
        PhaseTimer t(c, st, CWX_PHASE_COMBINE);
        if (A->norm_w)
            rc = launch_combine_norm(p.y, p.w, T, K, H, shared ? p.ys : nullptr, p.sgate, A->residual, A->norm_w,
                                     A->norm_eps, A->out, A->norm_out, st);
        else
            rc = launch_combine(p.y, p.w, T, K, H, shared ? p.ys : nullptr, p.sgate, A->residual, A->out, st);
        if (rc) return rc;
        t.end();
    }
    c->launches += 1;

    if (A->ids_out) CWX_CUDA(cudaMemcpyAsync(A->ids_out, p.ids, n * 4, cudaMemcpyDeviceToDevice, st));
    if (A->weights_out) CWX_CUDA(cudaMemcpyAsync(A->weights_out, p.w, n * 4, cudaMemcpyDeviceToDevice, st));
    if (A->pairs_out) CWX_CUDA(cudaMemcpyAsync(A->pairs_out, p.pairs, n * 4, cudaMemcpyDeviceToDevice, st));
    if (A->heads_out) CWX_CUDA(cudaMemcpyAsync(A->heads_out, p.heads, (size_t)3 * E * 4, cudaMemcpyDeviceToDevice, st));
    return CWX_OK;
}

extern "C" int cwx_add_rms_norm(const float* a, const float* b, const float* c, const float* alpha, float eps,
                                int64_t rows, int32_t hidden, float* sum, float* out, void* stream) {
    if (!a || !b || !alpha || !sum || !out) return fail(CWX_EINVAL, "cwx_add_rms_norm: null argument");
    if (rows < 0 || hidden <= 0 || rows > INT32_MAX)
        return fail(CWX_EINVAL, "cwx_add_rms_norm: rows %lld, hidden %d", (long long)rows, hidden);
    if (out == a || out == b || (c && out == c) || out == sum)
        return fail(CWX_EINVAL, "cwx_add_rms_norm: out must be a buffer of its own");
    return launch_add_norm(a, b, c, alpha, eps, rows, hidden, sum, out, (cudaStream_t)stream);
}

// ---------------------------------------------------------------- expert parallelism
// The three per-rank steps of an expert-parallel layer; the caller moves the rows between them
// with two all-to-all exchanges (counts first, so every rank knows its receive sizes).

static int ep_check(const cwx_moe_layer* L, const cwx_ep_group* g, const char* who) {
    if (!L || !g) return fail(CWX_EINVAL, "%s: null layer or group", who);
    if (g->world < 1 || g->rank < 0 || g->rank >= g->world || g->experts_per_rank < 1)
        return fail(CWX_EINVAL, "%s: bad group (world %d, rank %d, %d experts per rank)", who, g->world, g->rank,
                    g->experts_per_rank);
    if ((int64_t)g->world * g->experts_per_rank != L->n_experts)
        return fail(CWX_EINVAL, "%s: %d ranks x %d experts do not cover n_experts=%d", who, g->world,
                    g->experts_per_rank, L->n_experts);
    if (!L->gate || !L->up || !L->down || L->gate->L.n_experts != g->experts_per_rank ||
        L->up->L.n_experts != g->experts_per_rank || L->down->L.n_experts != g->experts_per_rank)
        return fail(CWX_EINVAL, "%s: the banks must hold this rank's %d experts", who, g->experts_per_rank);
    return CWX_OK;
}

// Rows travel as f16 when the routed gate/up products read f16 activations anyway (IQ banks take
// f16 activations on both product paths), which halves the dispatch exchange at no change in the
// result; other formats get their f32 rows.
// f16 rows only where nothing downstream re-quantises: with a down matrix that takes Q8
// activations, the f16 rounding of x moves the hidden state across Q8 rounding boundaries.
static bool ep_rows_f16(const cwx_moe_layer* L) {
    const int g = L->gate->L.fmt, u = L->up->L.fmt;
    return iq_format(g) && iq_format(u) && act_mode_of(L->down, L->act_mode) == AM_F32;
}

extern "C" int cwx_ep_rows_f16(const cwx_moe_layer* L) { return L && L->gate && L->up && ep_rows_f16(L) ? 1 : 0; }

extern "C" int cwx_ep_dispatch(cwx_ctx* c, const cwx_moe_layer* L, const cwx_ep_group* g, const float* x,
                               int32_t tokens, uint32_t* ids, float* weights, float* sgate, int32_t* unit_of,
                               void* send_rows, int32_t* send_picks, int32_t* send_counts, void* stream) {
    if (!c) return fail(CWX_EINVAL, "cwx_ep_dispatch: null context");
    int rc = ep_check(L, g, "cwx_ep_dispatch");
    if (rc) return rc;
    if (!L->router_w || L->top_k < 1 || L->top_k > 16 || L->top_k > L->n_experts || L->n_experts > 1024)
        return fail(CWX_EINVAL, "cwx_ep_dispatch: router or top_k out of range");
    if (tokens < 0) return fail(CWX_EINVAL, "cwx_ep_dispatch: tokens %d", tokens);
    if (!send_counts || (tokens && (!x || !ids || !weights || !unit_of || !send_rows || !send_picks)))
        return fail(CWX_EINVAL, "cwx_ep_dispatch: null argument");
    if (L->hidden % 4 || ((uintptr_t)x & 15)) return fail(CWX_EINVAL, "cwx_ep_dispatch: x rows must be 16-byte aligned");
    const bool shared = L->sh_gate != nullptr;
    if (shared && tokens && !sgate) return fail(CWX_EINVAL, "cwx_ep_dispatch: the shared expert needs sgate");
    CWX_CUDA(cudaSetDevice(c->device));
    cudaStream_t st = (cudaStream_t)stream;
    const int T = tokens, H = L->hidden, E = L->n_experts, K = L->top_k, W = g->world;
    Carve sz{nullptr, 0};
    sz.take<float>((size_t)T * E + 1);
    sz.take<int32_t>((size_t)T * W + 1);
    sz.take<int32_t>((size_t)T * W + 1);
    if ((rc = ensure_ws(c, sz.off + 256, st))) return rc;
    Carve w{c->ws, 0};
    float* logits = w.take<float>((size_t)T * E + 1);
    int32_t* cnt = w.take<int32_t>((size_t)T * W + 1);
    int32_t* pbase = w.take<int32_t>((size_t)T * W + 1);
    if (T > 0) {
        if ((rc = launch_router(x, L->router_w, L->router_b, T, H, E, logits, st))) return rc;
        if ((rc = launch_route(logits, T, E, K, L->norm_topk_prob, ids, weights, x,
                               shared ? L->sh_gate_inp : nullptr, H, shared ? sgate : nullptr, st)))
            return rc;
        c->launches += 2;
    }
    if ((rc = launch_ep_units(x, T, H, K, W, g->experts_per_rank, g->placement, L->n_experts, ids, weights, cnt,
                              unit_of, pbase, send_counts, ep_rows_f16(L), send_rows, send_picks, st)))
        return rc;
    c->launches += T > 0 ? 3 : 0;
    return CWX_OK;
}

extern "C" int cwx_ep_experts(cwx_ctx* c, const cwx_moe_layer* L, const cwx_ep_group* g, const void* rows,
                              const int32_t* picks, int32_t n_units, int32_t n_picks, int32_t n_src,
                              const int32_t* src_units, const int32_t* src_picks, float* y_units, void* stream) {
    if (!c) return fail(CWX_EINVAL, "cwx_ep_experts: null context");
    int rc = ep_check(L, g, "cwx_ep_experts");
    if (rc) return rc;
    if (n_units < 0 || n_picks < 0 || n_src < 1 || n_src > 64 || !src_units || !src_picks)
        return fail(CWX_EINVAL, "cwx_ep_experts: bad sizes");
    EpOffsets off;
    off.n = n_src;
    int64_t su = 0, sp = 0;
    for (int s = 0; s < n_src; ++s) {
        off.ustart[s] = su;
        off.pstart[s] = sp;
        su += src_units[s];
        sp += src_picks[s];
    }
    off.ustart[n_src] = su;
    off.pstart[n_src] = sp;
    if (su != n_units || sp != n_picks) return fail(CWX_EINVAL, "cwx_ep_experts: per-source counts do not add up");
    if (n_picks == 0) return CWX_OK;
    if (!rows || !picks || !y_units) return fail(CWX_EINVAL, "cwx_ep_experts: null argument");
    // this rank's experts as a layer of their own: one pick per record, rows through the row map
    cwx_moe_layer lc = *L;
    lc.n_experts = g->experts_per_rank;
    lc.top_k = 1;
    lc.sh_gate = lc.sh_up = lc.sh_down = nullptr;
    lc.sh_gate_inp = nullptr;
    if ((rc = validate_layer(&lc))) return rc;
    CWX_CUDA(cudaSetDevice(c->device));
    cudaStream_t st = (cudaStream_t)stream;
    const int H = L->hidden, E = lc.n_experts;
    const bool f16 = ep_rows_f16(L);
    const int mma = mma_layer(c, &lc, n_picks) ? 1 : 0;
    LayerPlan p;
    plan_layer(&lc, n_picks, mma, nullptr, &p);
    const size_t base = (p.bytes + 255) & ~(size_t)255;
    Carve ex{nullptr, 0};
    ex.take<uint32_t>((size_t)n_picks);
    ex.take<uint32_t>((size_t)n_picks);
    ex.take<float>((size_t)n_picks);
    ex.take<int32_t>((size_t)n_units + 1);
    if (f16) ex.take<float>((size_t)n_units * H);
    if ((rc = ensure_ws(c, base + ex.off + 256, st))) return rc;
    plan_layer(&lc, n_picks, mma, c->ws, &p);
    Carve w{c->ws + base, 0};
    uint32_t* rowmap = w.take<uint32_t>((size_t)n_picks);
    uint32_t* eid = w.take<uint32_t>((size_t)n_picks);
    float* wgt = w.take<float>((size_t)n_picks);
    int32_t* first = w.take<int32_t>((size_t)n_units + 1);
    float* rows32 = f16 ? w.take<float>((size_t)n_units * H) : nullptr;
    if ((rc = launch_ep_recv(picks, n_picks, off, rowmap, eid, wgt, first, st))) return rc;
    const float* x = reinterpret_cast<const float*>(rows);
    if (f16) {
        if ((rc = launch_f16_to_f32(reinterpret_cast<const __half*>(rows), (int64_t)n_units * H, rows32, st)))
            return rc;
        x = rows32;
    }
    p.xrows = n_units;
    p.rowmap = rowmap;
    p.ids = eid;  // per-pick expert (the clamped SwiGLU biases index it)
    if ((rc = launch_permute(eid, n_picks, E, p.pairs, p.heads, p.used3, p.n_used, p.perm, c->d_err, st))) return rc;
    c->launches += 1 + (f16 ? 1 : 0) + perm_launches(n_picks, E);
    cwx_moe_args a;
    memset(&a, 0, sizeof a);
    a.x = x;
    a.tokens = n_units;
    if ((rc = p.mma ? moe_mma(c, &lc, &a, p, st) : moe_gemv(c, &lc, &a, p, st))) return rc;
    if ((rc = launch_ep_unit_sum(p.y, wgt, first, n_units, n_picks, H, y_units, st))) return rc;
    c->launches += 1;
    return CWX_OK;
}

// The shared expert on the local tokens into ys (T, H): the tensor-core products when they apply
// (f32 activations, large batch), else the grouped mma.sync products.
static int ep_shared(cwx_ctx* c, const cwx_moe_layer* L, const float* x, int T, float** ys_out, cudaStream_t st) {
    const int H = L->hidden, Is = (int)L->sh_gate->L.n;
    LayerPlan p;
    memset(&p, 0, sizeof p);
    p.T = T;
    p.xrows = T;
    p.H = H;
    p.K = 1;
    p.Is = Is;
    p.msgu = act_mode_of(L->sh_gate, L->act_mode);
    p.msd = act_mode_of(L->sh_down, L->act_mode);
    const bool tc = shared_mma_ok(L) && c->mma_min_pile > 0 && T >= c->mma_min_pile;
    for (int pass = 0; pass < 2; ++pass) {
        Carve w{pass ? c->ws : nullptr, 0};
        p.ys = w.take<float>((size_t)T * H);
        p.n_used = w.take<uint32_t>(4);
        p.used3 = w.take<uint32_t>(4);
        p.pairs = w.take<uint32_t>((size_t)T + 1);
        if (tc) {
            p.x16 = w.take<__half>((size_t)T * H);
            p.hs16 = w.take<__half>((size_t)T * Is);
        } else {
            p.xpk[p.msgu] = w.take<uint8_t>((size_t)(T * packed_row_bytes(H)));
            p.gs = w.take<float>((size_t)T * Is);
            p.us = w.take<float>((size_t)T * Is);
            p.hspk = w.take<uint8_t>((size_t)(T * packed_row_bytes(Is)));
        }
        if (!pass) {
            int rc = ensure_ws(c, w.off + 256, st);
            if (rc) return rc;
        }
    }
    int rc;
    if (tc) {
        if ((rc = launch_f16rows(x, (int64_t)T * H, p.x16, st))) return rc;
        if ((rc = launch_all_tokens(p.pairs, T, p.used3, p.n_used, st))) return rc;
        MmaArgs m;
        memset(&m, 0, sizeof m);
        m.pairs = p.pairs;
        m.used3 = p.used3;
        m.n_used = p.n_used;
        m.err = c->d_err;
        m.bdiv = 1;
        MmaArgs gu = m;
        gu.a0 = mref(L->sh_gate);
        gu.a1 = mref(L->sh_up);
        gu.fused = 1;
        gu.b = reinterpret_cast<const uint8_t*>(p.x16);
        gu.bstride = (int64_t)H * 2;
        gu.brows = T;
        gu.hout = p.hs16;
        gu.ostride = Is;
        if ((rc = launch_mma(gu, c->device, c->sm_count, st))) return rc;
        MmaArgs dn = m;
        dn.a0 = mref(L->sh_down);
        dn.b = reinterpret_cast<const uint8_t*>(p.hs16);
        dn.bstride = (int64_t)Is * 2;
        dn.brows = T;
        dn.out = p.ys;
        dn.ostride = H;
        if ((rc = launch_mma(dn, c->device, c->sm_count, st))) return rc;
        c->launches += 4;
    } else {
        CWX_CUDA(cudaMemsetAsync(p.n_used, 0, 16, st));  // the shared-only product launches read it
        if ((rc = launch_prep(prep(x, nullptr, T, H, p.msgu, p.xpk[p.msgu]), st))) return rc;
        if ((rc = shared_gemv(c, L, p, 0, st))) return rc;
        if ((rc = launch_prep(prep(p.gs, p.us, T, Is, p.msd, p.hspk), st))) return rc;
        if ((rc = shared_gemv(c, L, p, 1, st))) return rc;
        c->launches += 4;
    }
    *ys_out = p.ys;
    return CWX_OK;
}

extern "C" int cwx_ep_combine(cwx_ctx* c, const cwx_moe_layer* L, const cwx_ep_group* g, const float* x,
                              int32_t tokens, const int32_t* unit_of, const float* back_rows, const float* sgate,
                              const float* residual, float* out, void* stream) {
    if (!c || !L || !g) return fail(CWX_EINVAL, "cwx_ep_combine: null argument");
    if (tokens < 0) return fail(CWX_EINVAL, "cwx_ep_combine: tokens %d", tokens);
    if (tokens == 0) return CWX_OK;
    if (!x || !unit_of || !out || g->world < 1 || g->world > 64) return fail(CWX_EINVAL, "cwx_ep_combine: bad argument");
    const bool shared = L->sh_gate != nullptr;
    if (shared && (!sgate || !L->sh_up || !L->sh_down || !L->sh_gate_inp))
        return fail(CWX_EINVAL, "cwx_ep_combine: incomplete shared expert");
    CWX_CUDA(cudaSetDevice(c->device));
    cudaStream_t st = (cudaStream_t)stream;
    int rc;
    float* ys = nullptr;
    if (shared && (rc = ep_shared(c, L, x, tokens, &ys, st))) return rc;
    if ((rc = launch_ep_combine(back_rows, unit_of, tokens, g->world, L->hidden, ys, sgate, residual, out, st)))
        return rc;
    c->launches += 1;
    return CWX_OK;
}

// A whole expert-parallel layer with the library's own transport: the three steps above with
// fixed-capacity exchanges between them (ep_nccl.cu), so the receive sizes never travel through
// the host. Buffers that live across the exchanges (the routing, the units' places, the send and
// receive segments, the unit sums) are the communicator's; the workspace holds each step's
// temporaries.
extern "C" int cwx_ep_forward(cwx_ctx* c, cwx_ep_comm* comm, const cwx_moe_layer* L, const cwx_ep_group* g,
                              const float* x, int32_t tokens, int32_t cap_tokens, const float* residual, float* out,
                              uint32_t* ids_out, void* stream) {
    if (!c || !comm) return fail(CWX_EINVAL, "cwx_ep_forward: null context or communicator");
    int rc = ep_check(L, g, "cwx_ep_forward");
    if (rc) return rc;
    int cw = 0, cr = 0, cd = 0;
    if ((rc = ep_comm_info(comm, &cw, &cr, &cd))) return rc;
    if (cw != g->world || cr != g->rank || cd != c->device)
        return fail(CWX_EINVAL,
                    "cwx_ep_forward: the communicator is rank %d of %d on device %d, the group rank %d of %d and "
                    "the context device %d",
                    cr, cw, cd, g->rank, g->world, c->device);
    if (!L->router_w || L->top_k < 1 || L->top_k > 16 || L->top_k > L->n_experts || L->n_experts > 1024)
        return fail(CWX_EINVAL, "cwx_ep_forward: router or top_k out of range");
    if (tokens < 0 || cap_tokens < 1 || tokens > cap_tokens)
        return fail(CWX_EINVAL, "cwx_ep_forward: tokens %d with capacity %d", tokens, cap_tokens);
    if (tokens && (!x || !out)) return fail(CWX_EINVAL, "cwx_ep_forward: null x or out");
    if (L->hidden % 4 || ((uintptr_t)x & 15)) return fail(CWX_EINVAL, "cwx_ep_forward: x rows must be 16-byte aligned");
    const bool shared = L->sh_gate != nullptr;
    if (shared && (!L->sh_up || !L->sh_down || !L->sh_gate_inp))
        return fail(CWX_EINVAL, "cwx_ep_forward: incomplete shared expert");
    cwx_moe_layer lc = *L;  // this rank's experts as a layer of their own, one pick per record
    lc.n_experts = g->experts_per_rank;
    lc.top_k = 1;
    lc.sh_gate = lc.sh_up = lc.sh_down = nullptr;
    lc.sh_gate_inp = nullptr;
    if ((rc = validate_layer(&lc))) return rc;
    CWX_CUDA(cudaSetDevice(c->device));
    cudaStream_t st = (cudaStream_t)stream;
    const int T = tokens, cap = cap_tokens, H = L->hidden, E = L->n_experts, K = L->top_k, W = g->world;
    const int epr = g->experts_per_rank;
    const int cap_rec = cap * (K < epr ? K : epr);
    const bool f16 = ep_rows_f16(L);
    const size_t rb = f16 ? 2 : 4;
    const int64_t U = (int64_t)W * cap, P = (int64_t)W * cap_rec;
    if (P > INT32_MAX / 2) return fail(CWX_EUNSUPPORTED, "cwx_ep_forward: %lld record slots", (long long)P);

    // the communicator's buffers (sized in a first pass, carved in the second)
    uint32_t* ids = nullptr;
    float *wts = nullptr, *sgate = nullptr, *yu = nullptr, *back = nullptr;
    int32_t *unit_of = nullptr, *scnt = nullptr, *rcnt = nullptr, *spk = nullptr, *rpk = nullptr;
    void *srows = nullptr, *rrows = nullptr;
    size_t need = 0;
    for (int pass = 0; pass < 2; ++pass) {
        Carve b{nullptr, 0};
        if (pass) {
            void* base = nullptr;
            if ((rc = ep_comm_buffer(comm, need, st, &base))) return rc;
            b.base = static_cast<uint8_t*>(base);
        }
        ids = b.take<uint32_t>((size_t)cap * K);
        wts = b.take<float>((size_t)cap * K);
        sgate = b.take<float>((size_t)cap);
        unit_of = b.take<int32_t>((size_t)cap * W);
        scnt = b.take<int32_t>((size_t)2 * W);
        rcnt = b.take<int32_t>((size_t)2 * W);
        srows = b.take<uint8_t>((size_t)U * H * rb);
        rrows = b.take<uint8_t>((size_t)U * H * rb);
        spk = b.take<int32_t>((size_t)P * 3);
        rpk = b.take<int32_t>((size_t)P * 3);
        yu = b.take<float>((size_t)U * H);
        back = b.take<float>((size_t)U * H);
        need = b.off + 256;
    }

    // 1. dispatch into the fixed-capacity send segments
    {
        PhaseTimer t(c, st, CWX_PHASE_EP_DISPATCH);
        Carve sz{nullptr, 0};
        sz.take<float>((size_t)T * E + 1);
        sz.take<int32_t>((size_t)T * W + 1);
        sz.take<int32_t>((size_t)T * W + 1);
        if ((rc = ensure_ws(c, sz.off + 256, st))) return rc;
        Carve w{c->ws, 0};
        float* logits = w.take<float>((size_t)T * E + 1);
        int32_t* cnt = w.take<int32_t>((size_t)T * W + 1);
        int32_t* pbase = w.take<int32_t>((size_t)T * W + 1);
        if (T > 0) {
            if ((rc = launch_router(x, L->router_w, L->router_b, T, H, E, logits, st))) return rc;
            if ((rc = launch_route(logits, T, E, K, L->norm_topk_prob, ids, wts, x, shared ? L->sh_gate_inp : nullptr,
                                   H, shared ? sgate : nullptr, st)))
                return rc;
            c->launches += 2;
        }
        if ((rc = launch_ep_units(x, T, H, K, W, epr, g->placement, L->n_experts, ids, wts, cnt, unit_of, pbase, scnt,
                                  f16, srows, spk, st, cap, cap_rec)))
            return rc;
        c->launches += T > 0 ? 3 : 0;
        t.end();
    }
    // 2. counts, unit rows and pick records to every peer, in one group
    {
        const void* snd[3] = {scnt, srows, spk};
        void* rcv[3] = {rcnt, rrows, rpk};
        const size_t bytes[3] = {8, (size_t)cap * H * rb, (size_t)cap_rec * 12};
        PhaseTimer t(c, st, CWX_PHASE_EP_EXCHANGE);
        if ((rc = ep_comm_exchange(comm, 3, snd, rcv, bytes, st))) return rc;
        t.end();
    }
    // 3. this rank's experts over the received records; each unit's weighted sum
    {
        PhaseTimer t(c, st, CWX_PHASE_EP_EXPERTS);
        // the product path from the expected picks per rank (tokens spread evenly over the ranks)
        const int mma = mma_layer(c, &lc, cap * K) ? 1 : 0;
        LayerPlan p;
        plan_layer(&lc, (int)P, mma, nullptr, &p);
        const size_t base = (p.bytes + 255) & ~(size_t)255;
        Carve ex{nullptr, 0};
        ex.take<uint32_t>((size_t)P);
        ex.take<uint32_t>((size_t)P);
        ex.take<float>((size_t)P);
        ex.take<int32_t>((size_t)U);
        ex.take<int32_t>((size_t)U);
        ex.take<int32_t>(4);
        if (f16) ex.take<float>((size_t)U * H);
        if ((rc = ensure_ws(c, base + ex.off + 256, st))) return rc;
        plan_layer(&lc, (int)P, mma, c->ws, &p);
        Carve w{c->ws + base, 0};
        uint32_t* rowmap = w.take<uint32_t>((size_t)P);
        uint32_t* eid = w.take<uint32_t>((size_t)P);
        float* wgt = w.take<float>((size_t)P);
        int32_t* first = w.take<int32_t>((size_t)U);
        int32_t* end = w.take<int32_t>((size_t)U);
        int32_t* n_picks = w.take<int32_t>(4);
        float* rows32 = f16 ? w.take<float>((size_t)U * H) : nullptr;
        // pick slots past the received records still go through the hidden-row preparation, which
        // reads each slot's expert (the clamped SwiGLU biases): they get expert 0, a valid index
        CWX_CUDA(cudaMemsetAsync(eid, 0, (size_t)P * 4, st));
        if ((rc = launch_ep_recv_cap(rpk, rcnt, W, cap, cap_rec, rowmap, eid, wgt, first, end, n_picks, st))) return rc;
        const float* xr = reinterpret_cast<const float*>(rrows);
        if (f16) {
            if ((rc = launch_f16_to_f32(reinterpret_cast<const __half*>(rrows), U * H, rows32, st))) return rc;
            xr = rows32;
        }
        p.xrows = U;
        p.rowmap = rowmap;
        p.ids = eid;  // per-pick expert (the clamped SwiGLU biases index it)
        if ((rc = launch_permute(eid, P, epr, p.pairs, p.heads, p.used3, p.n_used, p.perm, c->d_err, st, n_picks)))
            return rc;
        c->launches += 1 + (f16 ? 1 : 0) + perm_launches(P, epr);
        cwx_moe_args a;
        memset(&a, 0, sizeof a);
        a.x = xr;
        a.tokens = (int32_t)U;
        if ((rc = p.mma ? moe_mma(c, &lc, &a, p, st) : moe_gemv(c, &lc, &a, p, st))) return rc;
        if ((rc = launch_ep_unit_sum_cap(p.y, wgt, first, end, rcnt, W, cap, H, yu, st))) return rc;
        c->launches += 1;
        t.end();
    }
    // 4. the unit sums back to their sources
    {
        const void* snd[1] = {yu};
        void* rcv[1] = {back};
        const size_t bytes[1] = {(size_t)cap * H * 4};
        PhaseTimer t(c, st, CWX_PHASE_EP_RETURN);
        if ((rc = ep_comm_exchange(comm, 1, snd, rcv, bytes, st))) return rc;
        t.end();
    }
    // 5. combine: the returned units in rank order, the shared expert, the residual
    if (T > 0) {
        PhaseTimer t(c, st, CWX_PHASE_EP_COMBINE);
        float* ys = nullptr;
        if (shared && (rc = ep_shared(c, L, x, T, &ys, st))) return rc;
        if ((rc = launch_ep_combine(back, unit_of, T, W, H, ys, sgate, residual, out, st))) return rc;
        c->launches += 1;
        if (ids_out) CWX_CUDA(cudaMemcpyAsync(ids_out, ids, (size_t)T * K * 4, cudaMemcpyDeviceToDevice, st));
        t.end();
    }
    return CWX_OK;
}
