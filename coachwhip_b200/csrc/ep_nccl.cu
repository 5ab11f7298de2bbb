// The expert-parallel transport inside the library: an NCCL communicator per rank and the
// fixed-capacity exchanges of cwx_ep_forward.
//
// The reference runs one device and has no collective; this is the transport of its layer split
// by expert over the GPUs of one node. NCCL is bound at run time (dlopen of libnccl.so.2, the copy
// already in the process when there is one, e.g. a framework's), so the library has no link-time
// dependency on it and a host without NCCL loses only the expert-parallel entry points.
//
// Exchanges have fixed sizes per peer: a token sends at most one row to each rank (a unit), so a
// rank receives at most cap_tokens units from every peer, and the records of a unit are at most
// min(top_k, experts per rank). Every segment is sent whole and the receiver reads the counts that
// travel in the same group, on the device: no host synchronisation in a layer.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <mutex>

#include "cwx_common.cuh"
#include "kernels.cuh"

struct cwx_ep_comm {
    ncclComm_t comm;
    int world, rank, device;
    int owned;     // created here (destroyed by cwx_ep_comm_destroy) or wrapped
    void* buf;     // the exchange buffers of cwx_ep_forward (grown on demand)
    size_t buf_bytes;
};

namespace cwx {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*);
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    ncclResult_t (*CommAbort)(ncclComm_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    const char* (*GetErrorString)(ncclResult_t);
};

static std::mutex g_nccl_mu;
static NcclApi g_nccl;
static int g_nccl_state = 0;  // 0 not tried, 1 bound, -1 unavailable

static int nccl_api(const NcclApi** out) {
    std::lock_guard<std::mutex> lock(g_nccl_mu);
    if (g_nccl_state == 0) {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the copy already loaded, if any
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        g_nccl_state = -1;
        if (h) {
            bool ok = true;
            auto sym = [&](const char* n) {
                void* p = dlsym(h, n);
                ok = ok && p;
                return p;
            };
            g_nccl.GetUniqueId = (ncclResult_t(*)(ncclUniqueId*))sym("ncclGetUniqueId");
            g_nccl.CommInitRank = (ncclResult_t(*)(ncclComm_t*, int, ncclUniqueId, int))sym("ncclCommInitRank");
            g_nccl.CommDestroy = (ncclResult_t(*)(ncclComm_t))sym("ncclCommDestroy");
            g_nccl.CommAbort = (ncclResult_t(*)(ncclComm_t))sym("ncclCommAbort");
            g_nccl.GroupStart = (ncclResult_t(*)())sym("ncclGroupStart");
            g_nccl.GroupEnd = (ncclResult_t(*)())sym("ncclGroupEnd");
            g_nccl.Send =
                (ncclResult_t(*)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t))sym("ncclSend");
            g_nccl.Recv =
                (ncclResult_t(*)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t))sym("ncclRecv");
            g_nccl.GetErrorString = (const char* (*)(ncclResult_t))sym("ncclGetErrorString");
            if (ok) g_nccl_state = 1;
        }
    }
    if (g_nccl_state != 1) return fail(CWX_EUNSUPPORTED, "NCCL (libnccl.so.2) is not available in this process");
    *out = &g_nccl;
    return CWX_OK;
}

static int nccl_fail(const NcclApi* n, ncclResult_t r, const char* what) {
    return fail(CWX_ECOMM, "%s: %s", what, n && n->GetErrorString ? n->GetErrorString(r) : "NCCL error");
}

int ep_comm_info(const cwx_ep_comm* c, int* world, int* rank, int* device) {
    if (!c || !c->comm) return fail(CWX_EINVAL, "null or aborted expert-parallel communicator");
    *world = c->world;
    *rank = c->rank;
    *device = c->device;
    return CWX_OK;
}

int ep_comm_buffer(cwx_ep_comm* c, size_t bytes, cudaStream_t st, void** out) {
    if (bytes > c->buf_bytes) {
        if (c->buf) {
            CWX_CUDA(cudaStreamSynchronize(st));
            cudaFree(c->buf);
            c->buf = nullptr;
            c->buf_bytes = 0;
        }
        const size_t nb = ((bytes + (1 << 20) - 1) >> 20) << 20;
        CWX_CUDA(cudaMalloc(&c->buf, nb));
        c->buf_bytes = nb;
    }
    *out = c->buf;
    return CWX_OK;
}

// One group of sends and receives: for each buffer b, the bytes[b] segment of every peer p at
// send[b] + p * bytes[b] goes to peer p, which receives it at recv[b] + rank * bytes[b].
int ep_comm_exchange(cwx_ep_comm* c, int nbuf, const void* const* send, void* const* recv, const size_t* bytes,
                     cudaStream_t st) {
    const NcclApi* n = nullptr;
    int rc = nccl_api(&n);
    if (rc) return rc;
    ncclResult_t r = n->GroupStart();
    if (r != ncclSuccess) return nccl_fail(n, r, "ncclGroupStart");
    for (int b = 0; b < nbuf; ++b) {
        if (!bytes[b]) continue;
        for (int p = 0; p < c->world; ++p) {
            r = n->Send(static_cast<const uint8_t*>(send[b]) + (size_t)p * bytes[b], bytes[b], ncclUint8, p, c->comm, st);
            if (r == ncclSuccess)
                r = n->Recv(static_cast<uint8_t*>(recv[b]) + (size_t)p * bytes[b], bytes[b], ncclUint8, p, c->comm, st);
            if (r != ncclSuccess) {
                n->GroupEnd();
                return nccl_fail(n, r, "ncclSend/ncclRecv");
            }
        }
    }
    r = n->GroupEnd();
    return r == ncclSuccess ? CWX_OK : nccl_fail(n, r, "ncclGroupEnd");
}

}  // namespace cwx

using namespace cwx;

extern "C" int cwx_ep_unique_id(void* out, int64_t cap) {
    if (!out || cap < NCCL_UNIQUE_ID_BYTES)
        return fail(CWX_EINVAL, "cwx_ep_unique_id: needs a buffer of %d bytes", NCCL_UNIQUE_ID_BYTES);
    const NcclApi* n = nullptr;
    int rc = nccl_api(&n);
    if (rc) return rc;
    ncclUniqueId id;
    ncclResult_t r = n->GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(n, r, "ncclGetUniqueId");
    memcpy(out, &id, NCCL_UNIQUE_ID_BYTES);
    return CWX_OK;
}

extern "C" int cwx_ep_comm_create(int device, const void* id, int32_t world, int32_t rank, cwx_ep_comm** out) {
    if (!id || !out) return fail(CWX_EINVAL, "cwx_ep_comm_create: null argument");
    if (world < 1 || world > 64 || rank < 0 || rank >= world)
        return fail(CWX_EINVAL, "cwx_ep_comm_create: rank %d of %d (1..64 ranks)", rank, world);
    *out = nullptr;
    const NcclApi* n = nullptr;
    int rc = nccl_api(&n);
    if (rc) return rc;
    CWX_CUDA(cudaSetDevice(device));
    ncclUniqueId uid;
    memcpy(&uid, id, NCCL_UNIQUE_ID_BYTES);
    ncclComm_t comm = nullptr;
    ncclResult_t r = n->CommInitRank(&comm, world, uid, rank);
    if (r != ncclSuccess) return nccl_fail(n, r, "ncclCommInitRank");
    cwx_ep_comm* c = new cwx_ep_comm();
    memset(c, 0, sizeof *c);
    c->comm = comm;
    c->world = world;
    c->rank = rank;
    c->device = device;
    c->owned = 1;
    *out = c;
    return CWX_OK;
}

extern "C" int cwx_ep_comm_wrap(void* nccl_comm, int32_t world, int32_t rank, int device, cwx_ep_comm** out) {
    if (!nccl_comm || !out) return fail(CWX_EINVAL, "cwx_ep_comm_wrap: null argument");
    if (world < 1 || world > 64 || rank < 0 || rank >= world)
        return fail(CWX_EINVAL, "cwx_ep_comm_wrap: rank %d of %d (1..64 ranks)", rank, world);
    cwx_ep_comm* c = new cwx_ep_comm();
    memset(c, 0, sizeof *c);
    c->comm = (ncclComm_t)nccl_comm;
    c->world = world;
    c->rank = rank;
    c->device = device;
    *out = c;
    return CWX_OK;
}

extern "C" int cwx_ep_comm_abort(cwx_ep_comm* c) {
    if (!c) return fail(CWX_EINVAL, "cwx_ep_comm_abort: null communicator");
    const NcclApi* n = nullptr;
    int rc = nccl_api(&n);
    if (rc) return rc;
    if (c->comm && c->owned) {
        ncclResult_t r = n->CommAbort(c->comm);
        c->comm = nullptr;
        if (r != ncclSuccess) return nccl_fail(n, r, "ncclCommAbort");
    }
    c->comm = nullptr;
    return CWX_OK;
}

extern "C" int cwx_ep_comm_destroy(cwx_ep_comm* c) {
    if (!c) return CWX_OK;
    int rc = CWX_OK;
    cudaSetDevice(c->device);
    if (c->owned && c->comm) {
        const NcclApi* n = nullptr;
        rc = nccl_api(&n);
        if (!rc) {
            ncclResult_t r = n->CommDestroy(c->comm);
            if (r != ncclSuccess) rc = nccl_fail(n, r, "ncclCommDestroy");
        }
    }
    if (c->buf) cudaFree(c->buf);
    delete c;
    return rc;
}
