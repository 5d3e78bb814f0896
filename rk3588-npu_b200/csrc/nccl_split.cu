// nccl_split.cu -- split-KV across GPUs with the merge over an NCCL all-gather.
//
// A long sequence is split along its positions across the GPUs of a node
// (one process per GPU).  Per layer every rank attends over its slice and
// gets, per (sequence, query head) row, a partial state (m, l, o); the
// states of all ranks are all-gathered and merged with the log-sum-exp
// identity (the same merge as attn_combine_lse_packed).  The reference has
// no split-KV (it runs one sequence on one device).
//
// The communicator is NCCL's, created here from a unique id the caller
// passes between its processes, so a C++ worker needs no other framework.
// NCCL is loaded at run time: the copy already in the process if there is
// one (e.g. the one a Python framework linked), so a communicator and the
// collectives on it always come from the same library; otherwise
// libnccl.so.2 from the library path.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "kvattn.h"
#include "kvattn_internal.h"

struct kvn_comm {
    int device = 0, rank = 0, world = 1, max_rows = 0;
    ncclComm_t comm = nullptr;
    float* send = nullptr;  // [m rows][l rows][o rows x 128] of this rank
    float* recv = nullptr;  // world x the same
    std::mutex mu;
};

namespace kvattn {
namespace {

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) init_rank = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    bool ok = false;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
        api.init_rank = (decltype(api.init_rank))dlsym(h, "ncclCommInitRank");
        api.destroy = (decltype(api.destroy))dlsym(h, "ncclCommDestroy");
        api.all_gather = (decltype(api.all_gather))dlsym(h, "ncclAllGather");
        api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
        api.ok = api.get_unique_id && api.init_rank && api.destroy && api.all_gather && api.error_string;
    });
    return api;
}

int nccl_fail(ncclResult_t r, const char* what) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
    return set_error(KV_ERR_CUDA, buf);
}

}  // namespace

int nccl_prepare(::kvn_comm* c, int device, int rows, float** m, float** l, float** o) {
    if (c->device != device) return set_error(KV_ERR_INVAL, "communicator and pool are on different devices");
    if (rows > c->max_rows) return set_error(KV_ERR_RANGE, "more rows than the communicator was created for");
    *m = c->send;
    *l = c->send + rows;
    *o = c->send + 2 * (size_t)rows;
    return KV_OK;
}

int nccl_gather_combine(::kvn_comm* c, int rows, float* out, cudaStream_t st) {
    std::lock_guard<std::mutex> lk(c->mu);
    const size_t per = (size_t)rows * (2 + kHeadDim);
    // The packed states of every rank land at recv + g * per: the layout the
    // merge reads.  (Only `rows` rows of the send buffer are filled.)
    const ncclResult_t r = nccl().all_gather(c->send, c->recv, per, ncclFloat32, c->comm, st);
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
    const float* pk = c->recv;
    cudaError_t e = launch_combine(c->world, rows, kHeadDim, pk, pk + rows, pk + 2 * (size_t)rows, per, per, out, st);
    if (e != cudaSuccess) return set_error(KV_ERR_CUDA, cudaGetErrorString(e));
    return KV_OK;
}

}  // namespace kvattn

using namespace kvattn;

extern "C" {

int kvn_unique_id(void* id) {
    if (!id) return set_error(KV_ERR_INVAL, "id is NULL");
    if (!nccl().ok) return set_error(KV_ERR_STATE, "NCCL (libnccl.so.2) could not be loaded");
    ncclUniqueId u;
    const ncclResult_t r = nccl().get_unique_id(&u);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(id, &u, sizeof u);
    return KV_OK;
}

int kvn_create(int device, int rank, int world, const void* id, int max_rows, kvn_comm** out) {
    if (!out || !id) return set_error(KV_ERR_INVAL, "NULL argument");
    *out = nullptr;
    if (world < 1 || rank < 0 || rank >= world || max_rows < 1)
        return set_error(KV_ERR_INVAL, "bad rank, world or max_rows");
    if (!nccl().ok) return set_error(KV_ERR_STATE, "NCCL (libnccl.so.2) could not be loaded");
    DeviceGuard dg(device);
    if (!dg.ok) return set_error(KV_ERR_CUDA, "cudaSetDevice failed");
    kvn_comm* c = new kvn_comm();
    c->device = device;
    c->rank = rank;
    c->world = world;
    c->max_rows = max_rows;
    const size_t per = (size_t)max_rows * (2 + kHeadDim);
    if (cudaMalloc((void**)&c->send, per * sizeof(float)) != cudaSuccess ||
        cudaMalloc((void**)&c->recv, per * world * sizeof(float)) != cudaSuccess) {
        cudaFree(c->send);
        cudaFree(c->recv);
        delete c;
        return set_error(KV_ERR_CUDA, "cudaMalloc of the exchange buffers failed");
    }
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    const ncclResult_t r = nccl().init_rank(&c->comm, world, u, rank);
    if (r != ncclSuccess) {
        cudaFree(c->send);
        cudaFree(c->recv);
        delete c;
        return nccl_fail(r, "ncclCommInitRank");
    }
    *out = c;
    return KV_OK;
}

int kvn_destroy(kvn_comm* c) {
    if (!c) return KV_OK;
    {
        DeviceGuard dg(c->device);
        cudaDeviceSynchronize();
        if (c->comm) nccl().destroy(c->comm);
        cudaFree(c->send);
        cudaFree(c->recv);
    }
    delete c;
    return KV_OK;
}

}  // extern "C"
