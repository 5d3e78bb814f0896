// sched_host.cpp -- placement of requests onto GPUs (host-only C ABI).
//
// The reference engine serves one sequence on one device
// (worker/src/engine/llm_engine.cpp:68-98); there is no scheduler to mirror.
// Serving many sequences on one 8-GPU box partitions the work by request:
// every GPU owns whole sequences, their blocks and their block tables, and
// the decode path needs no collective.  What remains is choosing the GPU, so
// that the resident context (the bytes each GPU streams per decode step)
// stays balanced: a new request goes to the GPU with the fewest resident KV
// blocks among those with room for it, ties to the lowest index.
//
// The state is deterministic host data, so each rank may run its own copy
// on the same request stream and reach the same decisions.
#include <stdio.h>

#include <mutex>
#include <unordered_map>
#include <vector>

#include "kvattn.h"
#include "kvattn_internal.h"

using kvattn::set_error;

struct kvs_sched {
    int block_tokens = 16;
    std::vector<long long> capacity;  // blocks per GPU
    std::vector<long long> resident;  // blocks held by placed requests
    std::vector<int> requests;        // placed requests per GPU
    struct Req {
        int gpu;
        long long blocks;
    };
    std::unordered_map<long long, Req> reqs;
    mutable std::mutex mu;

    long long blocks_for(long long tokens) const { return (tokens + block_tokens - 1) / block_tokens; }
};

namespace {

int err(int status, const char* fmt, long long a = 0, long long b = 0) {
    char buf[256];
    snprintf(buf, sizeof buf, fmt, a, b);
    return set_error(status, buf);
}

}  // namespace

extern "C" {

int kvs_create(int n_gpus, int block_tokens, const long long* blocks_per_gpu, kvs_sched** out) {
    if (!out || !blocks_per_gpu) return err(KV_ERR_INVAL, "NULL argument");
    *out = nullptr;
    if (n_gpus < 1 || block_tokens < 1) return err(KV_ERR_INVAL, "n_gpus %lld / block_tokens %lld must be positive", n_gpus, block_tokens);
    for (int g = 0; g < n_gpus; ++g)
        if (blocks_per_gpu[g] < 0) return err(KV_ERR_INVAL, "GPU %lld has negative capacity %lld", g, blocks_per_gpu[g]);
    kvs_sched* s = new kvs_sched;
    s->block_tokens = block_tokens;
    s->capacity.assign(blocks_per_gpu, blocks_per_gpu + n_gpus);
    s->resident.assign(n_gpus, 0);
    s->requests.assign(n_gpus, 0);
    *out = s;
    return KV_OK;
}

int kvs_destroy(kvs_sched* s) {
    delete s;
    return KV_OK;
}

int kvs_place(kvs_sched* s, long long request, int tokens, int* gpu) {
    if (!s || !gpu) return err(KV_ERR_INVAL, "NULL argument");
    if (tokens < 0) return err(KV_ERR_INVAL, "tokens %lld < 0", tokens);
    std::lock_guard<std::mutex> lk(s->mu);
    if (s->reqs.count(request)) return err(KV_ERR_INVAL, "request %lld is already placed", request);
    const long long need = s->blocks_for(tokens);
    int best = -1;
    for (int g = 0; g < (int)s->capacity.size(); ++g) {
        if (s->resident[g] + need > s->capacity[g]) continue;
        if (best < 0 || s->resident[g] < s->resident[best]) best = g;
    }
    if (best < 0) return err(KV_ERR_OOM, "no GPU has room for %lld blocks (request %lld)", need, request);
    s->resident[best] += need;
    s->requests[best] += 1;
    s->reqs[request] = kvs_sched::Req{best, need};
    *gpu = best;
    return KV_OK;
}

int kvs_resize(kvs_sched* s, long long request, int tokens) {
    if (!s) return err(KV_ERR_INVAL, "NULL argument");
    if (tokens < 0) return err(KV_ERR_INVAL, "tokens %lld < 0", tokens);
    std::lock_guard<std::mutex> lk(s->mu);
    auto it = s->reqs.find(request);
    if (it == s->reqs.end()) return err(KV_ERR_BADSEQ, "request %lld is not placed", request);
    const long long need = s->blocks_for(tokens);
    const int g = it->second.gpu;
    const long long delta = need - it->second.blocks;
    if (delta > 0 && s->resident[g] + delta > s->capacity[g])
        return err(KV_ERR_OOM, "GPU %lld has no room for %lld more blocks", g, delta);
    s->resident[g] += delta;
    it->second.blocks = need;
    return KV_OK;
}

int kvs_release(kvs_sched* s, long long request) {
    if (!s) return err(KV_ERR_INVAL, "NULL argument");
    std::lock_guard<std::mutex> lk(s->mu);
    auto it = s->reqs.find(request);
    if (it == s->reqs.end()) return err(KV_ERR_BADSEQ, "request %lld is not placed", request);
    s->resident[it->second.gpu] -= it->second.blocks;
    s->requests[it->second.gpu] -= 1;
    s->reqs.erase(it);
    return KV_OK;
}

int kvs_gpu_of(const kvs_sched* s, long long request, int* gpu) {
    if (!s || !gpu) return err(KV_ERR_INVAL, "NULL argument");
    std::lock_guard<std::mutex> lk(s->mu);
    auto it = s->reqs.find(request);
    if (it == s->reqs.end()) return err(KV_ERR_BADSEQ, "request %lld is not placed", request);
    *gpu = it->second.gpu;
    return KV_OK;
}

int kvs_load(const kvs_sched* s, int gpu, long long* resident_blocks, int* resident_requests) {
    if (!s) return err(KV_ERR_INVAL, "NULL argument");
    std::lock_guard<std::mutex> lk(s->mu);
    if (gpu < 0 || gpu >= (int)s->capacity.size()) return err(KV_ERR_INVAL, "GPU %lld out of range", gpu);
    if (resident_blocks) *resident_blocks = s->resident[gpu];
    if (resident_requests) *resident_requests = s->requests[gpu];
    return KV_OK;
}

}  // extern "C"
