// Drives include/kvattn_kvcache.hpp the way Qwen2Model::forward drives KVCache
// (worker/src/model/qwen2_model.cpp:131-274): prefill, then decode steps, then
// the op_attention shim on the gathered contiguous rows.  Test program:
//   kvcache_adapter host          bookkeeping on a host-only pool, prints "ok"
//   kvcache_adapter gpu <file>    runs on cuda:0 and writes inputs and outputs
//                                 (float32 arrays, then uint16 rows) to <file>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "kvattn_kvcache.hpp"

namespace {

int fails = 0;
#define CHECK(c)                                                   \
    do {                                                           \
        if (!(c)) {                                                \
            std::fprintf(stderr, "CHECK failed line %d: %s (%s)\n", \
                         __LINE__, #c, kv_last_error());           \
            ++fails;                                               \
        }                                                          \
    } while (0)

uint64_t rng_state = 0x9E3779B97F4A7C15ull;
float urand() {  // xorshift64*, uniform in [-2, 2)
    rng_state ^= rng_state >> 12;
    rng_state ^= rng_state << 25;
    rng_state ^= rng_state >> 27;
    const uint64_t x = rng_state * 0x2545F4914F6CDD1Dull;
    return (float)((x >> 40) * (1.0 / 16777216.0) * 4.0 - 2.0);
}

std::vector<float> rand_vec(size_t n) {
    std::vector<float> v(n);
    for (auto& x : v) x = urand();
    return v;
}

float* to_dev(const std::vector<float>& h) {
    float* d = nullptr;
    cudaMalloc(&d, h.size() * 4);
    cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice);
    return d;
}

int host_mode() {
    kvattn::KVCacheConfig cfg;
    cfg.device = KVP_HOST_ONLY;
    kvattn::PagedKVCache kc(cfg);
    CHECK(kc.init(28, 512, 256));
    CHECK(kc.capacity() == 512 && kc.kv_dim() == 256 && kc.cur_pos() == 0);
    kc.set_cur_pos(100);
    CHECK(kc.cur_pos() == 100);
    CHECK(kc.begin_step());
    CHECK(kc.end_step());
    CHECK(kc.cur_pos() == 101);
    kc.reset();
    CHECK(kc.cur_pos() == 0 && kc.capacity() == 512);
    CHECK(!kc.init(2, 64, 100));  // kv_dim not a multiple of 128
    if (fails == 0) std::printf("ok\n");
    return fails ? 1 : 0;
}

int gpu_mode(const char* path) {
    const int L = 2, KVD = 256, HID = 1536, P = 40, STEPS = 5, CAP = 64;
    kvattn::PagedKVCache kc;  // device 0, fp16, 12 query heads
    CHECK(kc.init(L, CAP, KVD));
    std::FILE* f = std::fopen(path, "wb");
    if (!f) return 2;
    auto put = [&](const std::vector<float>& v) { std::fwrite(v.data(), 4, v.size(), f); };
    // prefill: P tokens, every layer, then the position advances once
    for (int li = 0; li < L; ++li) {
        auto k = rand_vec((size_t)P * KVD), v = rand_vec((size_t)P * KVD);
        float *kd = to_dev(k), *vd = to_dev(v);
        CHECK(kc.append_prefill(li, P, kd, vd));
        put(k);
        put(v);
        cudaFree(kd);
        cudaFree(vd);
    }
    kc.set_cur_pos(kc.cur_pos() + P);
    CHECK(kc.cur_pos() == P);
    // decode steps
    float* outd = nullptr;
    cudaMalloc(&outd, HID * 4);
    std::vector<float> out(HID);
    for (int s = 0; s < STEPS; ++s) {
        CHECK(kc.begin_step());
        for (int li = 0; li < L; ++li) {
            auto q = rand_vec(HID), k = rand_vec(KVD), v = rand_vec(KVD);
            float *qd = to_dev(q), *kd = to_dev(k), *vd = to_dev(v);
            CHECK(kc.decode_layer(li, qd, kd, vd, outd));
            cudaMemcpy(out.data(), outd, HID * 4, cudaMemcpyDeviceToHost);
            put(q);
            put(k);
            put(v);
            put(out);
            cudaFree(qd);
            cudaFree(kd);
            cudaFree(vd);
        }
        CHECK(kc.end_step());
    }
    const int T = kc.cur_pos();
    CHECK(T == P + STEPS);
    // contiguous rows of layer 0, then op_attention over them (3 queries)
    uint16_t *kr = nullptr, *vr = nullptr;
    cudaMalloc(&kr, (size_t)T * KVD * 2);
    cudaMalloc(&vr, (size_t)T * KVD * 2);
    CHECK(kc.gather(0, kr, vr));
    auto q3 = rand_vec((size_t)3 * HID);
    float* q3d = to_dev(q3);
    float* o3d = nullptr;
    cudaMalloc(&o3d, (size_t)3 * HID * 4);
    kvattn::op_attention(q3d, kr, vr, o3d, 3, T, 12, 2, 128, T - 3);
    std::vector<float> o3((size_t)3 * HID);
    cudaMemcpy(o3.data(), o3d, o3.size() * 4, cudaMemcpyDeviceToHost);
    put(q3);
    put(o3);
    std::vector<uint16_t> kh((size_t)T * KVD), vh((size_t)T * KVD);
    cudaMemcpy(kh.data(), kr, kh.size() * 2, cudaMemcpyDeviceToHost);
    cudaMemcpy(vh.data(), vr, vh.size() * 2, cudaMemcpyDeviceToHost);
    std::fwrite(kh.data(), 2, kh.size(), f);
    std::fwrite(vh.data(), 2, vh.size(), f);
    std::fclose(f);
    CHECK(cudaDeviceSynchronize() == cudaSuccess);
    int st = 0;
    CHECK(kvp_device_status(kc.pool(), nullptr, &st) == KV_OK && st == 0);
    if (fails == 0) std::printf("ok\n");
    return fails ? 1 : 0;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc >= 2 && std::strcmp(argv[1], "host") == 0) return host_mode();
    if (argc >= 3 && std::strcmp(argv[1], "gpu") == 0) return gpu_mode(argv[2]);
    std::fprintf(stderr, "usage: %s host | gpu <file>\n", argv[0]);
    return 2;
}
