// qwen2_chat -- the reference's line-protocol REPL (worker/src/chat_main.cpp)
// on the device model (include/qwen2_engine.h).
//
// Protocol, as chat_main.cpp:4-19:
//   stdin   one request per line: space-separated token ids; "EXIT" quits,
//           "RESET" clears the KV cache (answers "OK");
//   stdout  "READY" once the model is loaded, then per request
//           "OK <id1> <id2> ..." (the generated ids) or "ERR <message>";
//   stderr  per-request statistics.
// Every request is a single turn: the cache is cleared first
// (chat_main.cpp:101-102), then LLMEngine::generate's loop runs with the
// default GenerationConfig stop tokens {151645, 151643} and repetition
// window 6 (generation_config.h:9-25) and max_new_tokens from the command
// line (default 128).
//
// Usage: qwen2_chat <model_dir> [max_new_tokens]
//   <model_dir>/model.safetensors holds the weights; an optional
//   <model_dir>/config.json (Hugging Face keys hidden_size,
//   num_hidden_layers, num_attention_heads, num_key_value_heads,
//   intermediate_size, vocab_size, rms_norm_eps, rope_theta, plus
//   max_position for the KV capacity) overrides Qwen2Config's defaults.
//   QWEN2_DEVICE selects the GPU (default 0).
#include <chrono>
#include <csignal>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "qwen2_engine.h"

namespace {

qw2_model* g_model = nullptr;

void on_signal(int sig) {
    std::fprintf(stderr, "\n[qwen2_chat] signal %d: releasing the model\n", sig);
    if (g_model) qw2_destroy(g_model);
    g_model = nullptr;
    std::_Exit(0);
}

std::vector<int> parse_ids(const std::string& line) {  // chat_main.cpp:44-50
    std::vector<int> ids;
    std::istringstream iss(line);
    int v;
    while (iss >> v) ids.push_back(v);
    return ids;
}

// The number after "key": in a flat JSON object (config.json), if present.
bool json_number(const std::string& js, const char* key, double* out) {
    const std::string k = std::string("\"") + key + "\"";
    size_t p = js.find(k);
    if (p == std::string::npos) return false;
    p = js.find(':', p + k.size());
    if (p == std::string::npos) return false;
    const char* s = js.c_str() + p + 1;
    char* end = nullptr;
    const double v = std::strtod(s, &end);
    if (end == s) return false;
    *out = v;
    return true;
}

void read_config(const std::string& dir, qw2_config* c) {
    std::ifstream f(dir + "/config.json");
    if (!f) return;
    std::stringstream ss;
    ss << f.rdbuf();
    const std::string js = ss.str();
    double v;
    if (json_number(js, "hidden_size", &v)) c->hidden = (int)v;
    if (json_number(js, "num_hidden_layers", &v)) c->layers = (int)v;
    if (json_number(js, "num_attention_heads", &v)) c->q_heads = (int)v;
    if (json_number(js, "num_key_value_heads", &v)) c->kv_heads = (int)v;
    if (json_number(js, "intermediate_size", &v)) c->intermediate = (int)v;
    if (json_number(js, "vocab_size", &v)) c->vocab = (int)v;
    if (json_number(js, "rms_norm_eps", &v)) c->rms_eps = (float)v;
    if (json_number(js, "rope_theta", &v)) c->rope_theta = (float)v;
    if (json_number(js, "max_position", &v)) c->max_position = (int)v;
    if (c->q_heads > 0) c->head_dim = c->hidden / c->q_heads;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "Usage: %s <model_dir> [max_new_tokens]\n", argv[0]);
        return 1;
    }
    std::signal(SIGINT, on_signal);
    std::signal(SIGTERM, on_signal);
    const std::string dir = argv[1];
    const int max_new = argc >= 3 ? std::atoi(argv[2]) : 128;
    const char* dev_env = std::getenv("QWEN2_DEVICE");
    const int device = dev_env ? std::atoi(dev_env) : 0;

    qw2_config cfg;
    qw2_config_default(&cfg);
    read_config(dir, &cfg);
    std::fprintf(stderr, "[qwen2_chat] loading %s\n", dir.c_str());
    if (qw2_create(device, &cfg, &g_model) != KV_OK ||
        qw2_load_safetensors(g_model, (dir + "/model.safetensors").c_str()) != KV_OK ||
        qw2_ready(g_model) != KV_OK) {
        std::fprintf(stderr, "[qwen2_chat] load failed: %s\n", kv_last_error());
        if (g_model) qw2_destroy(g_model);
        return 1;
    }
    std::fprintf(stderr, "[qwen2_chat] ready (max_new_tokens = %d)\n", max_new);
    std::printf("READY\n");
    std::fflush(stdout);

    const int stops[2] = {151645, 151643};
    const qw2_gen_config gen = {max_new, 6, stops, 2};
    std::vector<int> out((size_t)(max_new > 0 ? max_new : 1));
    std::string line;
    while (std::getline(std::cin, line)) {
        const size_t a = line.find_first_not_of(" \t\r\n");
        const size_t b = line.find_last_not_of(" \t\r\n");
        if (a == std::string::npos) continue;
        line = line.substr(a, b - a + 1);
        if (line == "EXIT") break;
        if (line == "RESET") {
            if (qw2_reset(g_model) == KV_OK) std::printf("OK\n");
            else std::printf("ERR %s\n", kv_last_error());
            std::fflush(stdout);
            continue;
        }
        const std::vector<int> ids = parse_ids(line);
        if (ids.empty()) {
            std::printf("ERR empty_input\n");
            std::fflush(stdout);
            continue;
        }
        qw2_result res{};
        int rc = qw2_reset(g_model);  // a single turn: a fresh cache
        if (rc == KV_OK)
            rc = qw2_generate_session(g_model, 0, ids.data(), (int)ids.size(), &gen, out.data(), (int)out.size(), &res);
        if (rc == KV_OK) rc = res.status;
        if (rc != KV_OK) {
            std::printf("ERR %s\n", kv_last_error());
            std::fflush(stdout);
            continue;
        }
        std::printf("OK");
        for (int i = 0; i < res.n_out && i < (int)out.size(); ++i) std::printf(" %d", out[i]);
        std::printf("\n");
        std::fprintf(stderr, "[qwen2_chat] prefill=%d tok %.0f ms, decode=%d tok %.0f ms (%.2f tok/s) stop=%s\n",
                     res.prefill_tokens, res.prefill_ms, res.decode_tokens, res.decode_ms,
                     res.decode_ms > 0 ? res.decode_tokens / (res.decode_ms / 1000.0f) : 0.0f,
                     res.hit_stop ? "eos" : res.hit_repetition ? "repetition" : "max_tokens");
        std::fflush(stdout);
    }
    qw2_destroy(g_model);
    g_model = nullptr;
    std::fprintf(stderr, "[qwen2_chat] exit\n");
    return 0;
}
