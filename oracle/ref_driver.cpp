// Driver around the reference's own LlamaRuntime — TEST INFRASTRUCTURE ONLY.
//
// Linked against the reference sources (src/inference_v2.cpp, src/quant_v2.cpp,
// src/gguf.cpp, src/tokenizer.cpp, src/compute_dot.cpp, src/cache.cpp,
// src/prefetch.cpp, src/half.cpp) compiled unmodified by oracle/Makefile.
// It produces the golden vectors the oracle restatement is pinned against and
// times the reference CPU decode loop for the benchmark's baseline arm.
//
// LlamaRuntime::step()/sample() and pos_ are private in
// include/laic/inference.hpp:29-33; this test driver reaches them by compiling
// that header with `private` defined as `public` (after every standard header
// it uses has been included normally), so the id-prompted workloads can run
// without going through the text tokenizer — the same per-token loop as
// generate_ids (src/inference_v2.cpp:34) minus the EOS stop.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <functional>
#include <iostream>
#include <limits>
#include <numeric>
#include <random>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>
#include <variant>
#include <vector>
#define private public
#include "laic/inference.hpp"
#undef private
#include "laic/quant_v2.hpp"

namespace {

std::vector<uint32_t> read_u32(const std::string& path) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) throw std::runtime_error("cannot open " + path);
    size_t n = size_t(f.tellg()) / 4;
    std::vector<uint32_t> v(n);
    f.seekg(0);
    f.read(reinterpret_cast<char*>(v.data()), std::streamsize(n * 4));
    return v;
}

void write_bytes(const std::string& path, const void* p, size_t n) {
    std::ofstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot write " + path);
    f.write(static_cast<const char*>(p), std::streamsize(n));
}

struct Args {
    std::unordered_map<std::string, std::string> kv;
    std::string get(const std::string& k, const std::string& fb = "") const {
        auto it = kv.find(k); return it == kv.end() ? fb : it->second;
    }
};

Args parse(int argc, char** argv, int from) {
    Args a;
    for (int i = from; i + 1 < argc; i += 2) a.kv[argv[i]] = argv[i + 1];
    return a;
}

void reset(laic::LlamaRuntime& rt) {
    rt.cache_.assign(rt.layers_, {});
    rt.pos_ = 0;
}

laic::GenerationConfig config(const Args& a) {
    laic::GenerationConfig c;
    c.temperature = std::stof(a.get("--temperature", "0"));
    c.top_k = std::stoul(a.get("--top-k", "0"));
    c.top_p = std::stof(a.get("--top-p", "1"));
    c.repeat_penalty = std::stof(a.get("--repeat-penalty", "1"));
    c.seed = std::stoull(a.get("--seed", "0"));
    return c;
}

// dump MODEL --prompt ids.u32 --steps N [sampling flags] --out PREFIX
//   PREFIX.ids.u32      generated ids (no EOS stop)
//   PREFIX.logits.f32   [prompt_len + steps - 1][vocab] logits of every step() call
int cmd_dump(const std::string& model, const Args& a) {
    laic::LlamaRuntime rt;
    rt.load(model);
    reset(rt);
    auto prompt = read_u32(a.get("--prompt"));
    size_t steps = std::stoul(a.get("--steps", "8"));
    bool all_logits = a.get("--all-logits", "1") == "1";
    auto cfg = config(a);
    std::vector<uint32_t> hist = prompt, ids;
    std::vector<float> logits, dump;
    for (uint32_t id : prompt) {
        logits = rt.step(id);
        ++rt.pos_;
        if (all_logits) dump.insert(dump.end(), logits.begin(), logits.end());
    }
    for (size_t s = 0; s < steps; ++s) {
        uint32_t next = rt.sample(logits, cfg, hist);
        ids.push_back(next);
        hist.push_back(next);
        if (s + 1 < steps) {
            logits = rt.step(next);
            ++rt.pos_;
            dump.insert(dump.end(), logits.begin(), logits.end());
        }
    }
    std::string out = a.get("--out");
    write_bytes(out + ".ids.u32", ids.data(), ids.size() * 4);
    write_bytes(out + ".logits.f32", dump.data(), dump.size() * 4);
    std::printf("{\"vocab\": %zu, \"l1_tile_bytes\": %zu, \"threads\": %zu}\n", rt.tokenizer().vocab_size(),
                rt.cache_plan_.l1_tile_bytes, size_t(std::thread::hardware_concurrency()));
    return 0;
}

// time MODEL --prompt ids.u32 --warmup W --steps K : decode-step wall time after the prompt
int cmd_time(const std::string& model, const Args& a) {
    laic::LlamaRuntime rt;
    rt.load(model);
    reset(rt);
    auto prompt = read_u32(a.get("--prompt"));
    size_t warm = std::stoul(a.get("--warmup", "1")), steps = std::stoul(a.get("--steps", "8"));
    auto cfg = config(a);
    std::vector<uint32_t> hist = prompt;
    std::vector<float> logits;
    auto t0 = std::chrono::steady_clock::now();
    for (uint32_t id : prompt) { logits = rt.step(id); ++rt.pos_; }
    auto t1 = std::chrono::steady_clock::now();
    double timed = 0;
    std::vector<double> per;
    for (size_t s = 0; s < warm + steps; ++s) {
        auto a0 = std::chrono::steady_clock::now();
        uint32_t next = rt.sample(logits, cfg, hist);
        hist.push_back(next);
        logits = rt.step(next);
        ++rt.pos_;
        auto a1 = std::chrono::steady_clock::now();
        if (s >= warm) { double dt = std::chrono::duration<double>(a1 - a0).count(); timed += dt; per.push_back(dt); }
    }
    std::printf("{\"prefill_s\": %.6f, \"prompt\": %zu, \"steps\": %zu, \"decode_s\": %.6f, \"tok_s\": %.4f, "
                "\"threads\": %u, \"pos\": %zu}\n",
                std::chrono::duration<double>(t1 - t0).count(), prompt.size(), steps, timed,
                steps / std::max(timed, 1e-12), std::thread::hardware_concurrency(), rt.pos_);
    return 0;
}

// dequant MODEL TENSOR OUT.f32 : quant_v2::value / GgufTensor::value over the whole tensor
int cmd_dequant(const std::string& model, const std::string& name, const std::string& out) {
    laic::GgufModel m;
    m.load(model);
    const auto& t = m.tensor(name);
    std::vector<float> v(t.elements());
    bool scalar = t.type == laic::GgmlType::F16 || t.type == laic::GgmlType::F32;
    for (size_t i = 0; i < v.size(); ++i) v[i] = scalar ? t.value(i) : laic::quant_v2::value(t.type, t.data, i);
    write_bytes(out, v.data(), v.size() * 4);
    return 0;
}

// encode MODEL TEXT : token ids of the reference tokenizer, one per line
int cmd_encode(const std::string& model, const std::string& text) {
    laic::GgufModel m;
    m.load(model);
    laic::Gpt2Tokenizer tok;
    tok.load(m);
    for (uint32_t id : tok.encode(text)) std::printf("%u\n", id);
    return 0;
}

// generate MODEL PROMPT_TEXT N : the public generate_ids path, ids one per line
int cmd_generate(const std::string& model, const std::string& text, const Args& a) {
    laic::LlamaRuntime rt;
    rt.load(model);
    auto cfg = config(a);
    cfg.max_tokens = std::stoul(a.get("--max-tokens", "8"));
    for (uint32_t id : rt.generate_ids(text, cfg)) std::printf("%u\n", id);
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 3) {
        std::fprintf(stderr, "usage: %s dump|time|dequant|encode|generate MODEL ...\n", argv[0]);
        return 2;
    }
    try {
        std::string cmd = argv[1], model = argv[2];
        if (cmd == "dump") return cmd_dump(model, parse(argc, argv, 3));
        if (cmd == "time") return cmd_time(model, parse(argc, argv, 3));
        if (cmd == "dequant" && argc >= 5) return cmd_dequant(model, argv[3], argv[4]);
        if (cmd == "encode" && argc >= 4) return cmd_encode(model, argv[3]);
        if (cmd == "generate" && argc >= 4) return cmd_generate(model, argv[3], parse(argc, argv, 4));
        std::fprintf(stderr, "bad command\n");
        return 2;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "ref_driver: %s\n", e.what());
        return 1;
    }
}
