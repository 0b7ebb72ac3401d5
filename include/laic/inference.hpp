// Llama decode runtime: the reference's public C++ API (reference
// include/laic/inference.hpp:11-22), with the forward pass and the token
// choice on a B200 through the C ABI of laic_b200.h instead of host threads.
//
// Device selection comes from the environment: LAIC_DEVICE (CUDA ordinal,
// default 0) and LAIC_KV_F32=1 (FP32 KV cache, the reference's precision).
#pragma once
#include <atomic>
#include <cstdint>
#include <functional>
#include <string>
#include <vector>

#include "laic/gguf.hpp"
#include "laic/tokenizer.hpp"

struct laic_dev;

namespace laic {

struct GenerationConfig {
    size_t max_tokens = 32;
    float temperature = 0.0f;
    size_t top_k = 0;
    float top_p = 1.0f;
    float repeat_penalty = 1.0f;
    uint64_t seed = 0;
};

class LlamaRuntime {
public:
    using TokenCallback = std::function<bool(uint32_t)>;
    LlamaRuntime() = default;
    ~LlamaRuntime();
    LlamaRuntime(const LlamaRuntime&) = delete;
    LlamaRuntime& operator=(const LlamaRuntime&) = delete;

    void load(const std::string& path);
    std::vector<uint32_t> generate_ids(const std::string& prompt, const GenerationConfig& cfg = {});
    std::vector<uint32_t> generate_ids(const std::string& prompt, const GenerationConfig& cfg,
                                       const TokenCallback& callback);
    std::string generate(const std::string& prompt, const GenerationConfig& cfg = {});
    void request_stop() noexcept { stop_requested_.store(true, std::memory_order_relaxed); }
    bool stop_requested() const noexcept { return stop_requested_.load(std::memory_order_relaxed); }
    const GgufModel& model() const noexcept { return model_; }
    const Gpt2Tokenizer& tokenizer() const noexcept { return tokenizer_; }

    // Token-id entry used by tests and tools (no text template or tokenizer):
    // prompt ids in, generated ids out, same loop as generate_ids.
    std::vector<uint32_t> generate_from_ids(const std::vector<uint32_t>& ids, const GenerationConfig& cfg,
                                            const TokenCallback& callback = {});

private:
    GgufModel model_;
    Gpt2Tokenizer tokenizer_;
    std::atomic<bool> stop_requested_{false};
    laic_dev* dev_ = nullptr;
    size_t hidden_ = 0, layers_ = 0, heads_ = 0, kv_heads_ = 0, head_dim_ = 0, ffn_ = 0, ctx_ = 0, rope_dim_ = 0;
    float eps_ = 1e-5f, theta_ = 10000.f;
};

}  // namespace laic
