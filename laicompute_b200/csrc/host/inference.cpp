// LlamaRuntime (reference src/inference_v2.cpp:27-35) on the B200 engine.
//
// load() validates the llama.* metadata exactly as the reference does and
// uploads every tensor the decode path reads; generate_ids() keeps the
// reference's loop (chat-template wrap, encode, BOS, one step per prompt
// token, sample -> EOS check -> callback -> step) but each step is one call
// into the device engine, which returns the sampled id. The prompt's tokens
// before the last one go through laic_dev_prefill_batch in one pass (their
// logits are never read); the last prompt token and every generated token go
// through laic_dev_step (forward pass + sampling). The reference computes one more
// forward pass after the final generated token whose logits it never uses;
// that pass is skipped.
#include "laic/inference.hpp"

#include <cstdlib>
#include <stdexcept>

#include "laic_b200.h"

namespace laic {
namespace {

[[noreturn]] void raise() { throw std::runtime_error(laic_last_error()); }
void check(int rc) {
    if (rc != LAIC_OK) raise();
}

int env_int(const char* name, int fallback) {
    const char* v = std::getenv(name);
    return v && *v ? std::atoi(v) : fallback;
}

}  // namespace

LlamaRuntime::~LlamaRuntime() {
    if (dev_) laic_dev_destroy(dev_);
}

void LlamaRuntime::load(const std::string& path) {
    stop_requested_.store(false, std::memory_order_relaxed);
    if (dev_) { laic_dev_destroy(dev_); dev_ = nullptr; }
    model_.load(path);
    if (model_.str("general.architecture", "") != "llama")
        throw std::runtime_error("unsupported architecture: expected llama-family GGUF");
    hidden_ = model_.u64("llama.embedding_length");
    layers_ = model_.u64("llama.block_count");
    heads_ = model_.u64("llama.attention.head_count");
    kv_heads_ = model_.u64("llama.attention.head_count_kv", heads_);
    ffn_ = model_.u64("llama.feed_forward_length");
    ctx_ = model_.u64("llama.context_length", 2048);
    rope_dim_ = model_.u64("llama.rope.dimension_count", hidden_ / (heads_ ? heads_ : 1));
    theta_ = float(model_.f64("llama.rope.freq_base", 10000));
    eps_ = float(model_.f64("llama.attention.layer_norm_rms_epsilon", 1e-5));
    if (!hidden_ || !layers_ || !heads_ || !kv_heads_ || hidden_ % heads_ || heads_ % kv_heads_ || !ffn_)
        throw std::runtime_error("invalid llama architecture metadata");
    head_dim_ = hidden_ / heads_;
    if (!rope_dim_ || rope_dim_ > head_dim_ || (rope_dim_ & 1)) throw std::runtime_error("invalid RoPE dimension");
    tokenizer_.load(model_);
    if (!model_.has_tensor("token_embd.weight") || !model_.has_tensor("output_norm.weight"))
        throw std::runtime_error("missing required tensors");

    laic_dev_desc desc{};
    desc.hidden = uint32_t(hidden_); desc.layers = uint32_t(layers_); desc.heads = uint32_t(heads_);
    desc.kv_heads = uint32_t(kv_heads_); desc.ffn = uint32_t(ffn_); desc.vocab = uint32_t(tokenizer_.vocab_size());
    desc.ctx = uint32_t(ctx_); desc.rope_dim = uint32_t(rope_dim_); desc.rope_theta = theta_; desc.rms_eps = eps_;
    laic_dev_opts opts{};
    opts.device = env_int("LAIC_DEVICE", 0);
    opts.max_seqs = 1;
    opts.kv_capacity = 0;
    opts.tp_size = 1;
    opts.flags = env_int("LAIC_KV_F32", 0) ? LAIC_FLAG_KV_F32 : 0u;
    check(laic_dev_create(&desc, &opts, &dev_));

    std::vector<std::string> names = {"token_embd.weight", "output_norm.weight"};
    if (model_.has_tensor("output.weight")) names.push_back("output.weight");
    static const char* parts[] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                  "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};
    for (size_t l = 0; l < layers_; ++l)
        for (const char* p : parts) names.push_back("blk." + std::to_string(l) + "." + p + ".weight");
    for (const auto& n : names) {
        const GgufTensor& t = model_.tensor(n);  // throws "missing tensor: ..."
        check(laic_dev_upload(dev_, n.c_str(), int32_t(t.type), t.shape.data(), int32_t(t.shape.size()), t.data,
                              t.bytes()));
    }
}

std::vector<uint32_t> LlamaRuntime::generate_ids(const std::string& prompt, const GenerationConfig& cfg) {
    std::vector<uint32_t> out;
    generate_ids(prompt, cfg, [&](uint32_t id) { out.push_back(id); return true; });
    return out;
}

std::vector<uint32_t> LlamaRuntime::generate_ids(const std::string& prompt, const GenerationConfig& cfg,
                                                 const TokenCallback& cb) {
    stop_requested_.store(false, std::memory_order_relaxed);
    std::string input = prompt;
    const std::string templ = model_.str("tokenizer.chat_template", "");
    if (templ.find("<|im_start|>") != std::string::npos && input.find("<|im_start|>") == std::string::npos)
        input = "<|im_start|>user\n" + input + "<|im_end|>\n<|im_start|>assistant\n";
    std::vector<uint32_t> ids = tokenizer_.encode(input);
    if (ids.empty()) throw std::runtime_error("tokenization produced no tokens");
    if (tokenizer_.add_bos() && ids.front() != tokenizer_.bos_id()) ids.insert(ids.begin(), tokenizer_.bos_id());
    return generate_from_ids(ids, cfg, cb);
}

std::vector<uint32_t> LlamaRuntime::generate_from_ids(const std::vector<uint32_t>& ids, const GenerationConfig& cfg,
                                                      const TokenCallback& cb) {
    if (!dev_) throw std::runtime_error("model not loaded");
    if (ids.empty()) throw std::runtime_error("tokenization produced no tokens");
    stop_requested_.store(false, std::memory_order_relaxed);
    const int32_t slot = 0;
    check(laic_dev_reset_slot(dev_, slot));
    if (ids.size() > 1) {
        if (stop_requested()) throw std::runtime_error("generation stopped");
        check(laic_dev_prefill_batch(dev_, slot, ids.data(), int32_t(ids.size() - 1)));
    }
    laic_sample_params sp{cfg.temperature, uint32_t(cfg.top_k), cfg.top_p, cfg.repeat_penalty, cfg.seed};
    std::vector<uint32_t> generated;
    generated.reserve(cfg.max_tokens);
    if (cfg.max_tokens == 0) return generated;
    if (stop_requested()) throw std::runtime_error("generation stopped");
    uint32_t next = 0;
    check(laic_dev_step(dev_, 1, &ids.back(), &slot, &sp, 1, &next, nullptr));
    for (size_t n = 0; n < cfg.max_tokens; ++n) {
        if (stop_requested()) break;
        if (next == tokenizer_.eos_id()) break;
        generated.push_back(next);
        if (cb && !cb(next)) break;
        if (n + 1 == cfg.max_tokens) break;
        const uint32_t tok = next;
        check(laic_dev_step(dev_, 1, &tok, &slot, &sp, 1, &next, nullptr));
    }
    return generated;
}

std::string LlamaRuntime::generate(const std::string& prompt, const GenerationConfig& cfg) {
    std::string out;
    generate_ids(prompt, cfg, [&](uint32_t id) { out += tokenizer_.decode(id); return true; });
    return out;
}

}  // namespace laic
