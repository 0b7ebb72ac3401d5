// CPU restatement of the reference decode path — TEST INFRASTRUCTURE ONLY.
//
// This file is the parity oracle for the B200 engine. Only the tests, the
// smoke check and the CPU-baseline leg of the benchmark load it; the engine
// never links or calls it.
//
// It restates, operation by operation and in the same floating-point order,
// the reference CPU path of LAICompute:
//   * block dequantisation     src/quant_v2.cpp:9-10   (Q8_0, Q4_0)
//   * binary16 decode          src/half.cpp:30-51, src/compute_dot.cpp:9-25
//   * GGUF parsing             src/gguf.cpp:9-18
//   * row dot products         src/inference_v2.cpp:21-22, src/compute_dot.cpp:45-62
//   * rmsnorm / rope / silu    src/inference_v2.cpp:23-25
//   * matvec / embedding       src/inference_v2.cpp:28-29
//   * step (forward pass)      src/inference_v2.cpp:31
//   * sample                   src/inference_v2.cpp:32
// Compiled without -ffast-math and with -ffp-contract=off, every row sum is
// the same sequential float recurrence as the reference, so results are
// bit-identical to the reference's strict (-O3, non-native) build; the tests
// pin that against fixtures produced by the reference itself.
#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <limits>
#include <numeric>
#include <random>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>
#include <unistd.h>

namespace {

enum : uint32_t { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8 };

// Exact binary16 -> float (src/half.cpp:30-51).
float half_to_float(uint16_t h) {
    uint32_t sign = uint32_t(h & 0x8000u) << 16, exp = (h >> 10) & 0x1fu, mant = h & 0x3ffu, out;
    if (exp == 0) {
        if (mant == 0) out = sign;
        else {
            exp = 1;
            while ((mant & 0x400u) == 0) { mant <<= 1; --exp; }
            mant &= 0x3ffu;
            out = sign | ((exp + 112u) << 23) | (mant << 13);
        }
    } else if (exp == 0x1fu) out = sign | 0x7f800000u | (mant << 13);
    else out = sign | ((exp + 112u) << 23) | (mant << 13);
    float f; std::memcpy(&f, &out, 4); return f;
}
inline float h16(const uint8_t* p) { return half_to_float(uint16_t(p[0]) | (uint16_t(p[1]) << 8)); }

size_t block_bytes(uint32_t t) {
    switch (t) {
    case T_F32: return 4; case T_F16: return 2; case T_Q4_0: return 18; case T_Q8_0: return 34;
    case T_Q4_1: return 20; case T_Q5_0: return 22; case T_Q5_1: return 24;
    }
    throw std::runtime_error("unsupported GGML type");
}

// One element of a tensor (quant_v2::value for Q8_0/Q4_0/Q4_1/Q5_0/Q5_1, GgufTensor::value for F16/F32).
inline float value(uint32_t type, const uint8_t* data, size_t i) {
    switch (type) {
    case T_F32: { float v; std::memcpy(&v, data + i * 4, 4); return v; }
    case T_F16: return h16(data + i * 2);
    case T_Q8_0: { const uint8_t* p = data + (i / 32) * 34; return h16(p) * float(int8_t(p[2 + i % 32])); }
    case T_Q4_0: {
        const uint8_t* p = data + (i / 32) * 18; size_t o = i % 32; uint8_t z = p[2 + o / 2];
        return h16(p) * float(((o & 1) ? (z >> 4) : (z & 15)) - 8);
    }
    // src/quant_v2.cpp:11 (Q4_1: d * q + m), :12 (Q5_0: d * (v - 16)), :13 (Q5_1: d * v + m); the
    // fifth bit of element o is bit o of the 32-bit qh that follows the scale(s)
    case T_Q4_1: {
        const uint8_t* p = data + (i / 32) * 20; size_t o = i % 32; uint8_t z = p[4 + o / 2];
        return h16(p) * float((o & 1) ? (z >> 4) : (z & 15)) + h16(p + 2);
    }
    case T_Q5_0: {
        const uint8_t* p = data + (i / 32) * 22; size_t o = i % 32; uint32_t qh; std::memcpy(&qh, p + 2, 4);
        uint8_t z = p[6 + o / 2]; int v = ((o & 1) ? (z >> 4) : (z & 15)) | int(((qh >> o) & 1u) << 4);
        return h16(p) * float(v - 16);
    }
    case T_Q5_1: {
        const uint8_t* p = data + (i / 32) * 24; size_t o = i % 32; uint32_t qh; std::memcpy(&qh, p + 4, 4);
        uint8_t z = p[8 + o / 2]; int v = ((o & 1) ? (z >> 4) : (z & 15)) | int(((qh >> o) & 1u) << 4);
        return h16(p) * float(v) + h16(p + 2);
    }
    }
    throw std::runtime_error("unsupported quantized GGML type");
}

size_t detect_l1d() {
    size_t l1 = 0;
    long v = sysconf(_SC_LEVEL1_DCACHE_SIZE);
    if (v > 0) l1 = size_t(v);
    for (int idx = 0; idx < 16; ++idx) {
        std::string base = "/sys/devices/system/cpu/cpu0/cache/index" + std::to_string(idx) + "/";
        std::ifstream lf(base + "level"), tf(base + "type"), sf(base + "size");
        std::string ls, ts, ss;
        if (!std::getline(lf, ls) || !std::getline(tf, ts) || !std::getline(sf, ss)) continue;
        if (ls != "1" || ts != "Data" || ss.empty()) continue;
        size_t n = std::stoull(ss);
        if (ss.back() == 'K' || ss.back() == 'k') n *= 1024;
        if (ss.back() == 'M' || ss.back() == 'm') n *= 1024 * 1024;
        l1 = std::max(l1, n);
    }
    return l1;
}

// f(i) for i < n over a persistent pool of host threads when the job is large
// enough to repay waking them (`work` = elements one call of f touches); rows
// are handed out in chunks, and which thread runs a row never changes its result.
class RowPool {
public:
    static RowPool& get() { static RowPool p; return p; }
    size_t threads() const { return workers_.size() + 1; }
    template <class F>
    void run(size_t n, F& f) {
        std::unique_lock<std::mutex> job_lock(job_mu_);  // one job at a time
        {
            std::lock_guard<std::mutex> lk(mu_);
            fn_ = [&f](size_t i) { f(i); };
            n_ = n;
            chunk_ = std::max<size_t>(1, n / (4 * threads()));
            next_.store(0);
            busy_ = workers_.size();
            ++gen_;
        }
        cv_.notify_all();
        drain();
        std::unique_lock<std::mutex> lk(mu_);
        done_cv_.wait(lk, [&] { return busy_ == 0; });
    }
    ~RowPool() {
        { std::lock_guard<std::mutex> lk(mu_); stop_ = true; ++gen_; }
        cv_.notify_all();
        for (auto& t : workers_) t.join();
    }

private:
    RowPool() {
        const size_t nt = std::max(1u, std::thread::hardware_concurrency());
        for (size_t t = 1; t < nt; ++t) workers_.emplace_back([this] { loop(); });
    }
    void drain() {
        for (;;) {
            const size_t i0 = next_.fetch_add(chunk_);
            if (i0 >= n_) return;
            const size_t i1 = std::min(n_, i0 + chunk_);
            for (size_t i = i0; i < i1; ++i) fn_(i);
        }
    }
    void loop() {
        uint64_t seen = 0;
        for (;;) {
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return gen_ != seen; });
                seen = gen_;
                if (stop_) return;
            }
            drain();
            std::lock_guard<std::mutex> lk(mu_);
            if (--busy_ == 0) done_cv_.notify_one();
        }
    }
    std::vector<std::thread> workers_;
    std::mutex job_mu_, mu_;
    std::condition_variable cv_, done_cv_;
    std::function<void(size_t)> fn_;
    size_t n_ = 0, chunk_ = 1, busy_ = 0;
    std::atomic<size_t> next_{0};
    uint64_t gen_ = 0;
    bool stop_ = false;
};

template <class F>
void parallel_rows(size_t n, F&& f, size_t work = 1) {
    RowPool& pool = RowPool::get();
    if (n < 2 || pool.threads() == 1 || n * work < (size_t(1) << 15)) { for (size_t i = 0; i < n; ++i) f(i); return; }
    pool.run(n, f);
}

// Row dot product: dot_cached for F16/F32 (chunks of l1_tile_bytes/(2*sb) elements,
// each summed sequentially, then added into s), quant_dot for block types.
float row_dot(uint32_t type, const uint8_t* w, const float* x, size_t base, size_t n, size_t l1_tile_bytes) {
    if (type == T_F16 || type == T_F32) {
        const size_t sb = type == T_F16 ? 2 : 4;
        size_t tile = l1_tile_bytes / (sb * 2);
        if (!tile) tile = 32;
        float s = 0.f;
        for (size_t j = 0; j < n; j += tile) {
            size_t len = std::min(tile, n - j);
            const uint8_t* wp = w + (base + j) * sb;
            float c = 0.f;
            if (type == T_F16) for (size_t i = 0; i < len; ++i) c += h16(wp + 2 * i) * x[j + i];
            else for (size_t i = 0; i < len; ++i) { float v; std::memcpy(&v, wp + 4 * i, 4); c += x[j + i] * v; }
            s += c;
        }
        return s;
    }
    float s = 0.f;
    for (size_t i = 0; i < n; ++i) s += value(type, w, base + i) * x[i];
    return s;
}

struct Tensor {
    std::vector<uint64_t> shape;
    uint32_t type = 0;
    const uint8_t* data = nullptr;
    size_t elements() const { size_t n = 1; for (auto d : shape) n *= size_t(d); return n; }
};

struct Reader {
    const uint8_t* p; const uint8_t* e;
    void need(size_t n) { if (n > size_t(e - p)) throw std::runtime_error("invalid/truncated GGUF"); }
    uint8_t u8() { need(1); return *p++; }
    uint16_t u16() { need(2); uint16_t v = p[0] | (uint16_t(p[1]) << 8); p += 2; return v; }
    uint32_t u32() { need(4); uint32_t v; std::memcpy(&v, p, 4); p += 4; return v; }
    uint64_t u64() { need(8); uint64_t v; std::memcpy(&v, p, 8); p += 8; return v; }
    std::string str() { uint64_t n = u64(); need(n); std::string s((const char*)p, size_t(n)); p += n; return s; }
};

struct Meta { bool is_num = false; double num = 0; std::string s; size_t arr_len = 0; };

Meta read_value(Reader& r, uint32_t t) {
    Meta m; m.is_num = true;
    switch (t) {
    case 0: m.num = r.u8(); break;
    case 1: m.num = int8_t(r.u8()); break;
    case 2: m.num = r.u16(); break;
    case 3: m.num = int16_t(r.u16()); break;
    case 4: m.num = r.u32(); break;
    case 5: m.num = int32_t(r.u32()); break;
    case 6: { uint32_t x = r.u32(); float f; std::memcpy(&f, &x, 4); m.num = f; break; }
    case 7: m.num = r.u8() != 0; break;
    case 8: m.is_num = false; m.s = r.str(); break;
    case 10: m.num = double(r.u64()); break;
    case 11: m.num = double(int64_t(r.u64())); break;
    case 12: { uint64_t x = r.u64(); double d; std::memcpy(&d, &x, 8); m.num = d; break; }
    case 9: {
        m.is_num = false;
        uint32_t et = r.u32(); uint64_t n = r.u64(); m.arr_len = size_t(n);
        for (uint64_t i = 0; i < n; ++i) read_value(r, et);
        break;
    }
    default: throw std::runtime_error("unsupported GGUF metadata type");
    }
    return m;
}

struct Model {
    std::vector<uint8_t> file;
    std::unordered_map<std::string, Meta> meta;
    std::unordered_map<std::string, Tensor> tensors;
    size_t hidden = 0, layers = 0, heads = 0, kv_heads = 0, head_dim = 0, ffn = 0, ctx = 0, rope_dim = 0, vocab = 0, pos = 0;
    float eps = 1e-5f, theta = 10000.f;
    size_t l1_tile_bytes = 0;
    struct LayerCache { std::vector<float> k, v; };
    std::vector<LayerCache> cache;

    double num(const std::string& k, double fb) const {
        auto it = meta.find(k); return (it == meta.end() || !it->second.is_num) ? fb : it->second.num;
    }
    const Tensor& tensor(const std::string& n) const {
        auto it = tensors.find(n);
        if (it == tensors.end()) throw std::runtime_error("missing tensor: " + n);
        return it->second;
    }
    bool has(const std::string& n) const { return tensors.count(n) != 0; }

    void load(const std::string& path) {
        std::ifstream f(path, std::ios::binary | std::ios::ate);
        if (!f) throw std::runtime_error("cannot open GGUF: " + path);
        auto sz = f.tellg();
        file.resize(size_t(sz));
        f.seekg(0);
        f.read((char*)file.data(), std::streamsize(file.size()));
        Reader r{file.data(), file.data() + file.size()};
        if (r.u32() != 0x46554747u) throw std::runtime_error("bad GGUF magic");
        uint32_t ver = r.u32();
        if (ver < 2 || ver > 3) throw std::runtime_error("unsupported GGUF version");
        uint64_t nt = r.u64(), nm = r.u64();
        for (uint64_t i = 0; i < nm; ++i) { std::string k = r.str(); uint32_t t = r.u32(); meta[k] = read_value(r, t); }
        struct Info { std::string name; std::vector<uint64_t> shape; uint32_t type; uint64_t off; };
        std::vector<Info> infos;
        for (uint64_t i = 0; i < nt; ++i) {
            Info x; x.name = r.str(); uint32_t nd = r.u32(); x.shape.resize(nd);
            for (auto& d : x.shape) d = r.u64();
            x.type = r.u32(); x.off = r.u64(); block_bytes(x.type); infos.push_back(x);
        }
        uint64_t align = uint64_t(num("general.alignment", 32));
        if (!align || align > 4096) align = 32;
        size_t raw = size_t(r.p - file.data());
        size_t start = (raw + align - 1) / align * align;
        for (auto& x : infos) {
            Tensor t; t.shape = x.shape; t.type = x.type; t.data = file.data() + start + x.off;
            tensors[x.name] = t;
        }
        auto arch = meta.find("general.architecture");
        if (arch == meta.end() || arch->second.s != "llama") throw std::runtime_error("unsupported architecture: expected llama-family GGUF");
        hidden = size_t(num("llama.embedding_length", 0));
        layers = size_t(num("llama.block_count", 0));
        heads = size_t(num("llama.attention.head_count", 0));
        kv_heads = size_t(num("llama.attention.head_count_kv", double(heads)));
        ffn = size_t(num("llama.feed_forward_length", 0));
        ctx = size_t(num("llama.context_length", 2048));
        rope_dim = size_t(num("llama.rope.dimension_count", double(hidden / std::max<size_t>(1, heads))));
        theta = float(num("llama.rope.freq_base", 10000));
        eps = float(num("llama.attention.layer_norm_rms_epsilon", 1e-5));
        if (!hidden || !layers || !heads || !kv_heads || hidden % heads || heads % kv_heads || !ffn)
            throw std::runtime_error("invalid llama architecture metadata");
        head_dim = hidden / heads;
        auto tok = meta.find("tokenizer.ggml.tokens");
        vocab = tok == meta.end() ? 0 : tok->second.arr_len;
        if (!vocab) throw std::runtime_error("GGUF has no tokenizer vocabulary");
        l1_tile_bytes = detect_l1d() / 2;
        reset();
    }
    void reset() { cache.assign(layers, {}); pos = 0; }

    std::vector<float> matvec(const Tensor& w, const std::vector<float>& x, size_t out, size_t in) const {
        if (w.shape.size() != 2 || w.shape[0] != in || w.shape[1] != out) throw std::runtime_error("unexpected weight shape");
        std::vector<float> y(out);
        // each row is one sequential sum on one thread: the split never changes a result
        parallel_rows(out, [&](size_t o) { y[o] = row_dot(w.type, w.data, x.data(), o * in, in, l1_tile_bytes); }, in);
        return y;
    }
    void norm(std::vector<float>& x, const Tensor& w) const {
        float ss = 0.f;
        for (float v : x) ss += v * v;
        float inv = 1.f / std::sqrt(ss / float(x.size()) + eps);
        for (size_t i = 0; i < x.size(); ++i) x[i] *= inv * value(w.type, w.data, i);
    }
    void rope(std::vector<float>& x, size_t nh) const {
        size_t rd = std::min(rope_dim, head_dim);
        for (size_t h = 0; h < nh; ++h)
            for (size_t i = 0; i < rd; i += 2) {
                float a = float(pos) * std::pow(theta, -float(i) / float(head_dim));
                float c = std::cos(a), s = std::sin(a);
                size_t b = h * head_dim + i;
                float u = x[b], v = x[b + 1];
                x[b] = u * c - v * s;
                x[b + 1] = u * s + v * c;
            }
    }
    std::vector<float> step(uint32_t token) {
        if (pos >= ctx) throw std::runtime_error("context length exceeded");
        const Tensor& e = tensor("token_embd.weight");
        if (e.shape.size() != 2 || e.shape[0] != hidden || token >= e.shape[1]) throw std::runtime_error("invalid embedding tensor");
        std::vector<float> x(hidden);
        for (size_t i = 0; i < hidden; ++i) x[i] = value(e.type, e.data, size_t(token) * hidden + i);
        const size_t kvd = kv_heads * head_dim, group = heads / kv_heads;
        for (size_t l = 0; l < layers; ++l) {
            std::string p = "blk." + std::to_string(l) + ".";
            auto a = x;
            norm(a, tensor(p + "attn_norm.weight"));
            auto q = matvec(tensor(p + "attn_q.weight"), a, hidden, hidden);
            auto k = matvec(tensor(p + "attn_k.weight"), a, kvd, hidden);
            auto v = matvec(tensor(p + "attn_v.weight"), a, kvd, hidden);
            rope(q, heads);
            rope(k, kv_heads);
            auto& lc = cache[l];
            lc.k.insert(lc.k.end(), k.begin(), k.end());
            lc.v.insert(lc.v.end(), v.begin(), v.end());
            std::vector<float> attn(hidden);
            parallel_rows(heads, [&](size_t h) {
                size_t kh = h / group;
                std::vector<float> scores(pos + 1);
                float mx = -std::numeric_limits<float>::infinity();
                for (size_t t = 0; t <= pos; ++t) {
                    float s = 0.f;
                    for (size_t d = 0; d < head_dim; ++d) s += q[h * head_dim + d] * lc.k[t * kvd + kh * head_dim + d];
                    scores[t] = s / std::sqrt(float(head_dim));
                    mx = std::max(mx, scores[t]);
                }
                float den = 0.f;
                for (float& s : scores) { s = std::exp(s - mx); den += s; }
                for (float& s : scores) s /= den;
                for (size_t d = 0; d < head_dim; ++d) {
                    float z = 0.f;
                    for (size_t t = 0; t <= pos; ++t) z += scores[t] * lc.v[t * kvd + kh * head_dim + d];
                    attn[h * head_dim + d] = z;
                }
            }, (pos + 1) * head_dim * 2);
            auto ao = matvec(tensor(p + "attn_output.weight"), attn, hidden, hidden);
            for (size_t i = 0; i < hidden; ++i) x[i] += 1.f * ao[i];
            auto f = x;
            norm(f, tensor(p + "ffn_norm.weight"));
            auto gate = matvec(tensor(p + "ffn_gate.weight"), f, ffn, hidden);
            auto up = matvec(tensor(p + "ffn_up.weight"), f, ffn, hidden);
            for (size_t i = 0; i < ffn; ++i) gate[i] = (gate[i] / (1.f + std::exp(-gate[i]))) * up[i];
            auto down = matvec(tensor(p + "ffn_down.weight"), gate, hidden, ffn);
            for (size_t i = 0; i < hidden; ++i) x[i] += 1.f * down[i];
        }
        norm(x, tensor("output_norm.weight"));
        const Tensor& out = has("output.weight") ? tensor("output.weight") : tensor("token_embd.weight");
        auto logits = matvec(out, x, vocab, hidden);
        ++pos;
        return logits;
    }
};

struct SampleParams { float temperature; uint32_t top_k; float top_p; float repeat_penalty; uint64_t seed; };

// LlamaRuntime::sample (src/inference_v2.cpp:32), with the same standard-library
// algorithms (nth_element order, mt19937_64 re-seeded per call, discrete_distribution).
uint32_t sample(const float* logits, size_t n, const SampleParams& c, const uint32_t* hist, size_t nh) {
    std::vector<float> l(logits, logits + n);
    if (c.repeat_penalty != 1.f)
        for (size_t j = 0; j < nh; ++j) {
            uint32_t id = hist[j];
            if (id < l.size()) { if (l[id] >= 0) l[id] /= c.repeat_penalty; else l[id] *= c.repeat_penalty; }
        }
    if (c.temperature <= 0.f) return uint32_t(std::max_element(l.begin(), l.end()) - l.begin());
    size_t k = c.top_k ? std::min<size_t>(c.top_k, l.size()) : l.size();
    std::vector<size_t> ix(l.size());
    std::iota(ix.begin(), ix.end(), 0);
    if (k < ix.size()) {
        std::nth_element(ix.begin(), ix.begin() + k, ix.end(), [&](size_t a, size_t b) { return l[a] > l[b]; });
        ix.resize(k);
    }
    float mx = -std::numeric_limits<float>::infinity();
    for (size_t i : ix) mx = std::max(mx, l[i]);
    std::vector<double> p(k);
    double sum = 0;
    for (size_t j = 0; j < k; ++j) { p[j] = std::exp((l[ix[j]] - mx) / c.temperature); sum += p[j]; }
    for (double& v : p) v /= sum;
    if (c.top_p < 1.f) {
        std::vector<size_t> ord(k);
        std::iota(ord.begin(), ord.end(), 0);
        std::sort(ord.begin(), ord.end(), [&](size_t a, size_t b) { return p[a] > p[b]; });
        double acc = 0; size_t keep = 0;
        for (size_t j : ord) { acc += p[j]; keep++; if (acc >= c.top_p) break; }
        std::vector<size_t> nix; std::vector<double> np;
        for (size_t j : ord) if (nix.size() < keep) { nix.push_back(ix[j]); np.push_back(p[j]); }
        double ns = 0;
        for (double v : np) ns += v;
        ix.swap(nix); p.swap(np);
        for (double& v : p) v /= ns;
    }
    std::mt19937_64 rng(c.seed ? c.seed : std::random_device{}());
    std::discrete_distribution<size_t> d(p.begin(), p.end());
    return uint32_t(ix[d(rng)]);
}

thread_local std::string g_err;

}  // namespace

extern "C" {

const char* oracle_last_error() { return g_err.c_str(); }

void* oracle_load(const char* path) {
    try { auto* m = new Model(); m->load(path); return m; }
    catch (const std::exception& e) { g_err = e.what(); return nullptr; }
}
void oracle_free(void* m) { delete static_cast<Model*>(m); }

// hidden, layers, heads, kv_heads, head_dim, ffn, ctx, rope_dim, vocab, l1_tile_bytes
void oracle_arch(void* mp, uint64_t* out) {
    auto* m = static_cast<Model*>(mp);
    uint64_t v[10] = {m->hidden, m->layers, m->heads, m->kv_heads, m->head_dim, m->ffn, m->ctx, m->rope_dim, m->vocab, m->l1_tile_bytes};
    std::memcpy(out, v, sizeof v);
}
void oracle_set_l1_tile_bytes(void* mp, uint64_t b) { static_cast<Model*>(mp)->l1_tile_bytes = size_t(b); }
void oracle_reset(void* mp) { static_cast<Model*>(mp)->reset(); }
uint64_t oracle_pos(void* mp) { return static_cast<Model*>(mp)->pos; }

int oracle_step(void* mp, uint32_t token, float* logits) {
    try {
        auto* m = static_cast<Model*>(mp);
        auto l = m->step(token);
        if (logits) std::memcpy(logits, l.data(), l.size() * 4);
        return 0;
    } catch (const std::exception& e) { g_err = e.what(); return 1; }
}

// Runs a prompt then `steps` decode steps without stopping on EOS. Writes the
// generated ids; logits of every decode step (the logits each id was sampled
// from) go to `all_logits` ([steps][vocab]) when it is non-null.
int oracle_generate(void* mp, const uint32_t* prompt, size_t n_prompt, size_t steps, const SampleParams* sp,
                    uint32_t* out_ids, float* all_logits) {
    try {
        auto* m = static_cast<Model*>(mp);
        m->reset();
        std::vector<uint32_t> hist(prompt, prompt + n_prompt);
        std::vector<float> logits;
        for (size_t i = 0; i < n_prompt; ++i) logits = m->step(prompt[i]);
        for (size_t s = 0; s < steps; ++s) {
            if (all_logits) std::memcpy(all_logits + s * m->vocab, logits.data(), m->vocab * 4);
            uint32_t next = sample(logits.data(), logits.size(), *sp, hist.data(), hist.size());
            out_ids[s] = next;
            hist.push_back(next);
            if (s + 1 < steps) logits = m->step(next);
        }
        return 0;
    } catch (const std::exception& e) { g_err = e.what(); return 1; }
}

uint32_t oracle_sample(const float* logits, size_t n, const SampleParams* sp, const uint32_t* hist, size_t nh) {
    return sample(logits, n, *sp, hist, nh);
}

float oracle_value(uint32_t type, const uint8_t* data, uint64_t i) { return value(type, data, size_t(i)); }

void oracle_dequant(uint32_t type, const uint8_t* data, uint64_t n, float* out) {
    for (size_t i = 0; i < size_t(n); ++i) out[i] = value(type, data, i);
}

// y[b][o] = row o of W (GGUF [in, out]) dotted with x[b] — LlamaRuntime::matvec per sequence.
void oracle_matvec(uint32_t type, const uint8_t* w, const float* x, float* y, uint64_t out, uint64_t in,
                   uint64_t batch, uint64_t l1_tile_bytes) {
    parallel_rows(size_t(out), [&](size_t o) {
        for (size_t b = 0; b < size_t(batch); ++b)
            y[b * out + o] = row_dot(type, w, x + b * in, o * size_t(in), size_t(in), size_t(l1_tile_bytes));
    }, size_t(in) * size_t(batch));
}

// The uniform draw discrete_distribution makes from a freshly seeded mt19937_64
// (generate_canonical<double,53>: one 64-bit output / 2^64, clamped below 1).
double oracle_canonical_u(uint64_t seed) {
    std::mt19937_64 rng(seed);
    return std::generate_canonical<double, std::numeric_limits<double>::digits>(rng);
}

uint64_t oracle_detect_l1d() { return detect_l1d(); }

}  // extern "C"
