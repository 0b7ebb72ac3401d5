// Exercises the C++ host surface (include/laic/gguf.hpp, tokenizer.hpp) without a GPU.
//   host_check MODEL enc TEXT        token ids, one per line
//   host_check MODEL dec ID...       decoded bytes as hex, one line per id
//   host_check MODEL val TENSOR I... GgufTensor::value, one per line
//   host_check MODEL meta            vocab, bos, eos, add_bos, tensor count
//   host_check MODEL gen TEXT MAX [TEMP TOPK TOPP PENALTY SEED]
//                                    LlamaRuntime::generate_ids on the GPU, one id per line
#include <cstdio>
#include <cstdlib>
#include <string>

#include "laic/gguf.hpp"
#include "laic/inference.hpp"
#include "laic/tokenizer.hpp"

int main(int argc, char** argv) {
    if (argc < 3) return 2;
    try {
        laic::GgufModel m;
        m.load(argv[1]);
        laic::Gpt2Tokenizer tok;
        tok.load(m);
        const std::string cmd = argv[2];
        if (cmd == "gen" && argc > 4) {
            laic::LlamaRuntime rt;
            rt.load(argv[1]);
            laic::GenerationConfig cfg;
            cfg.max_tokens = size_t(std::atoll(argv[4]));
            if (argc > 9) {
                cfg.temperature = float(std::atof(argv[5]));
                cfg.top_k = size_t(std::atoll(argv[6]));
                cfg.top_p = float(std::atof(argv[7]));
                cfg.repeat_penalty = float(std::atof(argv[8]));
                cfg.seed = uint64_t(std::strtoull(argv[9], nullptr, 10));
            }
            for (uint32_t id : rt.generate_ids(argv[3], cfg)) std::printf("%u\n", id);
        } else if (cmd == "enc" && argc > 3) {
            for (uint32_t id : tok.encode(argv[3])) std::printf("%u\n", id);
        } else if (cmd == "dec") {
            for (int i = 3; i < argc; ++i) {
                for (unsigned char c : tok.decode(uint32_t(std::atoi(argv[i])))) std::printf("%02x", c);
                std::printf("\n");
            }
        } else if (cmd == "val" && argc > 4) {
            const auto& t = m.tensor(argv[3]);
            for (int i = 4; i < argc; ++i) std::printf("%.9g\n", t.value(size_t(std::atoll(argv[i]))));
        } else if (cmd == "meta") {
            std::printf("%zu %u %u %d %zu %s\n", tok.vocab_size(), tok.bos_id(), tok.eos_id(), int(tok.add_bos()),
                        m.tensors().size(), m.str("general.architecture").c_str());
        } else {
            return 2;
        }
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "host_check: %s\n", e.what());
        return 1;
    }
}
