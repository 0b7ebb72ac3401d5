// HTTP API server over the decode runtime: the reference's public class
// (reference include/laic/server.hpp, routes of src/server_runtime.cpp:29-39),
// serving a directory of GGUF models with generation on a B200 through
// laic::LlamaRuntime.
//
// Routes (HTTP/1.1, one request per connection, JSON bodies):
//   GET  /api/models         [{"name", "size", "loaded"}] of the directory's *.gguf
//   GET  /api/status         {"generating", "tokens", "tokens_per_sec", "cpu_percent",
//                             "ram_percent", "cpu_logical", "cpu_physical",
//                             "inference_threads", "loaded"}
//   POST /api/models/upload  body = GGUF bytes, X-Filename header -> 201 {"name", "size"}
//   POST /api/models/load    {"name"} -> {"ok": true}
//   POST /api/models/unload  -> {"ok": true} (409 while generating)
//   POST /api/stop           LlamaRuntime::request_stop() -> {"ok": true, "stopping": true}
//   POST /api/chat           {"message", "max_tokens"} -> {"text", "tokens", "tokens_per_sec", "stopped"}
//   POST /api/chat/stream    the same as server-sent events: one {"token", "tokens",
//                            "tokens_per_sec"} per token, then {"done": true, ...}
//   GET  /                   web/index_v2.html of the working directory (404 when absent)
// One generation at a time (409 otherwise); greedy, at most 2048 tokens.
#pragma once
#include <cstdint>
#include <memory>
#include <string>

namespace laic {

class ApiServer {
public:
    explicit ApiServer(uint16_t port = 8080, std::string model_dir = "models");
    ~ApiServer();
    ApiServer(const ApiServer&) = delete;
    ApiServer& operator=(const ApiServer&) = delete;
    // Listen on all interfaces and serve until stop(); throws std::runtime_error when the
    // socket cannot be opened, bound or listened on.
    void run();
    void stop() noexcept;

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

}  // namespace laic
