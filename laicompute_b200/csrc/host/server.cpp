// laic::ApiServer: the reference's HTTP API (routes of src/server_runtime.cpp:29-39)
// over this repository's LlamaRuntime. A plain blocking-socket HTTP/1.1 server:
// one detached thread per connection, one request per connection, one generation
// at a time. Model files live in one directory; loading a model builds a
// LlamaRuntime (weights uploaded to the GPU), unloading frees it.
#include "laic/server.hpp"

#include <netinet/in.h>
#include <sys/socket.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cctype>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <mutex>
#include <set>
#include <sstream>
#include <stdexcept>
#include <thread>
#include <utility>

#include "laic/inference.hpp"

namespace laic {
namespace {

namespace fs = std::filesystem;
using Clock = std::chrono::steady_clock;

// ---- minimal JSON: string quoting, and the two field kinds the API reads
std::string json_quote(const std::string& s) {
    std::string o = "\"";
    for (unsigned char ch : s) {
        switch (ch) {
        case '"': o += "\\\""; break;
        case '\\': o += "\\\\"; break;
        case '\n': o += "\\n"; break;
        case '\r': o += "\\r"; break;
        case '\t': o += "\\t"; break;
        default:
            if (ch < 0x20) {
                char u[8];
                std::snprintf(u, sizeof u, "\\u%04x", ch);
                o += u;
            } else {
                o += static_cast<char>(ch);
            }
        }
    }
    return o + "\"";
}

// Position just after `"key":` (and spaces) in a flat JSON object, or npos.
size_t field_value(const std::string& body, const std::string& key) {
    const std::string k = "\"" + key + "\"";
    size_t p = body.find(k);
    if (p == std::string::npos) return p;
    p = body.find(':', p + k.size());
    if (p == std::string::npos) return p;
    ++p;
    while (p < body.size() && std::isspace(static_cast<unsigned char>(body[p]))) ++p;
    return p;
}

std::string string_field(const std::string& body, const std::string& key) {
    size_t p = field_value(body, key);
    if (p == std::string::npos || p >= body.size() || body[p] != '"') return {};
    std::string out;
    for (++p; p < body.size() && body[p] != '"'; ++p) {
        char ch = body[p];
        if (ch == '\\' && p + 1 < body.size()) {
            const char e = body[++p];
            switch (e) {
            case 'n': ch = '\n'; break;
            case 't': ch = '\t'; break;
            case 'r': ch = '\r'; break;
            case 'u':
                if (p + 4 < body.size()) {  // \uXXXX below 0x80 (what json_quote() writes); others dropped
                    const unsigned v = static_cast<unsigned>(std::strtoul(body.substr(p + 1, 4).c_str(), nullptr, 16));
                    p += 4;
                    if (v >= 0x80) continue;
                    ch = static_cast<char>(v);
                }
                break;
            default: ch = e;
            }
        }
        out += ch;
    }
    return out;
}

size_t number_field(const std::string& body, const std::string& key, size_t fallback) {
    const size_t p = field_value(body, key);
    if (p == std::string::npos || p >= body.size() || !std::isdigit(static_cast<unsigned char>(body[p])))
        return fallback;
    return static_cast<size_t>(std::strtoull(body.c_str() + p, nullptr, 10));
}

// ---- HTTP
const char* reason(int code) {
    switch (code) {
    case 200: return "OK";
    case 201: return "Created";
    case 400: return "Bad Request";
    case 404: return "Not Found";
    case 409: return "Conflict";
    default: return "Internal Server Error";
    }
}

constexpr const char* kCors =
    "Access-Control-Allow-Origin: *\r\nAccess-Control-Allow-Headers: Content-Type,X-Filename\r\n"
    "Access-Control-Allow-Methods: GET,POST,OPTIONS\r\n";

std::string http_response(int code, const std::string& body, const char* type = "application/json") {
    std::ostringstream o;
    o << "HTTP/1.1 " << code << ' ' << reason(code) << "\r\nContent-Type: " << type
      << "\r\nContent-Length: " << body.size() << "\r\n" << kCors << "Connection: close\r\n\r\n" << body;
    return o.str();
}

bool send_all(int fd, const std::string& s) {
    size_t done = 0;
    while (done < s.size()) {
        const ssize_t n = ::send(fd, s.data() + done, s.size() - done, MSG_NOSIGNAL);
        if (n <= 0) return false;
        done += static_cast<size_t>(n);
    }
    return true;
}

struct Request {
    std::string method, path, head, body;
    std::string header(const std::string& name) const {  // case-sensitive, "Name: value"
        const std::string k = "\r\n" + name + ":";
        size_t p = head.find(k);
        if (p == std::string::npos) return {};
        p += k.size();
        while (p < head.size() && head[p] == ' ') ++p;
        return head.substr(p, head.find("\r\n", p) - p);
    }
};

// Headers up to the blank line, then Content-Length bytes of body. False on a closed or
// malformed connection.
bool read_request(int fd, Request& r) {
    std::string buf;
    char chunk[16384];
    size_t end = std::string::npos;
    while (end == std::string::npos) {
        const ssize_t n = ::recv(fd, chunk, sizeof chunk, 0);
        if (n <= 0) return false;
        buf.append(chunk, static_cast<size_t>(n));
        end = buf.find("\r\n\r\n");
        if (end == std::string::npos && buf.size() > (1u << 20)) return false;  // no end of headers
    }
    r.head = buf.substr(0, end);
    std::istringstream first(r.head);
    first >> r.method >> r.path;
    r.body = buf.substr(end + 4);
    const std::string len = r.header("Content-Length");
    const size_t want = len.empty() ? 0 : static_cast<size_t>(std::strtoull(len.c_str(), nullptr, 10));
    while (r.body.size() < want) {
        const ssize_t n = ::recv(fd, chunk, sizeof chunk, 0);
        if (n <= 0) return false;
        r.body.append(chunk, static_cast<size_t>(n));
    }
    if (r.body.size() > want) r.body.resize(want);
    return true;
}

// ---- host statistics for /api/status
unsigned physical_cores() {
    std::ifstream f("/proc/cpuinfo");
    std::set<std::pair<std::string, std::string>> cores;
    std::string line, phys;
    while (std::getline(f, line)) {
        const size_t c = line.find(':');
        if (c == std::string::npos) continue;
        std::string key = line.substr(0, c);
        key.erase(key.find_last_not_of(" \t") + 1);
        const std::string val = c + 2 <= line.size() ? line.substr(c + 2) : std::string();
        if (key == "physical id") phys = val;
        if (key == "core id") cores.emplace(phys, val);
    }
    return cores.empty() ? std::max(1u, std::thread::hardware_concurrency()) : static_cast<unsigned>(cores.size());
}

size_t ram_percent() {
    std::ifstream f("/proc/meminfo");
    std::string key;
    size_t v = 0, total = 0, avail = 0;
    while (f >> key >> v) {
        if (key == "MemTotal:") total = v;
        if (key == "MemAvailable:") avail = v;
        f.ignore(64, '\n');
    }
    return total ? (total - std::min(avail, total)) * 100 / total : 0;
}

}  // namespace

struct ApiServer::Impl {
    uint16_t port;
    fs::path dir;
    std::atomic<int> listen_fd{-1};
    std::atomic<bool> running{false};

    std::mutex mu;  // guards runtime and loaded
    std::unique_ptr<LlamaRuntime> runtime;
    std::string loaded;
    std::atomic<bool> generating{false};
    std::atomic<size_t> tokens{0};
    std::atomic<double> tps{0.0};
    Clock::time_point started{};

    std::mutex cpu_mu;
    unsigned long long cpu_total = 0, cpu_idle = 0;
    double cpu_pct = 0.0;
    const unsigned logical = std::max(1u, std::thread::hardware_concurrency());
    const unsigned physical = physical_cores();

    Impl(uint16_t p, std::string d) : port(p), dir(std::move(d)) { fs::create_directories(dir); }

    double cpu_percent() {  // busy share of all CPUs since the previous call
        std::ifstream f("/proc/stat");
        std::string label;
        unsigned long long v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (!(f >> label)) return cpu_pct;
        for (auto& x : v) f >> x;
        unsigned long long total = 0;
        for (auto x : v) total += x;
        const unsigned long long idle = v[3] + v[4];
        std::lock_guard<std::mutex> g(cpu_mu);
        if (cpu_total && total > cpu_total)
            cpu_pct = 100.0 * double((total - cpu_total) - (idle - cpu_idle)) / double(total - cpu_total);
        cpu_total = total;
        cpu_idle = idle;
        return cpu_pct;
    }

    std::string models_json() {
        std::string loaded_now;
        {
            std::lock_guard<std::mutex> g(mu);
            loaded_now = loaded;
        }
        std::vector<std::pair<std::string, uintmax_t>> files;
        for (const auto& e : fs::directory_iterator(dir))
            if (e.is_regular_file() && e.path().extension() == ".gguf")
                files.emplace_back(e.path().filename().string(), fs::file_size(e.path()));
        std::sort(files.begin(), files.end());
        std::string o = "[";
        for (size_t i = 0; i < files.size(); ++i) {
            if (i) o += ',';
            o += "{\"name\":" + json_quote(files[i].first) + ",\"size\":" + std::to_string(files[i].second) +
                 ",\"loaded\":" + (files[i].first == loaded_now ? "true" : "false") + "}";
        }
        return o + "]";
    }

    std::string status_json() {
        std::string loaded_now;
        {
            std::lock_guard<std::mutex> g(mu);
            loaded_now = loaded;
        }
        std::ostringstream o;
        o << "{\"generating\":" << (generating ? "true" : "false") << ",\"tokens\":" << tokens.load()
          << ",\"tokens_per_sec\":" << tps.load() << ",\"cpu_percent\":" << cpu_percent()
          << ",\"ram_percent\":" << ram_percent() << ",\"cpu_logical\":" << logical
          << ",\"cpu_physical\":" << physical << ",\"inference_threads\":" << logical
          << ",\"loaded\":" << json_quote(loaded_now) << "}";
        return o.str();
    }

    // The model file `name` inside the directory (no path components), or empty.
    fs::path model_path(const std::string& name) const {
        const fs::path base = fs::path(name).filename();
        if (name.empty() || base.extension() != ".gguf") return {};
        return dir / base;
    }

    void upload(int fd, const Request& r) {
        std::string name = r.header("X-Filename");
        if (name.empty()) name = "model.gguf";
        const fs::path p = model_path(name);
        if (p.empty() || r.body.size() < 4 || r.body.compare(0, 4, "GGUF") != 0) {
            send_all(fd, http_response(400, "{\"error\":\"Valid GGUF file required\"}"));
            return;
        }
        std::ofstream o(p, std::ios::binary | std::ios::trunc);
        o.write(r.body.data(), static_cast<std::streamsize>(r.body.size()));
        if (!o) {
            send_all(fd, http_response(500, "{\"error\":\"cannot write model file\"}"));
            return;
        }
        send_all(fd, http_response(201, "{\"name\":" + json_quote(p.filename().string()) +
                                             ",\"size\":" + std::to_string(r.body.size()) + "}"));
    }

    void load(int fd, const Request& r) {
        try {
            const fs::path p = model_path(string_field(r.body, "name"));
            if (p.empty() || !fs::exists(p)) throw std::runtime_error("model not found");
            if (generating) throw std::runtime_error("generation in progress");
            auto rt = std::make_unique<LlamaRuntime>();
            rt->load(p.string());
            std::lock_guard<std::mutex> g(mu);
            if (generating) throw std::runtime_error("generation in progress");
            runtime = std::move(rt);
            loaded = p.filename().string();
            send_all(fd, http_response(200, "{\"ok\":true}"));
        } catch (const std::exception& e) {
            send_all(fd, http_response(400, "{\"error\":" + json_quote(e.what()) + "}"));
        }
    }

    void unload(int fd) {
        std::lock_guard<std::mutex> g(mu);
        if (generating) {
            send_all(fd, http_response(409, "{\"error\":\"stop generation before unloading\"}"));
            return;
        }
        runtime.reset();
        loaded.clear();
        send_all(fd, http_response(200, "{\"ok\":true}"));
    }

    void request_stop(int fd) {
        {
            std::lock_guard<std::mutex> g(mu);
            if (runtime) runtime->request_stop();
        }
        send_all(fd, http_response(200, "{\"ok\":true,\"stopping\":true}"));
    }

    std::string progress(size_t n) {
        const double sec = std::chrono::duration<double>(Clock::now() - started).count();
        const double r = sec > 0 ? double(n) / sec : 0.0;
        tps = r;
        std::ostringstream o;
        o << "\"tokens\":" << n << ",\"tokens_per_sec\":" << r;
        return o.str();
    }

    void chat(int fd, const Request& r, bool stream) {
        LlamaRuntime* rt = nullptr;
        {
            std::lock_guard<std::mutex> g(mu);
            if (!runtime || generating) {
                send_all(fd, http_response(409, runtime ? "{\"error\":\"generation already running\"}"
                                                        : "{\"error\":\"no model loaded\"}"));
                return;
            }
            rt = runtime.get();  // stays alive: unload and load refuse while generating
            generating = true;
            tokens = 0;
            tps = 0.0;
            started = Clock::now();
        }
        GenerationConfig cfg;
        cfg.max_tokens = std::min<size_t>(number_field(r.body, "max_tokens", 128), 2048);
        cfg.temperature = 0.0f;  // the API's generations are greedy
        if (stream)
            send_all(fd, std::string("HTTP/1.1 200 OK\r\nContent-Type: text/event-stream\r\nCache-Control: no-cache\r\n") +
                             kCors + "Connection: close\r\n\r\n");
        std::string text, error;
        try {
            rt->generate_ids(string_field(r.body, "message"), cfg, [&](uint32_t id) {
                const std::string piece = rt->tokenizer().decode(id);
                text += piece;
                const size_t n = ++tokens;
                if (stream) send_all(fd, "data: {\"token\":" + json_quote(piece) + "," + progress(n) + "}\n\n");
                return !rt->stop_requested();
            });
        } catch (const std::exception& e) {
            error = e.what();
        }
        const bool stopped = rt->stop_requested();
        const std::string tail = progress(tokens.load()) + ",\"stopped\":" + (stopped ? "true" : "false");
        generating = false;
        if (stream) {
            if (!error.empty() && !stopped) send_all(fd, "data: {\"error\":" + json_quote(error) + "}\n\n");
            send_all(fd, "data: {\"done\":true," + tail + "}\n\n");
        } else if (!error.empty() && !stopped) {
            send_all(fd, http_response(500, "{\"error\":" + json_quote(error) + "}"));
        } else {
            send_all(fd, http_response(200, "{\"text\":" + json_quote(text) + "," + tail + "}"));
        }
    }

    void serve(int fd) {
        Request r;
        if (read_request(fd, r)) {
            if (r.method == "OPTIONS") {
                send_all(fd, http_response(200, "{}"));
            } else if (r.method == "GET" && r.path == "/") {
                std::ifstream f("web/index_v2.html", std::ios::binary);
                const std::string page((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
                send_all(fd, page.empty() ? http_response(404, "{\"error\":\"web/index_v2.html not found\"}")
                                          : http_response(200, page, "text/html; charset=utf-8"));
            } else if (r.method == "GET" && r.path == "/api/models") {
                send_all(fd, http_response(200, models_json()));
            } else if (r.method == "GET" && r.path == "/api/status") {
                send_all(fd, http_response(200, status_json()));
            } else if (r.method == "POST" && r.path == "/api/models/upload") {
                upload(fd, r);
            } else if (r.method == "POST" && r.path == "/api/models/load") {
                load(fd, r);
            } else if (r.method == "POST" && r.path == "/api/models/unload") {
                unload(fd);
            } else if (r.method == "POST" && r.path == "/api/stop") {
                request_stop(fd);
            } else if (r.method == "POST" && (r.path == "/api/chat" || r.path == "/api/chat/stream")) {
                chat(fd, r, r.path == "/api/chat/stream");
            } else {
                send_all(fd, http_response(404, "{\"error\":\"not found\"}"));
            }
        }
        ::close(fd);
    }

    void run() {
        const int fd = ::socket(AF_INET, SOCK_STREAM, 0);
        if (fd < 0) throw std::runtime_error("socket failed");
        const int one = 1;
        ::setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof one);
        sockaddr_in a{};
        a.sin_family = AF_INET;
        a.sin_addr.s_addr = htonl(INADDR_ANY);
        a.sin_port = htons(port);
        if (::bind(fd, reinterpret_cast<sockaddr*>(&a), sizeof a) < 0) {
            ::close(fd);
            throw std::runtime_error("bind failed");
        }
        if (::listen(fd, 32) < 0) {
            ::close(fd);
            throw std::runtime_error("listen failed");
        }
        listen_fd = fd;
        running = true;
        while (running) {
            const int c = ::accept(fd, nullptr, nullptr);
            if (c < 0) {
                if (!running) break;
                continue;
            }
            std::thread([this, c] { serve(c); }).detach();
        }
    }

    void stop() noexcept {
        running = false;
        const int fd = listen_fd.exchange(-1);
        if (fd >= 0) {
            ::shutdown(fd, SHUT_RDWR);
            ::close(fd);
        }
    }

    ~Impl() { stop(); }
};

ApiServer::ApiServer(uint16_t port, std::string model_dir) : impl_(new Impl(port, std::move(model_dir))) {}
ApiServer::~ApiServer() = default;
void ApiServer::run() { impl_->run(); }
void ApiServer::stop() noexcept { impl_->stop(); }

}  // namespace laic
