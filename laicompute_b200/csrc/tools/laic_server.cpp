// HTTP API server over the B200 decode runtime, with the reference's usage
// (reference tools/server.cpp): laic_server [port] [model_dir]
#include <cstdint>
#include <iostream>
#include <string>

#include "laic/server.hpp"

int main(int argc, char** argv) {
    const uint16_t port = argc > 1 ? static_cast<uint16_t>(std::stoul(argv[1])) : 8080;
    const std::string dir = argc > 2 ? argv[2] : "models";
    try {
        laic::ApiServer server(port, dir);
        std::cout << "LAICompute UI/API: http://0.0.0.0:" << port << "\nModels: " << dir << "\n" << std::flush;
        server.run();
    } catch (const std::exception& e) {
        std::cerr << "laic_server: " << e.what() << "\n";
        return 1;
    }
    return 0;
}
