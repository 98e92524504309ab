// Drives forge::Engine in reference-compat mode through the script of
// oracle/literal_script.hpp for tests/test_literal_gpu.py:
//   literal_driver <model.squeeze> <seed> <max_memory or 0> <long_tokens> [env]
// With a fifth argument "env" the mode comes from FORGE_REFERENCE_COMPAT in the
// environment (the route an unmodified program takes); otherwise the driver
// calls set_reference_compat(true).  Prints the transcript.
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "forge/engine.hpp"
#include "literal_script.hpp"

int main(int argc, char** argv) {
    if (argc < 5) return 2;
    const unsigned seed = (unsigned)std::strtoul(argv[2], nullptr, 10);
    const size_t max_memory = (size_t)std::strtoull(argv[3], nullptr, 10);
    const uint32_t long_tokens = (uint32_t)std::strtoul(argv[4], nullptr, 10);
    const bool from_env = argc > 5 && std::strcmp(argv[5], "env") == 0;
    forge::Engine e;
    if (!from_env) e.set_reference_compat(true);
    if (!e.reference_compat()) {
        std::printf("reference-compat mode is off\n");
        return 3;
    }
    const std::string t = literal_script::run(e, argv[1], seed, max_memory, long_tokens);
    std::fputs(t.c_str(), stdout);
    return t.rfind("load failed", 0) == 0 ? 1 : 0;
}
