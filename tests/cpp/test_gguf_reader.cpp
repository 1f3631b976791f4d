// Reads a GGUF file with samq_io::GgufReader and prints what it parsed:
//   tensor <name> <type> <dims...> | <size_bytes> <offset> <fnv1a64 of the bytes>
//   key <name> <type> [value]
// or "error <message>" with exit status 1 when the reader rejects the file.
// tests/test_gguf_reader.py compares the listing with gguf-py's view.
#include <cinttypes>
#include <cstdio>
#include <string>

#include "gguf_reader.hpp"

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    using namespace sam::internal::samq_io;
    try {
        GgufReader reader(argv[1]);
        for (const GgufTensor& t : reader.tensors()) {
            std::uint64_t h = 1469598103934665603ull;
            for (std::uint8_t b : reader.tensor_bytes(t)) h = (h ^ b) * 1099511628211ull;
            std::printf("tensor %s %d", t.name.c_str(), t.type);
            for (std::int64_t d : t.dimensions) std::printf(" %lld", static_cast<long long>(d));
            std::printf(" | %" PRIu64 " %" PRIu64 " %016" PRIx64 "\n", t.size_bytes, t.offset, h);
        }
        for (const auto& kv : reader.metadata()) {
            std::printf("key %s %u", kv.first.c_str(), static_cast<unsigned>(kv.second.type));
            if (kv.second.type == GgufValueType::Uint32) std::printf(" %u", reader.u32(kv.first));
            if (kv.second.type == GgufValueType::String) std::printf(" %s", reader.string(kv.first).c_str());
            if (kv.second.type == GgufValueType::Array)
                std::printf(" %u %" PRIu64, static_cast<unsigned>(kv.second.element_type), kv.second.count);
            std::printf("\n");
        }
    } catch (const std::exception& e) {
        std::printf("error %s\n", e.what());
        return 1;
    }
    return 0;
}
