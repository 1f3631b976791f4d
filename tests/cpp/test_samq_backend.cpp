// C++ host-layer test in the style of the reference's runtime tests
// (tests/runtime/ggml/test_quantization.cpp, test_native_activation.cpp):
// throw on failure, exit 0 on success.  Inputs are raw little-endian files
// written by tests/test_gpu_cpp_host.py: meta.txt (type k n m epilogue),
// rows.bin (GGUF rows), x.bin (f32 [m][k]), bias.bin (f32 [n]), ref.bin
// (f32 [m][n] oracle product of decoded weights and decoded Q8_1 activations).
#include <cuda_runtime_api.h>

#include <cmath>
#include <cstdio>
#include <fstream>
#include <iostream>
#include <iterator>
#include <stdexcept>
#include <string>
#include <vector>

#include "samq_backend.hpp"

namespace {

void require(bool condition, const char* message) {
    if (!condition) throw std::runtime_error(message);
}

void check(cudaError_t err) {
    if (err != cudaSuccess) throw std::runtime_error(cudaGetErrorString(err));
}

template <class T>
std::vector<T> read_file(const std::string& path) {
    std::ifstream in(path, std::ios::binary);
    require(in.good(), "missing fixture file");
    std::vector<char> bytes((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
    std::vector<T> out(bytes.size() / sizeof(T));
    std::copy(bytes.begin(), bytes.begin() + out.size() * sizeof(T), reinterpret_cast<char*>(out.data()));
    return out;
}

template <class F>
void rejects(F f, const char* message) {
    try {
        f();
    } catch (const std::runtime_error&) {
        return;
    }
    throw std::runtime_error(message);
}

}  // namespace

int main(int argc, char** argv) {
    try {
        require(argc == 2, "usage: test_samq_backend FIXTURE_DIR");
        const std::string dir = argv[1];
        int type = 0, epilogue = 0;
        long long k = 0, n = 0, m = 0;
        {
            std::ifstream meta(dir + "/meta.txt");
            meta >> type >> k >> n >> m >> epilogue;
            require(meta.good() || meta.eof(), "bad meta");
        }
        const auto rows = read_file<unsigned char>(dir + "/rows.bin");
        const auto x = read_file<float>(dir + "/x.bin");
        const auto bias = read_file<float>(dir + "/bias.bin");
        const auto ref = read_file<float>(dir + "/ref.bin");
        require(x.size() == static_cast<size_t>(m * k) && ref.size() == static_cast<size_t>(m * n), "fixture sizes");

        auto driver = sam::internal::make_samq_backend(0);
        require(driver.sm_count > 0 && !driver.device_name.empty(), "driver identity missing");
        cudaStream_t stream = nullptr;
        check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
        sam::internal::QuantizedLinear linear(driver, type, k, n, rows.data(), rows.size(), stream);

        std::vector<unsigned char> exported(rows.size());
        linear.export_rows(exported.data(), exported.size());
        require(exported == rows, "load-time repack did not round-trip the GGUF rows");

        float *dx = nullptr, *dbias = nullptr, *dy = nullptr;
        check(cudaMalloc(reinterpret_cast<void**>(&dx), x.size() * sizeof(float)));
        check(cudaMalloc(reinterpret_cast<void**>(&dbias), bias.size() * sizeof(float)));
        check(cudaMalloc(reinterpret_cast<void**>(&dy), ref.size() * sizeof(float)));
        check(cudaMemcpy(dx, x.data(), x.size() * sizeof(float), cudaMemcpyHostToDevice));
        check(cudaMemcpy(dbias, bias.data(), bias.size() * sizeof(float), cudaMemcpyHostToDevice));

        sam::internal::ActivationCounters counters;
        const auto epi = epilogue ? sam::internal::LinearEpilogue::GeluErf : sam::internal::LinearEpilogue::None;
        linear.forward(dx, m, k, dbias, epi, dy, n, stream, &counters);
        sam::internal::samq_check_device(driver, stream);
        require(counters.activation_requests == 1 && counters.activation_launches == 1 &&
                    counters.activation_payload_peak_bytes == static_cast<unsigned long long>(m * k * 2),
                "activation counters differ from one request");

        std::vector<float> y(ref.size());
        check(cudaMemcpy(y.data(), dy, y.size() * sizeof(float), cudaMemcpyDeviceToHost));
        double dot = 0, ny = 0, nr = 0, max_err = 0, max_ref = 0;
        for (size_t i = 0; i < y.size(); ++i) {
            require(std::isfinite(y[i]), "non-finite output");
            dot += double(y[i]) * ref[i];
            ny += double(y[i]) * y[i];
            nr += double(ref[i]) * ref[i];
            max_err = std::max(max_err, std::abs(double(y[i]) - ref[i]));
            max_ref = std::max(max_ref, std::abs(double(ref[i])));
        }
        const double cosine = dot / std::sqrt(ny * nr), rel = max_err / max_ref;
        std::cout << "cosine=" << cosine << " normalized_max_error=" << rel << "\n";
        require(cosine >= 0.9999 && rel <= 2e-3, "quantized linear differs from the oracle beyond tolerance");

        // Malformed payloads and arguments surface as std::runtime_error.
        rejects([&] { sam::internal::QuantizedLinear bad(driver, type, k, n, rows.data(), rows.size() - 1, stream); },
                "short GGUF payload was accepted");
        rejects([&] { linear.forward(dx, m, k - 1, dbias, epi, dy, n, stream); }, "bad row stride was accepted");

        check(cudaFree(dx));
        check(cudaFree(dbias));
        check(cudaFree(dy));
        check(cudaStreamDestroy(stream));
        return 0;
    } catch (const std::exception& e) {
        std::cerr << e.what() << "\n";
        return 1;
    }
}
