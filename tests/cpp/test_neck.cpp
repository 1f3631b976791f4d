// Drives sam::internal::SimpleFpnNeck (sam.cpp_b200/host/samq_backend.hpp) the
// way the neck would run after encode_image: its 11 dense layers and their
// biases loaded from a GGUF checkpoint (F32 tensors with the names of
// src/models/sam3/tensors.hpp:131-160) by samq_io::GgufReader.  The input x and
// the four NHWC outputs travel through files written / read by
// tests/test_gpu_cpp_host.py.
#include <cuda_runtime_api.h>

#include <cstdio>
#include <fstream>
#include <string>
#include <vector>

#include "samq_backend.hpp"

namespace {

std::vector<char> read_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot read " + path);
    return std::vector<char>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

float* device_copy(const void* host, std::size_t bytes) {
    void* d = nullptr;
    if (cudaMalloc(&d, bytes) != cudaSuccess) throw std::runtime_error("cudaMalloc");
    if (cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice) != cudaSuccess) throw std::runtime_error("cudaMemcpy");
    return static_cast<float*>(d);
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    const std::string dir = argv[1];
    try {
        int gw = 0, gh = 0;
        long long embed = 0, d = 0;
        {
            std::ifstream meta(dir + "/meta.txt");
            meta >> gw >> gh >> embed >> d;
        }
        using namespace sam::internal;
        SamqDriver driver = make_samq_backend(0);
        samq_io::GgufReader checkpoint(dir + "/weights.gguf");
        const char* names[SimpleFpnNeck::kLayers] = {"0.dconv_2x2_0", "0.dconv_2x2_1", "0.conv_1x1", "0.conv_3x3",
                                                     "1.dconv_2x2",   "1.conv_1x1",    "1.conv_3x3", "2.conv_1x1",
                                                     "2.conv_3x3",    "3.conv_1x1",    "3.conv_3x3"};
        std::vector<DenseModule> layers;
        std::vector<const float*> biases;
        for (const char* name : names) {
            const std::string base = std::string("neck.det.") + name;
            const bool deconv = base.find("dconv") != std::string::npos;
            layers.push_back(load_dense(driver, checkpoint, base + ".weight",
                                        deconv ? SAMQ_DENSE_DECONV2X2 : SAMQ_DENSE_CONV));
            const samq_io::GgufTensor& b = checkpoint.tensor(base + ".bias");
            const std::vector<std::uint8_t> bytes = checkpoint.tensor_bytes(b);
            biases.push_back(device_copy(bytes.data(), bytes.size()));
        }
        SimpleFpnNeck neck(std::move(layers), biases);
        const std::vector<char> x_host = read_file(dir + "/x.bin");
        float* x = device_copy(x_host.data(), x_host.size());
        const int sides[4][2] = {{4 * gw, 4 * gh}, {2 * gw, 2 * gh}, {gw, gh}, {gw / 2, gh / 2}};
        float* out[4];
        for (int i = 0; i < 4; ++i) {
            void* p = nullptr;
            if (cudaMalloc(&p, static_cast<std::size_t>(sides[i][0]) * sides[i][1] * d * sizeof(float)) != cudaSuccess)
                throw std::runtime_error("cudaMalloc");
            out[i] = static_cast<float*>(p);
        }
        neck.forward(x, gw, gh, out, nullptr);
        samq_check_device(driver, nullptr);
        for (int i = 0; i < 4; ++i) {
            std::vector<float> host(static_cast<std::size_t>(sides[i][0]) * sides[i][1] * d);
            if (cudaMemcpy(host.data(), out[i], host.size() * sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess)
                throw std::runtime_error("cudaMemcpy");
            std::ofstream f(dir + "/out" + std::to_string(i) + ".bin", std::ios::binary);
            f.write(reinterpret_cast<const char*>(host.data()), static_cast<std::streamsize>(host.size() * 4));
        }
        std::printf("neck ok\n");
        return 0;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "%s\n", e.what());
        return 1;
    }
}
