// Drives sam::internal::VitBackbone (sam.cpp_b200/host/samq_backend.hpp) the
// way encode_image would: linears loaded from a GGUF checkpoint by
// samq_io::GgufReader, prefix + blocks on device buffers.  Inputs come from
// files written by tests/test_gpu_cpp_host.py; the output x goes back to a file
// that the Python side compares with the oracle.
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

float* to_device(const std::vector<char>& host) {
    void* d = nullptr;
    if (cudaMalloc(&d, host.size()) != cudaSuccess) throw std::runtime_error("cudaMalloc");
    if (cudaMemcpy(d, host.data(), host.size(), cudaMemcpyHostToDevice) != cudaSuccess)
        throw std::runtime_error("cudaMemcpy");
    return static_cast<float*>(d);
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    const std::string dir = argv[1];
    try {
        int size = 0, patch = 0, pos_grid = 0, window = 0, qtype = 0, fc2_type = 0;
        long long embed = 0, mlp = 0;
        {
            std::ifstream meta(dir + "/meta.txt");
            meta >> size >> patch >> pos_grid >> embed >> mlp >> window >> qtype >> fc2_type;
        }
        using namespace sam::internal;
        SamqDriver driver = make_samq_backend(0);
        VitBackbone vit(driver, embed);
        VitPrefixTensors pre;
        pre.patch_embed_w = to_device(read_file(dir + "/patch_w.bin"));
        pre.pos_embed = to_device(read_file(dir + "/pos.bin"));
        pre.ln_pre_w = to_device(read_file(dir + "/ln_w.bin"));
        pre.ln_pre_b = to_device(read_file(dir + "/ln_b.bin"));
        pre.patch = patch;
        pre.pos_grid = pos_grid;
        vit.set_prefix(pre);
        // The four linears come from a GGUF checkpoint (tensor names of tensors.hpp:108-121).
        samq_io::GgufReader checkpoint(dir + "/weights.gguf");
        auto linear = [&](const char* name, int type, long long k, long long n) {
            const std::string full = std::string("vit.blocks.0.") + name + ".weight";
            const samq_io::GgufTensor& t = checkpoint.tensor(full);
            if (t.type != type || t.dimensions.size() != 2 || t.dimensions[0] != k || t.dimensions[1] != n)
                throw std::runtime_error("unexpected checkpoint tensor " + full);
            return load_quantized_linear(driver, checkpoint, full);
        };
        VitBlockTensors t;
        t.norm1_w = to_device(read_file(dir + "/norm1_w.bin"));
        t.norm1_b = to_device(read_file(dir + "/norm1_b.bin"));
        t.qkv_b = to_device(read_file(dir + "/qkv_b.bin"));
        t.proj_b = to_device(read_file(dir + "/proj_b.bin"));
        t.norm2_w = to_device(read_file(dir + "/norm2_w.bin"));
        t.norm2_b = to_device(read_file(dir + "/norm2_b.bin"));
        t.fc1_b = to_device(read_file(dir + "/fc1_b.bin"));
        t.fc2_b = to_device(read_file(dir + "/fc2_b.bin"));
        t.freqs_cis = to_device(read_file(dir + "/freqs.bin"));
        t.window = window;
        vit.add_block(linear("attn.qkv", qtype, embed, 3 * embed), linear("attn.proj", qtype, embed, embed),
                      linear("mlp.lin1", qtype, embed, mlp), linear("mlp.lin2", fc2_type, mlp, embed), t);
        const float* image = to_device(read_file(dir + "/image.bin"));
        const long long tokens = static_cast<long long>(size / patch) * (size / patch);
        void* x_mem = nullptr;
        if (cudaMalloc(&x_mem, tokens * embed * sizeof(float)) != cudaSuccess) throw std::runtime_error("cudaMalloc x");
        float* x = static_cast<float*>(x_mem);
        vit.encode(image, size, size, x, nullptr);
        samq_check_device(driver, nullptr);
        std::vector<float> out(static_cast<size_t>(tokens * embed));
        if (cudaMemcpy(out.data(), x, out.size() * sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess)
            throw std::runtime_error("cudaMemcpy out");
        std::ofstream(dir + "/out.bin", std::ios::binary)
            .write(reinterpret_cast<const char*>(out.data()), static_cast<std::streamsize>(out.size() * sizeof(float)));
        std::printf("vit backbone: %zu block(s), %lld tokens\n", vit.depth(), tokens);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "FAIL: %s\n", e.what());
        return 1;
    }
    return 0;
}
