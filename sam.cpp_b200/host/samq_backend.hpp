// samq_backend.hpp -- C++17 host layer over the samq C ABI, shaped like the
// reference runtime's backend driver so SAM.cpp's runtime can select it.
//
// Mirrors (paths relative to the SAM.cpp tree):
//   make_samq_backend     <- make_cuda_backend (src/runtime/ggml/backends/cuda.hpp:156-189):
//                            same argument meaning (visible CUDA device index, compute mode
//                            with F32 as default) and the same failure style
//                            (std::runtime_error with a message).
//   QuantizedLinear       <- one ggml_mul_mat(W_packed, X_f32) node built by
//                            sam3_channel_projection (src/models/sam3/ops.hpp:40-45) with its
//                            bias add and optional ggml_gelu_erf (src/models/sam3/vision.hpp:234-238).
//   ActivationCounters    <- CudaActivationPolicy::record (src/runtime/ggml/backends/cuda_activation.hpp:62-77):
//                            one launch per request, payload and allocation peaks.
//   load_quantized_linear <- the WEIGHTS upload of a packed tensor (src/models/sam3/model.hpp:114-133)
//                            read by samq_io::GgufReader (gguf_reader.hpp, mirrors src/io/gguf_reader.hpp).
//   VitBackbone           <- sam3_build_vit_graph (src/models/sam3/vision.hpp:252-293) as
//                            encode_image runs it (src/models/sam3/execution.hpp:55-124): the
//                            prefix, then every block on the device path, in place on x.
// Header-only; link with libsamq.so.
#pragma once

#include <cuda_runtime_api.h>

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "gguf_reader.hpp"
#include "weight_policy.hpp"
#include "samq.h"

namespace sam::internal {

enum class LinearEpilogue { None = SAMQ_EPILOGUE_NONE, GeluErf = SAMQ_EPILOGUE_GELU_ERF };

// sam::CudaComputeMode (include/sam/types.hpp:13), passed through
// BackendOptions::cuda_compute: F32 (the default) keeps the ViT attention and
// the patch-embedding columns in f32; F16 is the opt-in reduced mode.
enum class CudaComputeMode { F32 = SAMQ_COMPUTE_F32, F16 = SAMQ_COMPUTE_F16 };

inline void samq_require(samq_status status, const char* what) {
    if (status != SAMQ_OK) throw std::runtime_error(std::string(what) + ": " + samq_last_error_v1());
}

// Device-side ownership and identity, as BackendDriver carries them.
struct SamqDriver {
    int cuda_device = -1;
    std::string device_name;
    int sm_count = 0;
    CudaComputeMode compute = CudaComputeMode::F32;
};

inline SamqDriver make_samq_backend(int device_index, CudaComputeMode compute = CudaComputeMode::F32) {
    if (device_index < 0) throw std::runtime_error("requested CUDA device index is out of range for visible devices");
    struct samq_capabilities_v1 info{};  // "struct": the function of the same name hides the type
    samq_require(samq_capabilities_v1(device_index, &info), "requested samq CUDA device is unavailable");
    samq_require(samq_init_v1(device_index), "requested samq CUDA backend failed initialization");
    SamqDriver driver;
    driver.cuda_device = device_index;
    driver.device_name = info.name;
    driver.sm_count = info.sm_count;
    driver.compute = compute;
    return driver;
}

// Counters in the shape of RuntimeStats' activation fields (include/sam/types.hpp:56-57).
struct ActivationCounters {
    std::uint64_t activation_requests = 0, activation_launches = 0;
    std::uint64_t activation_payload_peak_bytes = 0, activation_allocation_peak_bytes = 0;
};

// One packed weight matrix resident on the driver's device and the linear it feeds.
class QuantizedLinear {
public:
    QuantizedLinear(const SamqDriver& driver, int ggml_type, std::int64_t k, std::int64_t n, const void* gguf_rows,
                    std::size_t bytes, cudaStream_t stream = nullptr)
        : k_(k), n_(n) {
        samq_require(samq_weights_create_v1(driver.cuda_device, ggml_type, k, n, gguf_rows, bytes, stream, &weights_),
                     "samq rejected the packed weight");
    }
    QuantizedLinear(const QuantizedLinear&) = delete;
    QuantizedLinear& operator=(const QuantizedLinear&) = delete;
    QuantizedLinear(QuantizedLinear&& other) noexcept
        : weights_(std::exchange(other.weights_, nullptr)), k_(other.k_), n_(other.n_) {}
    ~QuantizedLinear() {
        if (weights_) samq_weights_destroy_v1(weights_);
    }

    std::int64_t width() const { return k_; }
    std::int64_t rows() const { return n_; }

    // Y[m][n] = epilogue(X[m][k] . W^T + bias); device pointers, caller-owned.
    void forward(const float* x, std::int64_t m, std::int64_t ldx, const float* bias, LinearEpilogue epilogue,
                 float* y, std::int64_t ldy, cudaStream_t stream, ActivationCounters* counters = nullptr) const {
        samq_counters_v1 before{};
        if (counters) samq_require(samq_query_v1(weights_, &before), "samq execution identity missing");
        samq_require(samq_linear_v1(weights_, x, m, ldx, bias, static_cast<int>(epilogue), y, ldy, stream),
                     "samq quantized linear failed");
        if (counters && m > 0) {
            samq_counters_v1 after{};
            samq_require(samq_query_v1(weights_, &after), "samq execution identity missing");
            if (after.version != 1 || after.launches != before.launches + 1 || after.payload_bytes == 0 ||
                after.allocation_bytes < after.payload_bytes)
                throw std::runtime_error("samq request did not execute exactly one tensor-core GEMM");
            ++counters->activation_requests;
            ++counters->activation_launches;
            counters->activation_payload_peak_bytes =
                std::max<std::uint64_t>(counters->activation_payload_peak_bytes, after.payload_bytes);
            counters->activation_allocation_peak_bytes =
                std::max<std::uint64_t>(counters->activation_allocation_peak_bytes, after.allocation_bytes);
        }
    }

    // Packed bytes back in GGUF layout (bit-exact round trip of the load-time repack).
    void export_rows(void* gguf_rows, std::size_t bytes) const {
        samq_require(samq_weights_export_v1(weights_, gguf_rows, bytes), "samq weight export failed");
    }

    const samq_weights* handle() const { return weights_; }

private:
    samq_weights* weights_ = nullptr;
    std::int64_t k_ = 0, n_ = 0;
};

// A packed linear weight straight from a GGUF checkpoint: a 2-D tensor with
// ne = [K, N] (tensors.hpp T2 weights), its GGUF rows handed to K4 unchanged.
inline QuantizedLinear load_quantized_linear(const SamqDriver& driver, samq_io::GgufReader& reader,
                                             const std::string& name, cudaStream_t stream = nullptr) {
    const samq_io::GgufTensor& t = reader.tensor(name);
    if (t.dimensions.size() != 2) throw std::runtime_error("GGUF linear weight must be 2-D: " + name);
    const std::vector<std::uint8_t> bytes = reader.tensor_bytes(t);
    return QuantizedLinear(driver, t.type, t.dimensions[0], t.dimensions[1], bytes.data(), bytes.size(), stream);
}

// The same, after checking the tensor's stored type against the checkpoint's
// weight-precision policy (samq_policy::inspect_weight_policy, the reference's
// inspect_weights): a tensor stored with another type than its profile
// assigns (for example a K-quant fc2 that is not the Q8_0 fallback) is
// rejected before any device memory is touched.
inline QuantizedLinear load_quantized_linear(const SamqDriver& driver, samq_io::GgufReader& reader,
                                             const samq_policy::WeightPolicy& policy, const std::string& name,
                                             cudaStream_t stream = nullptr) {
    const samq_io::GgufTensor& t = reader.tensor(name);
    if (t.type != policy.expected_type(t.name, t.dimensions))
        throw std::runtime_error("incompatible SAM 3 tensor precision: " + name);
    return load_quantized_linear(driver, reader, name, stream);
}

// Device pointers to one ViT block's F32 tensors (src/models/sam3/tensors.hpp:108-126).
struct VitBlockTensors {
    const float* norm1_w = nullptr;
    const float* norm1_b = nullptr;
    const float* qkv_b = nullptr;
    const float* proj_b = nullptr;
    const float* norm2_w = nullptr;
    const float* norm2_b = nullptr;
    const float* fc1_b = nullptr;
    const float* fc2_b = nullptr;
    const float* freqs_cis = nullptr;  // [positions][32][2]
    int window = 0;                    // 24 windowed, 0 global (hparams.is_global_attn)
};

// Device pointers to the prefix tensors (tensors.hpp:97-106).
struct VitPrefixTensors {
    const float* patch_embed_w = nullptr;  // [E][3][patch][patch]
    const float* pos_embed = nullptr;      // [pos_grid][pos_grid][E]
    const float* ln_pre_w = nullptr;
    const float* ln_pre_b = nullptr;
    int patch = 14;
    int pos_grid = 24;
};

class VitBackbone {
public:
    VitBackbone(const SamqDriver& driver, std::int64_t embed) : driver_(driver), embed_(embed) {}

    void set_prefix(const VitPrefixTensors& prefix) { prefix_ = prefix; }

    // Appends a block; the backbone owns its four linears (qkv E->3E, proj
    // E->E, fc1 E->MLP with GELU, fc2 MLP->E).
    void add_block(QuantizedLinear qkv, QuantizedLinear proj, QuantizedLinear fc1, QuantizedLinear fc2,
                   const VitBlockTensors& t) {
        samq_vit_block_v1 b{};
        b.version = 2;
        b.compute = static_cast<int32_t>(driver_.compute);
        b.window = t.window;
        b.norm1_w = t.norm1_w;
        b.norm1_b = t.norm1_b;
        b.qkv = qkv.handle();
        b.qkv_b = t.qkv_b;
        b.proj = proj.handle();
        b.proj_b = t.proj_b;
        b.norm2_w = t.norm2_w;
        b.norm2_b = t.norm2_b;
        b.fc1 = fc1.handle();
        b.fc1_b = t.fc1_b;
        b.fc2 = fc2.handle();
        b.fc2_b = t.fc2_b;
        b.freqs_cis = t.freqs_cis;
        blocks_.push_back(b);
        linears_.push_back(std::move(qkv));
        linears_.push_back(std::move(proj));
        linears_.push_back(std::move(fc1));
        linears_.push_back(std::move(fc2));
    }

    std::size_t depth() const { return blocks_.size(); }

    // image: device [3][height][width] f32, normalized; x: device [tokens][E] f32 (receives the
    // backbone output, the [E, W, H, 1] tensor the neck consumes).
    void encode(const float* image, int width, int height, float* x, cudaStream_t stream) const {
        encode_batch(image, 1, width, height, x, stream);
    }

    // `batch` images ([batch][3][height][width], consecutive) into x
    // ([batch][tokens][E]); every block runs once for the whole batch.
    void encode_batch(const float* images, int batch, int width, int height, float* x, cudaStream_t stream) const {
        if (prefix_.patch_embed_w == nullptr) throw std::runtime_error("ViT prefix tensors were not set");
        const int grid_w = width / prefix_.patch, grid_h = height / prefix_.patch;
        const std::int64_t tokens = static_cast<std::int64_t>(grid_w) * grid_h;
        for (int i = 0; i < batch; ++i)
            samq_require(samq_vit_prefix_v2(images + static_cast<std::int64_t>(i) * 3 * width * height, width, height,
                                            prefix_.patch, prefix_.patch_embed_w, embed_, prefix_.pos_embed,
                                            prefix_.pos_grid, prefix_.ln_pre_w, prefix_.ln_pre_b,
                                            x + static_cast<std::int64_t>(i) * tokens * embed_,
                                            static_cast<int>(driver_.compute), stream),
                         "samq ViT prefix failed");
        for (const samq_vit_block_v1& b : blocks_)
            samq_require(batch == 1 ? samq_vit_block_forward_v1(&b, x, grid_w, grid_h, stream)
                                    : samq_vit_block_forward_batch_v1(&b, x, batch, grid_w, grid_h, stream),
                         "samq ViT block failed");
    }

private:
    SamqDriver driver_;
    std::int64_t embed_ = 0;
    VitPrefixTensors prefix_{};
    std::vector<QuantizedLinear> linears_;
    std::vector<samq_vit_block_v1> blocks_;
};

// An F32 / F16 tensor the reference keeps unquantized (neck convolutions,
// fusion / decoder linears), multiplied with F32 semantics.  `kind` is
// SAMQ_DENSE_LINEAR (ne = [k, n]), SAMQ_DENSE_CONV (ne = [kw, kh, cin, cout])
// or SAMQ_DENSE_DECONV2X2 (ne = [2, 2, cout, cin]); `data` is host memory.
class DenseModule {
public:
    DenseModule(const SamqDriver& driver, int kind, int ggml_type, const std::int64_t ne[4], const void* data,
                std::size_t bytes, cudaStream_t stream = nullptr)
        : kind_(kind) {
        const int type = ggml_type == 1 ? SAMQ_TYPE_F16 : SAMQ_TYPE_F32;
        if (ggml_type != 0 && ggml_type != 1) throw std::runtime_error("dense tensor must be F32 or F16");
        const bool deconv = kind == SAMQ_DENSE_DECONV2X2;
        const bool linear = kind == SAMQ_DENSE_LINEAR;
        const int kw = linear ? 1 : static_cast<int>(ne[0]), kh = linear ? 1 : static_cast<int>(ne[1]);
        cin_ = linear ? ne[0] : (deconv ? ne[3] : ne[2]);
        cout_ = linear ? ne[1] : (deconv ? ne[2] : ne[3]);
        samq_require(samq_dense_create_v1(driver.cuda_device, type, kind, kw, kh, cin_, cout_, data, bytes, stream,
                                          &dense_),
                     "samq rejected the dense tensor");
    }
    DenseModule(const DenseModule&) = delete;
    DenseModule& operator=(const DenseModule&) = delete;
    DenseModule(DenseModule&& other) noexcept
        : dense_(std::exchange(other.dense_, nullptr)), kind_(other.kind_), cin_(other.cin_), cout_(other.cout_) {}
    ~DenseModule() {
        if (dense_) samq_dense_destroy_v1(dense_);
    }

    std::int64_t in_channels() const { return cin_; }
    std::int64_t out_channels() const { return cout_; }
    const samq_dense* handle() const { return dense_; }

    // LINEAR: Y[m][n] = epilogue(X[m][k] . W^T + bias) (ggml_mul_mat at GGML_PREC_F32).
    void linear(const float* x, std::int64_t m, std::int64_t ldx, const float* bias, LinearEpilogue epilogue,
                float* y, std::int64_t ldy, cudaStream_t stream) const {
        samq_require(samq_dense_linear_v1(dense_, x, m, ldx, bias, static_cast<int>(epilogue), y, ldy, stream),
                     "samq dense linear failed");
    }

    // CONV / DECONV2X2 over an NHWC image (sam3_conv_2d_s1_ph, sam3_deconv_2x2).
    void conv(const float* x, int width, int height, const float* bias, LinearEpilogue epilogue, float* y,
              cudaStream_t stream) const {
        samq_require(samq_conv2d_v1(dense_, x, width, height, bias, static_cast<int>(epilogue), y, stream),
                     "samq convolution failed");
    }

private:
    samq_dense* dense_ = nullptr;
    int kind_ = 0;
    std::int64_t cin_ = 0, cout_ = 0;
};

// A dense tensor straight from a GGUF checkpoint (F32 / F16, GGML dimensions).
inline DenseModule load_dense(const SamqDriver& driver, samq_io::GgufReader& reader, const std::string& name,
                              int kind, cudaStream_t stream = nullptr) {
    const samq_io::GgufTensor& t = reader.tensor(name);
    std::int64_t ne[4] = {1, 1, 1, 1};
    for (std::size_t i = 0; i < t.dimensions.size() && i < 4; ++i) ne[i] = t.dimensions[i];
    const std::vector<std::uint8_t> bytes = reader.tensor_bytes(t);
    return DenseModule(driver, kind, t.type, ne, bytes.data(), bytes.size(), stream);
}

// The SimpleFPN neck of one path (src/models/sam3/vision.hpp:307-366).  Layer
// order and names follow samq_neck_v1 (tensors.hpp:131-160).
class SimpleFpnNeck {
public:
    static constexpr int kLayers = 11;
    // Device biases per layer, in the order of samq_neck_v1.
    SimpleFpnNeck(std::vector<DenseModule> layers, const std::vector<const float*>& biases)
        : layers_(std::move(layers)) {
        if (layers_.size() != kLayers || biases.size() != kLayers)
            throw std::runtime_error("the neck has 11 weighted layers");
        const samq_dense* w[kLayers];
        for (int i = 0; i < kLayers; ++i) w[i] = layers_[i].handle();
        desc_ = samq_neck_v1{1,          w[0], biases[0], w[1], biases[1], w[2], biases[2], w[3], biases[3],
                             w[4],       biases[4], w[5], biases[5], w[6], biases[6], w[7], biases[7],
                             w[8],       biases[8], w[9], biases[9], w[10], biases[10]};
    }

    // x: device [grid_h * grid_w][E] f32 (the backbone output); out[i]: the
    // four NHWC maps (4x, 2x, 1x, 0.5x).
    void forward(const float* x, int grid_w, int grid_h, float* const out[4], cudaStream_t stream) const {
        samq_require(samq_neck_forward_v1(&desc_, x, grid_w, grid_h, out, stream), "samq neck failed");
    }

private:
    std::vector<DenseModule> layers_;
    samq_neck_v1 desc_{};
};

// Post-compute device findings (range / timeout), as the reference's RHS check raises them.
inline void samq_check_device(const SamqDriver& driver, cudaStream_t stream) {
    samq_require(samq_check_v1(driver.cuda_device, stream), "samq device check failed");
}

}  // namespace sam::internal
