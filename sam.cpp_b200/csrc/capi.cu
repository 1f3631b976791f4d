// capi.cu -- the extern "C" boundary declared in include/samq.h.
//
// Every entry point validates its arguments, runs on the device that owns
// the data (weights handle) or the current device, converts internal errors
// into a samq_status and records a thread-local message; no exception
// crosses the boundary (the reference converts codes to std::runtime_error
// itself, src/runtime/ggml/workspace.hpp:174-177).
#include <cuda_fp16.h>

#include <cstdio>
#include <cstring>
#include <memory>
#include <vector>

#include <map>
#include <set>

#include "samq_internal.hpp"

namespace samq {
namespace {
thread_local std::string g_last_error;
std::mutex g_states_mutex;
DeviceState* g_states[64] = {};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        check_cuda(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q),
                   "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
        if (!ptr || q != cudaDriverEntryPointSuccess) fail(SAMQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
        return reinterpret_cast<EncodeTiledFn>(ptr);
    }();
    return fn;
}

}  // namespace

void fail(samq_status status, const std::string& message) { throw Error{status, message}; }

void check_cuda(cudaError_t err, const char* what) {
    if (err == cudaSuccess) return;
    const samq_status status = err == cudaErrorMemoryAllocation ? SAMQ_ERR_OUT_OF_MEMORY : SAMQ_ERR_CUDA;
    fail(status, std::string(what) + ": " + cudaGetErrorName(err) + " (" + cudaGetErrorString(err) + ")");
}

void set_last_error(const std::string& message) { g_last_error = message; }

DeviceGuard::DeviceGuard(int device) {
    check_cuda(cudaGetDevice(&previous), "cudaGetDevice");
    if (previous != device) check_cuda(cudaSetDevice(device), "cudaSetDevice");
}

DeviceGuard::~DeviceGuard() {
    int current = -1;
    if (cudaGetDevice(&current) == cudaSuccess && current != previous && previous >= 0) cudaSetDevice(previous);
}

DeviceState& device_state(int device) {
    if (device < 0 || device >= 64) fail(SAMQ_ERR_INVALID_ARGUMENT, "device index out of range");
    std::lock_guard<std::mutex> lock(g_states_mutex);
    if (g_states[device]) return *g_states[device];
    int count = 0;
    check_cuda(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if (device >= count) fail(SAMQ_ERR_INVALID_ARGUMENT, "device index is not visible");
    cudaDeviceProp prop{};
    check_cuda(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (prop.major != 10 || prop.minor != 0)
        fail(SAMQ_ERR_UNSUPPORTED, std::string("samq kernels are built for sm_100a; device '") + prop.name +
                                       "' is sm_" + std::to_string(prop.major * 10 + prop.minor));
    DeviceGuard guard(device);
    auto state = std::make_unique<DeviceState>();
    state->device = device;
    state->sm_count = prop.multiProcessorCount;
    state->cc_major = prop.major;
    state->cc_minor = prop.minor;
    check_cuda(cudaMalloc(reinterpret_cast<void**>(&state->status), sizeof(DeviceStatus)), "cudaMalloc(status)");
    check_cuda(cudaMemset(state->status, 0, sizeof(DeviceStatus)), "cudaMemset(status)");
    g_states[device] = state.release();
    return *g_states[device];
}

DeviceState* existing_device_state(int device) {
    if (device < 0 || device >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_states_mutex);
    return g_states[device];
}

Scratch& scratch_for(DeviceState& state, cudaStream_t stream, size_t bytes) {
    std::lock_guard<std::mutex> lock(state.mutex);
    Scratch& s = state.scratch[stream];
    if (s.bytes < bytes) {
        if (s.ptr) {
            // The old buffer may still be read by work queued on this stream.
            check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize(scratch growth)");
            check_cuda(cudaFree(s.ptr), "cudaFree(scratch)");
            s.ptr = nullptr;
            s.bytes = 0;
        }
        const size_t rounded = (bytes + (size_t(2) << 20) - 1) / (size_t(2) << 20) * (size_t(2) << 20);
        check_cuda(cudaMalloc(&s.ptr, rounded), "cudaMalloc(scratch)");
        s.bytes = rounded;
    }
    return s;
}

void set_smem_limit_once(DeviceState& state, const void* kernel, int bytes, const char* what) {
    static std::mutex mutex;
    static std::set<std::pair<const void*, int>> done;
    std::lock_guard<std::mutex> lock(mutex);
    if (done.count({kernel, state.device})) return;
    DeviceGuard guard(state.device);
    check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what);
    done.insert({kernel, state.device});
}

int pair_clusters_resident(DeviceState& state, const void* kernel, int threads, int smem, const char* what) {
    static std::mutex mutex;
    static std::map<std::pair<const void*, int>, int> cache;
    std::lock_guard<std::mutex> lock(mutex);
    auto it = cache.find({kernel, state.device});
    if (it != cache.end()) return it->second;
    DeviceGuard guard(state.device);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    check_cuda(cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg), what);
    if (clusters <= 0) fail(SAMQ_ERR_CUDA, "no CTA pair of the GEMM kernel fits on this device");
    cache[{kernel, state.device}] = clusters;
    return clusters;
}

void encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                          uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                          CUtensorMapSwizzle swizzle) {
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t elem_strides[2] = {1, 1};
    const CUresult r = encode_fn()(map, dtype, 2, const_cast<void*>(base), dims, strides, box, elem_strides,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(SAMQ_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled rejected a tensor (code " +
                                                               std::to_string(static_cast<int>(r)) + ")");
}

void encode_tensor_map_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t d0, uint64_t d1,
                          uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1,
                          CUtensorMapSwizzle swizzle) {
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
    const cuuint32_t box[3] = {box0, box1, 1};
    const cuuint32_t elem_strides[3] = {1, 1, 1};
    const CUresult r = encode_fn()(map, dtype, 3, const_cast<void*>(base), dims, strides, box, elem_strides,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(SAMQ_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled rejected a 3-D tensor (code " +
                                                               std::to_string(static_cast<int>(r)) + ")");
}

void encode_tensor_map_3d_box(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t d0,
                              uint64_t d1, uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                              uint32_t box1, uint32_t box2, CUtensorMapSwizzle swizzle) {
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
    const cuuint32_t box[3] = {box0, box1, box2};
    const cuuint32_t elem_strides[3] = {1, 1, 1};
    const CUresult r = encode_fn()(map, dtype, 3, const_cast<void*>(base), dims, strides, box, elem_strides,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(SAMQ_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled rejected a 3-D box (code " +
                                                               std::to_string(static_cast<int>(r)) + ")");
}

namespace {

template <class F>
samq_status guarded(F&& body) {
    try {
        body();
        g_last_error.clear();
        return SAMQ_OK;
    } catch (const Error& e) {
        g_last_error = e.message;
        return e.status;
    } catch (const std::bad_alloc&) {
        g_last_error = "host allocation failed";
        return SAMQ_ERR_OUT_OF_MEMORY;
    } catch (...) {
        g_last_error = "unexpected internal failure";
        return SAMQ_ERR_CUDA;
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

void require(bool condition, const char* message) {
    if (!condition) fail(SAMQ_ERR_INVALID_ARGUMENT, message);
}

bool supported_type(int type) {
    return type == SAMQ_TYPE_Q8_0 || type == SAMQ_TYPE_Q4_K || type == SAMQ_TYPE_Q5_K || type == SAMQ_TYPE_Q6_K;
}

int current_device() {
    int device = 0;
    check_cuda(cudaGetDevice(&device), "cudaGetDevice");
    return device;
}

void release_dense(samq_dense* w) {
    if (!w) return;
    if (w->device >= 0) {
        int previous = -1;
        cudaGetDevice(&previous);
        cudaSetDevice(w->device);
        if (w->hi) cudaFree(w->hi);
        if (w->lo) cudaFree(w->lo);
        if (previous >= 0) cudaSetDevice(previous);
    }
    delete w;
}

void release(samq_weights* w) {
    if (!w) return;
    if (w->device >= 0) {
        int previous = -1;
        cudaGetDevice(&previous);
        cudaSetDevice(w->device);
        if (w->packets) cudaFree(w->packets);
        if (w->operand) cudaFree(w->operand);
        if (previous >= 0) cudaSetDevice(previous);
    }
    delete w;
}

}  // namespace

void check_activation_args(int64_t rows, int64_t k, int64_t ld, const void* x, const void* out) {
    require(rows >= 0 && rows <= (int64_t(1) << 31), "rows out of range");
    require(k > 0 && k % 32 == 0 && k <= (int64_t(1) << 20), "width must be a positive multiple of 32");
    require(ld >= k && ld % 4 == 0, "row stride must be >= width and a multiple of 4 floats");
    require(rows == 0 || (x && out), "null pointer");
    require(rows == 0 || aligned16(x), "activation pointer must be 16-byte aligned");
}

void check_linear_args(const samq_weights* w, int64_t m, const float* bias, int epilogue, const float* y,
                       int64_t ldy) {
    require(w != nullptr, "null weights");
    require(m >= 0 && m <= (int64_t(1) << 31), "row count out of range");
    require(epilogue == SAMQ_EPILOGUE_NONE || epilogue == SAMQ_EPILOGUE_GELU_ERF, "unknown epilogue");
    require(ldy >= w->n && ldy % 4 == 0, "output row stride must be >= n and a multiple of 4 floats");
    require(m == 0 || (y != nullptr && aligned16(y)), "output pointer must be 16-byte aligned");
    (void)bias;
}

}  // namespace samq

using namespace samq;

extern "C" {

const char* samq_last_error_v1(void) { return g_last_error.c_str(); }

samq_status samq_init_v1(int device) {
    return guarded([&] { device_state(device); });
}

samq_status samq_capabilities_v1(int device, struct samq_capabilities_v1* info) {
    return guarded([&] {
        require(info != nullptr, "null info");
        int count = 0;
        check_cuda(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
        require(device >= 0 && device < count, "device index is not visible");
        cudaDeviceProp prop{};
        check_cuda(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
        std::memset(info, 0, sizeof(*info));
        info->version = 1;
        info->device = device;
        info->cc_major = prop.major;
        info->cc_minor = prop.minor;
        info->sm_count = prop.multiProcessorCount;
        info->global_memory_bytes = prop.totalGlobalMem;
        info->max_shared_memory_per_block = prop.sharedMemPerBlockOptin;
        std::snprintf(info->name, sizeof(info->name), "%s", prop.name);
    });
}

samq_status samq_weights_create_v1(int device, int type, int64_t k, int64_t n, const void* gguf_rows, size_t bytes,
                                   void* stream_ptr, samq_weights** out) {
    return guarded([&] {
        require(out != nullptr, "null output handle");
        *out = nullptr;
        require(supported_type(type), "weight type must be Q8_0, Q4_K, Q5_K or Q6_K");
        require(n > 0 && n <= (int64_t(1) << 24), "row count out of range");
        const int64_t rb = row_bytes(type, k);
        require(rb > 0, "width is not a whole number of blocks");
        require(k % 32 == 0 && k <= (int64_t(1) << 20), "width out of range");
        require(gguf_rows != nullptr && bytes == static_cast<size_t>(rb * n), "GGUF payload size differs from n rows");
        DeviceState& state = device_state(device);
        DeviceGuard guard(device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        std::unique_ptr<samq_weights, void (*)(samq_weights*)> w(new samq_weights, release);
        w->device = device;
        w->type = type;
        w->k = k;
        w->n = n;
        const int64_t chunks = (k + 63) / 64;
        w->packet_bytes = static_cast<size_t>((n + 127) / 128 * chunks * packet_bytes(type));
        w->operand_bytes = static_cast<size_t>(n * k) * sizeof(__half);
        void* staging = nullptr;
        uint32_t* bad = nullptr;
        struct Cleanup {
            void*& s;
            uint32_t*& b;
            ~Cleanup() {
                if (s) cudaFree(s);
                if (b) cudaFree(b);
            }
        } cleanup{staging, bad};
        check_cuda(cudaMalloc(&staging, bytes), "cudaMalloc(weight staging)");
        check_cuda(cudaMalloc(reinterpret_cast<void**>(&bad), sizeof(uint32_t)), "cudaMalloc(scale check)");
        check_cuda(cudaMalloc(&w->packets, w->packet_bytes), "cudaMalloc(packets)");
        check_cuda(cudaMalloc(reinterpret_cast<void**>(&w->operand), w->operand_bytes), "cudaMalloc(operand)");
        check_cuda(cudaMemsetAsync(bad, 0, sizeof(uint32_t), stream), "cudaMemsetAsync");
        check_cuda(cudaMemsetAsync(w->packets, 0, w->packet_bytes, stream), "cudaMemsetAsync(packets)");
        check_cuda(cudaMemcpyAsync(staging, gguf_rows, bytes, cudaMemcpyHostToDevice, stream), "cudaMemcpyAsync(H2D)");
        launch_gguf_to_packets(type, k, n, static_cast<const uint8_t*>(staging), static_cast<uint8_t*>(w->packets), bad,
                               stream);
        uint32_t bad_host = 0;
        check_cuda(cudaMemcpyAsync(&bad_host, bad, sizeof(bad_host), cudaMemcpyDeviceToHost, stream),
                   "cudaMemcpyAsync(D2H)");
        check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize(repack)");
        if (bad_host) fail(SAMQ_ERR_PAYLOAD, "packed weight has " + std::to_string(bad_host) + " non-finite block scales");
        launch_packets_to_f16(type, k, n, static_cast<const uint8_t*>(w->packets), w->operand, stream);
        check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize(expand)");
        *out = w.release();
    });
}

samq_status samq_weights_destroy_v1(samq_weights* weights) {
    return guarded([&] { release(weights); });
}

samq_status samq_weights_export_v1(const samq_weights* w, void* gguf_rows, size_t bytes) {
    return guarded([&] {
        require(w != nullptr && gguf_rows != nullptr, "null argument");
        const int64_t rb = row_bytes(w->type, w->k);
        require(bytes == static_cast<size_t>(rb * w->n), "output size differs from n rows");
        DeviceGuard guard(w->device);
        void* rows = nullptr;
        check_cuda(cudaMalloc(&rows, bytes), "cudaMalloc(export)");
        struct Free {
            void* p;
            ~Free() { cudaFree(p); }
        } free_rows{rows};
        launch_packets_to_gguf(w->type, w->k, w->n, static_cast<const uint8_t*>(w->packets),
                               static_cast<uint8_t*>(rows), nullptr);
        check_cuda(cudaMemcpy(gguf_rows, rows, bytes, cudaMemcpyDeviceToHost), "cudaMemcpy(export)");
    });
}

samq_status samq_weights_packets_v1(const samq_weights* w, const void** packets, size_t* bytes) {
    return guarded([&] {
        require(w != nullptr && packets != nullptr && bytes != nullptr, "null argument");
        *packets = w->packets;
        *bytes = w->packet_bytes;
    });
}

samq_status samq_quantize_q8_1_v1(const float* x, int64_t rows, int64_t k, int64_t ld, void* out, void* stream) {
    return guarded([&] {
        check_activation_args(rows, k, ld, x, out);
        require(rows == 0 || (reinterpret_cast<uintptr_t>(out) & 3u) == 0, "output must be 4-byte aligned");
        DeviceState& state = device_state(current_device());
        launch_act_f16(x, rows, k, ld, nullptr, static_cast<uint8_t*>(out), state.status,
                       static_cast<cudaStream_t>(stream));
    });
}

size_t samq_mmq_d4_bytes_v1(int64_t rows, int64_t k) {
    if (rows < 0 || k <= 0) return 0;
    const int64_t padded = (k + 511) / 512 * 512;
    return static_cast<size_t>(rows * (padded / 128) * 144);
}

samq_status samq_quantize_mmq_q8_1_v1(const float* x, int64_t rows, int64_t k, int64_t ld, void* out, void* stream) {
    return guarded([&] {
        check_activation_args(rows, k, ld, x, out);
        require(rows == 0 || aligned16(out), "output must be 16-byte aligned");
        device_state(current_device());
        launch_mmq_d4(x, rows, k, ld, static_cast<uint8_t*>(out), static_cast<cudaStream_t>(stream));
    });
}

// K2 over an f16 operand: M <= kStreamMaxRows streams the packed weights
// (stream.cu), larger M runs the f16 tensor-core GEMM on the expanded weights.
size_t linear_scratch_bytes(const samq_weights* w, int64_t m, size_t operand_bytes, const DeviceState& state) {
    const size_t head = (operand_bytes + 255) / 256 * 256;
    return head + (stream_eligible(w, m) ? stream_partial_bytes(w, m, state.sm_count) : 0);
}

void run_linear(const samq_weights* w, const __half* a, int64_t lda, int64_t m, const float* bias, int epilogue,
                float* y, int64_t ldy, void* scratch, size_t operand_bytes, DeviceState& state, cudaStream_t stream) {
    if (stream_eligible(w, m)) {
        float* partials = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + (operand_bytes + 255) / 256 * 256);
        launch_linear_stream(w, a, lda, m, bias, epilogue, y, ldy, partials, state, stream);
    } else {
        launch_gemm_f16(a, lda, w->operand, m, w->n, w->k, bias, epilogue, y, ldy, state, stream);
    }
}

samq_status samq_linear_v1(const samq_weights* w, const float* x, int64_t m, int64_t ldx, const float* bias,
                           int epilogue, float* y, int64_t ldy, void* stream_ptr) {
    return guarded([&] {
        check_linear_args(w, m, bias, epilogue, y, ldy);
        check_activation_args(m, w->k, ldx, x, y);
        if (m == 0) return;
        DeviceGuard guard(w->device);
        DeviceState& state = device_state(w->device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        const size_t a_bytes = static_cast<size_t>(m * w->k) * sizeof(__half);
        Scratch& scratch = scratch_for(state, stream, linear_scratch_bytes(w, m, a_bytes, state));
        __half* a = static_cast<__half*>(scratch.ptr);
        launch_act_f16(x, m, w->k, ldx, a, nullptr, state.status, stream);
        run_linear(w, a, w->k, m, bias, epilogue, y, ldy, scratch.ptr, a_bytes, state, stream);
        const_cast<samq_weights*>(w)->launches.fetch_add(1);
        const_cast<samq_weights*>(w)->payload_bytes.store(a_bytes);
        const_cast<samq_weights*>(w)->allocation_bytes.store(scratch.bytes);
    });
}

samq_status samq_linear_q8_1_v1(const samq_weights* w, const void* x_q8_1, int64_t m, const float* bias, int epilogue,
                                float* y, int64_t ldy, void* stream_ptr) {
    return guarded([&] {
        check_linear_args(w, m, bias, epilogue, y, ldy);
        if (m == 0) return;
        require(x_q8_1 != nullptr && (reinterpret_cast<uintptr_t>(x_q8_1) & 3u) == 0,
                "Q8_1 activations must be 4-byte aligned");
        DeviceGuard guard(w->device);
        DeviceState& state = device_state(w->device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        const size_t a_bytes = static_cast<size_t>(m * w->k) * sizeof(__half);
        Scratch& scratch = scratch_for(state, stream, linear_scratch_bytes(w, m, a_bytes, state));
        __half* a = static_cast<__half*>(scratch.ptr);
        launch_q8_1_to_f16(static_cast<const uint8_t*>(x_q8_1), m, w->k, a, state.status, stream);
        run_linear(w, a, w->k, m, bias, epilogue, y, ldy, scratch.ptr, a_bytes, state, stream);
        const_cast<samq_weights*>(w)->launches.fetch_add(1);
        const_cast<samq_weights*>(w)->payload_bytes.store(static_cast<uint64_t>(m * (w->k / 32) * 36));
        const_cast<samq_weights*>(w)->allocation_bytes.store(scratch.bytes);
    });
}

samq_status samq_stage_f16_v1(const float* x, int64_t rows, int64_t k, int64_t ld, void* out_f16, void* stream) {
    return guarded([&] {
        check_activation_args(rows, k, ld, x, out_f16);
        require(rows == 0 || aligned16(out_f16), "output must be 16-byte aligned");
        DeviceState& state = device_state(current_device());
        launch_act_f16(x, rows, k, ld, static_cast<__half*>(out_f16), nullptr, state.status,
                       static_cast<cudaStream_t>(stream));
    });
}

samq_status samq_linear_f16_v1(const samq_weights* w, const void* x_f16, int64_t m, int64_t ldx, const float* bias,
                               int epilogue, float* y, int64_t ldy, void* stream_ptr) {
    return guarded([&] {
        check_linear_args(w, m, bias, epilogue, y, ldy);
        if (m == 0) return;
        require(x_f16 != nullptr && aligned16(x_f16), "f16 activations must be 16-byte aligned");
        require(ldx >= w->k && ldx % 8 == 0, "f16 row stride must be >= k and a multiple of 8");
        DeviceGuard guard(w->device);
        DeviceState& state = device_state(w->device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        void* scratch = nullptr;
        if (stream_eligible(w, m) && stream_partial_bytes(w, m, state.sm_count) > 0)
            scratch = scratch_for(state, stream, linear_scratch_bytes(w, m, 0, state)).ptr;
        run_linear(w, static_cast<const __half*>(x_f16), ldx, m, bias, epilogue, y, ldy, scratch, 0, state, stream);
        const_cast<samq_weights*>(w)->launches.fetch_add(1);
    });
}

static void vit_attention(const float* qkv, int64_t ldq, int grid_w, int grid_h, int heads, int head_dim,
                          int window, const float* freqs_cis, float* out, int64_t ldo, int compute,
                          void* stream_ptr) {
    {
        require(head_dim == 64, "head_dim must be 64");
        require(heads > 0 && heads <= 64, "heads out of range");
        require(grid_w > 0 && grid_h > 0 && static_cast<int64_t>(grid_w) * grid_h <= (int64_t(1) << 20),
                "grid out of range");
        require(window == 0 || (window > 0 && grid_w % window == 0 && grid_h % window == 0),
                "window must divide the grid (or be 0 for global attention)");
        const int64_t E = static_cast<int64_t>(heads) * head_dim;
        const int64_t group_n = window > 0 ? static_cast<int64_t>(window) * window
                                           : static_cast<int64_t>(grid_w) * grid_h;
        require(group_n % 8 == 0, "tokens per attention group must be a multiple of 8");
        require(ldq >= 3 * E && ldq % 4 == 0, "qkv row stride must be >= 3*heads*64 and a multiple of 4");
        require(ldo >= E && ldo % 4 == 0, "output row stride must be >= heads*64 and a multiple of 4");
        require(qkv && out && freqs_cis && aligned16(qkv) && aligned16(out) && aligned16(freqs_cis),
                "qkv, freqs_cis and out must be 16-byte aligned device pointers");
        require(compute == SAMQ_COMPUTE_F32 || compute == SAMQ_COMPUTE_F16, "compute must be SAMQ_COMPUTE_F32 or _F16");
        DeviceState& state = device_state(current_device());
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        if (compute == SAMQ_COMPUTE_F32) {
            launch_attention_f32(qkv, ldq, false, grid_w, grid_h, heads, window, 1, freqs_cis, out, nullptr, ldo, state,
                                 stream);
            return;
        }
        Scratch& scratch = scratch_for(state, stream, attention_scratch_bytes(grid_w, grid_h, heads));
        launch_vit_attention(qkv, ldq, grid_w, grid_h, heads, window, freqs_cis, out, ldo, scratch.ptr, state, stream);
    }
}

samq_status samq_vit_attention_v1(const float* qkv, int64_t ldq, int grid_w, int grid_h, int heads, int head_dim,
                                  int window, const float* freqs_cis, float* out, int64_t ldo, void* stream_ptr) {
    return guarded([&] {
        vit_attention(qkv, ldq, grid_w, grid_h, heads, head_dim, window, freqs_cis, out, ldo, SAMQ_COMPUTE_F16,
                      stream_ptr);
    });
}

samq_status samq_vit_attention_v2(const float* qkv, int64_t ldq, int grid_w, int grid_h, int heads, int head_dim,
                                  int window, const float* freqs_cis, float* out, int64_t ldo, int compute,
                                  void* stream_ptr) {
    return guarded([&] {
        vit_attention(qkv, ldq, grid_w, grid_h, heads, head_dim, window, freqs_cis, out, ldo, compute, stream_ptr);
    });
}

samq_status samq_vit_rope_v1(const float* x, int64_t tokens, int64_t head_batches, int head_dim,
                             const float* freqs_cis, float* out, void* stream_ptr) {
    return guarded([&] {
        require(head_dim == 64, "head_dim must be 64");
        require(tokens >= 0 && head_batches >= 0 && tokens <= (int64_t(1) << 24) && head_batches <= (int64_t(1) << 16),
                "tokens / head_batches out of range");
        if (tokens == 0 || head_batches == 0) return;
        require(x && out && freqs_cis && aligned16(x) && aligned16(out) && aligned16(freqs_cis),
                "x, freqs_cis and out must be 16-byte aligned device pointers");
        device_state(current_device());
        launch_rope_f32(x, freqs_cis, tokens, head_batches, out, static_cast<cudaStream_t>(stream_ptr));
    });
}

static void vit_block_forward(const samq_vit_block_v1* block, float* x, int batch, int grid_w, int grid_h,
                              void* stream_ptr) {
    {
        require(block != nullptr && (block->version == 1 || block->version == 2),
                "block descriptor missing or not version 1 / 2");
        const samq_vit_block_v1& b = *block;
        const int compute = b.version >= 2 ? b.compute : SAMQ_COMPUTE_F16;
        require(compute == SAMQ_COMPUTE_F32 || compute == SAMQ_COMPUTE_F16, "compute must be SAMQ_COMPUTE_F32 or _F16");
        require(b.qkv && b.proj && b.fc1 && b.fc2, "null weight handle");
        const int64_t E = b.qkv->k, mlp = b.fc1->n;
        require(E == 256 || E == 512 || E == 1024, "embedding width must be 256, 512 or 1024");
        require(b.qkv->n == 3 * E && b.proj->k == E && b.proj->n == E && b.fc1->k == E && b.fc2->k == mlp &&
                    b.fc2->n == E,
                "linear shapes must be qkv E->3E, proj E->E, fc1 E->MLP, fc2 MLP->E");
        require(mlp % 32 == 0, "MLP width must be a multiple of 32");
        require(grid_w > 0 && grid_h > 0 && static_cast<int64_t>(grid_w) * grid_h <= (int64_t(1) << 20),
                "grid out of range");
        require(batch > 0 && static_cast<int64_t>(batch) * grid_w * grid_h <= (int64_t(1) << 22),
                "batch out of range");
        const int window = b.window;
        require(window == 0 || (window > 0 && grid_w % window == 0 && grid_h % window == 0),
                "window must divide the grid (or be 0 for global attention)");
        const int64_t group_n = window > 0 ? static_cast<int64_t>(window) * window
                                           : static_cast<int64_t>(grid_w) * grid_h;
        require(group_n % 8 == 0, "tokens per attention group must be a multiple of 8");
        const float* params[] = {b.norm1_w, b.norm1_b, b.qkv_b, b.proj_b, b.norm2_w, b.norm2_b, b.fc1_b, b.fc2_b,
                                 b.freqs_cis, x};
        for (const float* p : params) require(p != nullptr && aligned16(p), "parameters must be 16-byte aligned device pointers");
        const int device = current_device();
        const samq_weights* handles[] = {b.qkv, b.proj, b.fc1, b.fc2};
        for (const samq_weights* w : handles) require(w->device == device, "weight handle belongs to another device");
        DeviceState& state = device_state(device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        const int64_t tokens = static_cast<int64_t>(batch) * grid_w * grid_h;
        Scratch& scratch = scratch_for(state, stream, vit_block_scratch_bytes(tokens, E, mlp, compute));
        VitBlockArgs args;
        args.window = window;
        args.compute = compute;
        args.norm1_w = b.norm1_w;
        args.norm1_b = b.norm1_b;
        args.norm2_w = b.norm2_w;
        args.norm2_b = b.norm2_b;
        args.qkv = b.qkv;
        args.proj = b.proj;
        args.fc1 = b.fc1;
        args.fc2 = b.fc2;
        args.qkv_b = b.qkv_b;
        args.proj_b = b.proj_b;
        args.fc1_b = b.fc1_b;
        args.fc2_b = b.fc2_b;
        args.freqs = b.freqs_cis;
        launch_vit_block(args, x, batch, grid_w, grid_h, scratch.ptr, state, stream);
        for (const samq_weights* w : handles) const_cast<samq_weights*>(w)->launches.fetch_add(1);
    }
}

samq_status samq_vit_block_forward_v1(const samq_vit_block_v1* block, float* x, int grid_w, int grid_h,
                                      void* stream_ptr) {
    return guarded([&] { vit_block_forward(block, x, 1, grid_w, grid_h, stream_ptr); });
}

samq_status samq_vit_block_forward_batch_v1(const samq_vit_block_v1* block, float* x, int batch, int grid_w,
                                            int grid_h, void* stream_ptr) {
    return guarded([&] { vit_block_forward(block, x, batch, grid_w, grid_h, stream_ptr); });
}

static void vit_prefix(const float* image, int width, int height, int patch, const float* patch_w, int64_t embed,
                       const float* pos_embed, int pos_grid, const float* ln_w, const float* ln_b, float* x,
                       int compute, void* stream_ptr) {
    {
        require(compute == SAMQ_COMPUTE_F32 || compute == SAMQ_COMPUTE_F16, "compute must be SAMQ_COMPUTE_F32 or _F16");
        require(embed == 256 || embed == 512 || embed == 1024, "embedding width must be 256, 512 or 1024");
        require(patch > 0 && patch <= 32 && width > 0 && height > 0 && width % patch == 0 && height % patch == 0,
                "image sides must be positive multiples of the patch size (patch <= 32)");
        const int64_t tokens = static_cast<int64_t>(width / patch) * (height / patch);
        require(tokens <= (int64_t(1) << 20), "too many tokens");
        require(pos_grid > 0, "pos_grid must be positive");
        const float* params[] = {image, patch_w, pos_embed, ln_w, ln_b, x};
        for (const float* p : params) require(p != nullptr && aligned16(p), "arguments must be 16-byte aligned device pointers");
        DeviceState& state = device_state(current_device());
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        Scratch& scratch = scratch_for(state, stream, vit_prefix_scratch_bytes(tokens, embed, patch, compute));
        launch_vit_prefix(image, width, height, patch, patch_w, embed, pos_embed, pos_grid, ln_w, ln_b, x, compute,
                          scratch.ptr, state, stream);
    }
}

samq_status samq_vit_prefix_v1(const float* image, int width, int height, int patch, const float* patch_w,
                               int64_t embed, const float* pos_embed, int pos_grid, const float* ln_w,
                               const float* ln_b, float* x, void* stream_ptr) {
    return guarded([&] {
        vit_prefix(image, width, height, patch, patch_w, embed, pos_embed, pos_grid, ln_w, ln_b, x, SAMQ_COMPUTE_F16,
                   stream_ptr);
    });
}

samq_status samq_vit_prefix_v2(const float* image, int width, int height, int patch, const float* patch_w,
                               int64_t embed, const float* pos_embed, int pos_grid, const float* ln_w,
                               const float* ln_b, float* x, int compute, void* stream_ptr) {
    return guarded([&] {
        vit_prefix(image, width, height, patch, patch_w, embed, pos_embed, pos_grid, ln_w, ln_b, x, compute,
                   stream_ptr);
    });
}

samq_status samq_text_block_forward_v1(const samq_text_block_v1* block, float* x, int tokens, void* stream_ptr) {
    return guarded([&] {
        require(block != nullptr && block->version == 1, "text block descriptor missing or not version 1");
        const samq_text_block_v1& b = *block;
        require(b.in_proj && b.out_proj && b.fc1 && b.fc2, "null weight handle");
        const int64_t E = b.in_proj->k, mlp = b.fc1->n;
        require(E % 64 == 0 && E <= 4096 && b.in_proj->n == 3 * E && b.out_proj->k == E && b.out_proj->n == E &&
                    b.fc1->k == E && b.fc2->k == mlp && b.fc2->n == E,
                "linear shapes must be in_proj E->3E, out_proj E->E, fc1 E->MLP, fc2 MLP->E (E % 64 == 0)");
        require(mlp % 32 == 0, "MLP width must be a multiple of 32");
        require(tokens > 0 && tokens <= 4096, "token count out of range");
        const float* params[] = {b.norm1_w, b.norm1_b, b.in_proj_b, b.out_proj_b, b.norm2_w, b.norm2_b,
                                 b.fc1_b, b.fc2_b, x};
        for (const float* p : params) require(p != nullptr && aligned16(p), "parameters must be 16-byte aligned device pointers");
        const int device = current_device();
        for (const samq_weights* w : {b.in_proj, b.out_proj, b.fc1, b.fc2})
            require(w->device == device, "weight handle belongs to another device");
        DeviceState& state = device_state(device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        TextBlockArgs args;
        args.norm1_w = b.norm1_w;
        args.norm1_b = b.norm1_b;
        args.norm2_w = b.norm2_w;
        args.norm2_b = b.norm2_b;
        args.in_proj = b.in_proj;
        args.out_proj = b.out_proj;
        args.fc1 = b.fc1;
        args.fc2 = b.fc2;
        args.in_proj_b = b.in_proj_b;
        args.out_proj_b = b.out_proj_b;
        args.fc1_b = b.fc1_b;
        args.fc2_b = b.fc2_b;
        Scratch& scratch = scratch_for(state, stream, text_block_scratch_bytes(args, tokens, state.sm_count));
        launch_text_block(args, x, tokens, scratch.ptr, state, stream);
        for (const samq_weights* w : {b.in_proj, b.out_proj, b.fc1, b.fc2})
            const_cast<samq_weights*>(w)->launches.fetch_add(1);
    });
}

samq_status samq_token_embed_v1(const float* table, int64_t vocab, int width, const int32_t* ids, int count,
                                const float* pos, float* out, void* stream_ptr) {
    return guarded([&] {
        require(vocab > 0 && width > 0 && width <= (1 << 20) && count >= 0 && count <= (1 << 20),
                "embedding sizes out of range");
        if (count == 0) return;
        require(table && ids && out, "null pointer");
        for (int i = 0; i < count; ++i)
            require(ids[i] >= 0 && ids[i] < vocab, "token id outside the vocabulary");
        DeviceState& state = device_state(current_device());
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        Scratch& scratch = scratch_for(state, stream, static_cast<size_t>(count) * sizeof(int32_t) + 256);
        check_cuda(cudaMemcpyAsync(scratch.ptr, ids, static_cast<size_t>(count) * sizeof(int32_t),
                                   cudaMemcpyHostToDevice, stream),
                   "cudaMemcpyAsync(token ids)");
        launch_embed_rows(table, static_cast<const int32_t*>(scratch.ptr), pos, count, width, out, stream);
        // The host ids may be reused by the caller as soon as this returns.
        check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize(token ids)");
    });
}

samq_status samq_layer_norm_v1(const float* x, int64_t rows, int width, int64_t ldx, const float* w, const float* b,
                               float eps, float* out, int64_t ldo, void* stream_ptr) {
    return guarded([&] {
        require(rows >= 0 && width > 0 && ldx >= width && ldo >= width, "layer norm sizes out of range");
        require(eps > 0.0f, "eps must be positive");
        if (rows == 0) return;
        require(x && w && out, "null pointer");
        device_state(current_device());
        launch_layer_norm_f32(x, rows, width, ldx, w, b, out, ldo, eps, static_cast<cudaStream_t>(stream_ptr));
    });
}

samq_status samq_attention_v1(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                              int lq, int lk, int heads, int head_dim, float scale, int causal, const float* bias,
                              int64_t bias_h, int64_t bias_q, float* out, int64_t ldo, void* stream_ptr) {
    return guarded([&] {
        require(head_dim == 32 || head_dim == 64, "head_dim must be 32 or 64");
        require(heads > 0 && heads <= 256 && lq >= 0 && lk > 0 && lq <= (1 << 22) && lk <= (1 << 22),
                "attention sizes out of range");
        const int64_t E = int64_t(heads) * head_dim;
        require(ldq >= E && ldk >= E && ldv >= E && ldo >= E && ldq % 4 == 0 && ldk % 4 == 0 && ldv % 4 == 0,
                "row strides must cover heads * head_dim and be multiples of 4 floats");
        if (lq == 0) return;
        require(q && k && v && out && aligned16(q) && aligned16(k) && aligned16(v), "q, k, v must be 16-byte aligned");
        DeviceState& state = device_state(current_device());
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        // Scratch: the key-split partials of the SIMT kernel, or the K / V^T
        // TF32 planes of the tensor-core kernel (never both).
        const size_t part = attention_partial_floats(lq, lk, heads, head_dim, causal, state.sm_count);
        const size_t plane_bytes = attention_gen_plane_bytes(lq, lk, heads, head_dim, causal, bias, out, ldo);
        float* partials = nullptr;
        float* planes = nullptr;
        if (plane_bytes > 0) planes = static_cast<float*>(scratch_for(state, stream, plane_bytes).ptr);
        else if (part > 0) partials = static_cast<float*>(scratch_for(state, stream, part * sizeof(float)).ptr);
        launch_attention_gen(q, ldq, k, ldk, v, ldv, lq, lk, heads, head_dim, scale, causal, bias, bias_h, bias_q,
                             out, ldo, state, stream, partials, part, planes);
    });
}

static void check_linear_ref(const samq_linear_ref_v1& l, int64_t k, int64_t n, int device, const char* what) {
    const std::string name(what);
    require((l.quantized != nullptr) != (l.dense != nullptr), (name + ": exactly one of quantized / dense").c_str());
    if (l.dense) require(l.dense->kind == SAMQ_DENSE_LINEAR, (name + ": dense handle is not a LINEAR").c_str());
    require(linear_in(l) == k && linear_out(l) == n, (name + ": unexpected shape").c_str());
    require((l.quantized ? l.quantized->device : l.dense->device) == device, (name + ": handle on another device").c_str());
    require(l.bias == nullptr || aligned16(l.bias), (name + ": bias must be 16-byte aligned").c_str());
}

samq_status samq_fusion_layer_forward_v1(const samq_fusion_layer_v1* layer, float* x, const float* pos, int tokens,
                                         const float* prompt, const float* prompt_bias, int prompt_tokens,
                                         void* stream_ptr) {
    return guarded([&] {
        require(layer != nullptr && layer->version == 1, "fusion layer descriptor missing or not version 1");
        const samq_fusion_layer_v1& ly = *layer;
        require(ly.sa_in_proj.quantized || ly.sa_in_proj.dense, "sa_in_proj missing");
        const int64_t D = linear_in(ly.sa_in_proj);
        require(D % 128 == 0 && D <= 4096 && ly.heads > 0 && D % ly.heads == 0 &&
                    (D / ly.heads == 32 || D / ly.heads == 64),
                "width must be a multiple of 128 with heads of 32 or 64 channels");
        const int device = current_device();
        require(ly.linear1.quantized || ly.linear1.dense, "linear1 missing");
        const int64_t F = linear_out(ly.linear1);
        check_linear_ref(ly.sa_in_proj, D, 3 * D, device, "sa_in_proj");
        check_linear_ref(ly.sa_out_proj, D, D, device, "sa_out_proj");
        check_linear_ref(ly.ca_in_proj, D, 3 * D, device, "ca_in_proj");
        check_linear_ref(ly.ca_out_proj, D, D, device, "ca_out_proj");
        check_linear_ref(ly.linear1, D, F, device, "linear1");
        check_linear_ref(ly.linear2, F, D, device, "linear2");
        require(F % 32 == 0, "FFN width must be a multiple of 32");
        require(tokens > 0 && tokens <= (1 << 22) && prompt_tokens > 0 && prompt_tokens <= 4096, "token counts out of range");
        const float* params[] = {ly.norm1_w, ly.norm1_b, ly.norm2_w, ly.norm2_b, ly.norm3_w, ly.norm3_b, x, pos, prompt};
        for (const float* p : params) require(p != nullptr && aligned16(p), "parameters must be 16-byte aligned device pointers");
        DeviceState& state = device_state(device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        Scratch& scratch = scratch_for(state, stream, fusion_layer_scratch_bytes(ly, tokens, prompt_tokens, state.sm_count));
        launch_fusion_layer(ly, x, pos, tokens, prompt, prompt_bias, prompt_tokens, scratch.ptr, state, stream);
    });
}

samq_status samq_decoder_forward_v1(const samq_decoder_v1* decoder, const float* enc, const float* enc_pos, int grid,
                                    const float* prompt, const float* prompt_bias, const float* prompt_valid,
                                    int prompt_tokens, float* queries_out, float* boxes, float* scores,
                                    float* presence, void* stream_ptr) {
    return guarded([&] {
        require(decoder != nullptr && decoder->version == 1, "decoder descriptor missing or not version 1");
        const samq_decoder_v1& d = *decoder;
        require(d.layers > 0 && d.layers <= 64 && d.layer != nullptr && d.queries > 0 && d.queries <= 4096,
                "decoder layer / query counts out of range");
        require(d.layer[0].sa_in_proj.quantized || d.layer[0].sa_in_proj.dense, "sa_in_proj missing");
        const int64_t D = linear_in(d.layer[0].sa_in_proj);
        require(D % 128 == 0 && d.heads > 0 && d.heads <= 16 && D % d.heads == 0 &&
                    (D / d.heads == 32 || D / d.heads == 64),
                "width must be a multiple of 128 with at most 16 heads of 32 or 64 channels");
        const int device = current_device();
        require(d.layer[0].linear1.quantized || d.layer[0].linear1.dense, "linear1 missing");
        const int64_t F = linear_out(d.layer[0].linear1);
        for (int i = 0; i < d.layers; ++i) {
            const samq_decoder_layer_v1& ly = d.layer[i];
            check_linear_ref(ly.sa_in_proj, D, 3 * D, device, "sa_in_proj");
            check_linear_ref(ly.sa_out_proj, D, D, device, "sa_out_proj");
            check_linear_ref(ly.ca_text_in_proj, D, 3 * D, device, "ca_text_in_proj");
            check_linear_ref(ly.ca_text_out_proj, D, D, device, "ca_text_out_proj");
            check_linear_ref(ly.ca_in_proj, D, 3 * D, device, "ca_in_proj");
            check_linear_ref(ly.ca_out_proj, D, D, device, "ca_out_proj");
            check_linear_ref(ly.linear1, D, F, device, "linear1");
            check_linear_ref(ly.linear2, F, D, device, "linear2");
            const float* norms[] = {ly.norm1_w, ly.norm1_b, ly.norm2_w, ly.norm2_b, ly.norm_ca_text_w,
                                    ly.norm_ca_text_b, ly.norm3_w, ly.norm3_b};
            for (const float* p : norms) require(p != nullptr, "decoder norm missing");
        }
        check_linear_ref(d.ref_point_head[0], 512, D, device, "ref_point_head.0");
        check_linear_ref(d.ref_point_head[1], D, D, device, "ref_point_head.1");
        check_linear_ref(d.bbox_embed[0], D, D, device, "bbox_embed.0");
        check_linear_ref(d.bbox_embed[1], D, D, device, "bbox_embed.1");
        check_linear_ref(d.bbox_embed[2], D, 4, device, "bbox_embed.2");
        check_linear_ref(d.rpb_x1, 256, d.heads, device, "boxRPB_embed_x.1");
        check_linear_ref(d.rpb_y1, 256, d.heads, device, "boxRPB_embed_y.1");
        check_linear_ref(d.presence_head[0], D, D, device, "presence_token_head.0");
        check_linear_ref(d.presence_head[1], D, D, device, "presence_token_head.1");
        check_linear_ref(d.presence_head[2], D, 1, device, "presence_token_head.2");
        require(d.prompt_mlp[0].quantized || d.prompt_mlp[0].dense, "prompt_mlp missing");
        const int64_t Fp = linear_out(d.prompt_mlp[0]);
        check_linear_ref(d.prompt_mlp[0], D, Fp, device, "prompt_mlp.0");
        check_linear_ref(d.prompt_mlp[1], Fp, D, device, "prompt_mlp.1");
        check_linear_ref(d.prompt_proj, D, D, device, "prompt_proj");
        check_linear_ref(d.hs_proj, D, D, device, "hs_proj");
        require(grid > 0 && grid <= 256 && prompt_tokens > 0 && prompt_tokens <= 4096, "grid / prompt out of range");
        const float* params[] = {d.query_embed, d.presence_token, d.reference_points, d.rpb_x0_w, d.rpb_x0_b,
                                 d.rpb_y0_w, d.rpb_y0_b, d.norm_w, d.norm_b, d.presence_norm_w, d.presence_norm_b,
                                 d.prompt_mlp_norm_w, d.prompt_mlp_norm_b, enc, enc_pos, prompt, queries_out, boxes,
                                 scores, presence};
        for (const float* p : params) require(p != nullptr, "decoder parameter or buffer missing");
        require(aligned16(enc) && aligned16(enc_pos) && aligned16(prompt) && aligned16(queries_out),
                "activations must be 16-byte aligned");
        DeviceState& state = device_state(device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        const int64_t tokens = int64_t(grid) * grid;
        Scratch& scratch =
            scratch_for(state, stream, decoder_scratch_bytes(d, tokens, prompt_tokens, grid, state.sm_count));
        launch_decoder(d, enc, enc_pos, tokens, grid, prompt, prompt_bias, prompt_valid, prompt_tokens, queries_out,
                       boxes, scores, presence, scratch.ptr, state, stream);
    });
}

samq_status samq_geometry_encoder_forward_v1(const samq_geometry_encoder_v1* encoder, const float* image,
                                             const float* pos, int tokens, float* out, void* stream_ptr) {
    return guarded([&] {
        require(encoder != nullptr && encoder->version == 1, "geometry encoder descriptor missing or not version 1");
        const samq_geometry_encoder_v1& g = *encoder;
        require(g.layers > 0 && g.layers <= 16 && g.layer != nullptr, "geometry layer count out of range");
        require(g.final_proj.quantized || g.final_proj.dense, "final_proj missing");
        const int64_t D = linear_in(g.final_proj);
        require(D % 128 == 0 && D <= 4096 && g.heads > 0 && D % g.heads == 0 &&
                    (D / g.heads == 32 || D / g.heads == 64),
                "width must be a multiple of 128 with heads of 32 or 64 channels");
        const int device = current_device();
        check_linear_ref(g.final_proj, D, D, device, "final_proj");
        require(g.layer[0].linear1.quantized || g.layer[0].linear1.dense, "linear1 missing");
        const int64_t F = linear_out(g.layer[0].linear1);
        for (int i = 0; i < g.layers; ++i) {
            const samq_geometry_layer_v1& ly = g.layer[i];
            check_linear_ref(ly.sa_in_proj, D, 3 * D, device, "sa_in_proj");
            check_linear_ref(ly.sa_out_proj, D, D, device, "sa_out_proj");
            check_linear_ref(ly.ca_in_proj, D, 3 * D, device, "ca_in_proj");
            check_linear_ref(ly.ca_out_proj, D, D, device, "ca_out_proj");
            check_linear_ref(ly.linear1, D, F, device, "linear1");
            check_linear_ref(ly.linear2, F, D, device, "linear2");
            const float* norms[] = {ly.norm1_w, ly.norm1_b, ly.norm2_w, ly.norm2_b, ly.norm3_w, ly.norm3_b};
            for (const float* p : norms) require(p != nullptr, "geometry norm missing");
        }
        const float* params[] = {g.cls_token, g.norm_w, g.norm_b, g.encode_norm_w, g.encode_norm_b, image, pos, out};
        for (const float* p : params) require(p != nullptr, "geometry parameter or buffer missing");
        require(tokens > 0 && tokens <= (1 << 22), "token count out of range");
        require(aligned16(image) && aligned16(pos) && aligned16(g.cls_token), "inputs must be 16-byte aligned");
        DeviceState& state = device_state(device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        Scratch& scratch = scratch_for(state, stream, geometry_scratch_bytes(g, tokens, state.sm_count));
        launch_geometry_encoder(g, image, pos, tokens, out, scratch.ptr, state, stream);
    });
}

samq_status samq_seg_head_forward_v1(const samq_seg_head_v1* head, const float* enc, int grid, const float* fpn0,
                                     const float* fpn1, const float* queries, int nq, const float* prompt,
                                     const float* prompt_bias, int prompt_tokens, float* mask_logits,
                                     void* stream_ptr) {
    return guarded([&] {
        require(head != nullptr && head->version == 1, "segmentation head descriptor missing or not version 1");
        const samq_seg_head_v1& h = *head;
        require(h.ca_in_proj.quantized || h.ca_in_proj.dense, "ca_in_proj missing");
        const int64_t D = linear_in(h.ca_in_proj);
        require((D == 128 || D == 256 || D == 512 || D == 1024) && h.heads > 0 && D % h.heads == 0 &&
                    (D / h.heads == 32 || D / h.heads == 64),
                "width must be 128, 256, 512 or 1024 with heads of 32 or 64 channels");
        const int device = current_device();
        check_linear_ref(h.ca_in_proj, D, 3 * D, device, "cross_attend_prompt.in_proj");
        check_linear_ref(h.ca_out_proj, D, D, device, "cross_attend_prompt.out_proj");
        for (int j = 0; j < 3; ++j) check_linear_ref(h.mask_embed[j], D, D, device, "mask_embed");
        for (int i = 0; i < 2; ++i) {
            const samq_dense* c = h.conv[i];
            require(c != nullptr && c->kind == SAMQ_DENSE_CONV && c->ks == 3 && c->cin == D && c->cout == D &&
                        c->device == device,
                    "pixel decoder convolutions must be 3x3 D -> D on this device");
            require(h.norm_w[i] != nullptr && h.norm_b[i] != nullptr, "pixel decoder norm missing");
        }
        const samq_dense* ins = h.instance;
        require(ins != nullptr && (ins->kind == SAMQ_DENSE_CONV || ins->kind == SAMQ_DENSE_LINEAR) && ins->ks == 1 &&
                    ins->cin == D && ins->cout == D && ins->device == device,
                "instance head must be a 1x1 D -> D convolution on this device");
        require(h.cross_attn_norm_w && h.cross_attn_norm_b, "cross_attn_norm missing");
        require(grid > 0 && grid <= 128 && nq > 0 && nq <= 4096 && prompt_tokens > 0 && prompt_tokens <= 4096,
                "grid / query / prompt count out of range");
        const float* bufs[] = {enc, fpn0, fpn1, queries, prompt, mask_logits};
        for (const float* p : bufs) require(p != nullptr, "segmentation head buffer missing");
        require(aligned16(enc) && aligned16(fpn0) && aligned16(fpn1) && aligned16(queries) && aligned16(prompt) &&
                    aligned16(mask_logits),
                "buffers must be 16-byte aligned");
        DeviceState& state = device_state(device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        Scratch& scratch =
            scratch_for(state, stream, seg_head_scratch_bytes(h, grid, nq, prompt_tokens, state.sm_count));
        launch_seg_head(h, enc, grid, fpn0, fpn1, queries, nq, prompt, prompt_bias, prompt_tokens, mask_logits,
                        scratch.ptr, state, stream);
    });
}

samq_status samq_mmq_weights_create_v1(int device, int type, int variant, int64_t k, int64_t n, const void* gguf_rows,
                                       size_t bytes, void* stream_ptr, samq_mmq_weights** out) {
    return guarded([&] {
        require(out != nullptr, "null output handle");
        *out = nullptr;
        require(type == SAMQ_TYPE_Q8_0, "the exact MMQ path takes Q8_0 weights");
        require(variant == SAMQ_MMQ_CODES_F16 || variant == SAMQ_MMQ_CODES_I8, "unknown code variant");
        require(k > 0 && k % 128 == 0 && k <= (int64_t(1) << 20), "width must be a positive multiple of 128");
        require(n > 0 && n % 2 == 0 && n <= (int64_t(1) << 24), "row count must be even and in range");
        require(gguf_rows != nullptr && bytes == static_cast<size_t>(row_bytes(type, k) * n),
                "GGUF payload size differs from n rows");
        DeviceState& state = device_state(device);
        (void)state;
        DeviceGuard guard(device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        auto* w = new samq_mmq_weights;
        std::unique_ptr<samq_mmq_weights, void (*)(samq_mmq_weights*)> hold(w, [](samq_mmq_weights* p) {
            if (p->codes) cudaFree(p->codes);
            if (p->scales) cudaFree(p->scales);
            delete p;
        });
        w->device = device;
        w->variant = variant;
        w->k = k;
        w->n = n;
        void* staging = nullptr;
        check_cuda(cudaMalloc(&staging, bytes), "cudaMalloc(mmq staging)");
        struct Free {
            void* p;
            ~Free() { cudaFree(p); }
        } free_staging{staging};
        check_cuda(cudaMalloc(&w->codes, static_cast<size_t>(n * k) * mmq_code_bytes(variant)), "cudaMalloc(codes)");
        check_cuda(cudaMalloc(reinterpret_cast<void**>(&w->scales), static_cast<size_t>(n * (k / 32)) * sizeof(float)),
                   "cudaMalloc(scales)");
        check_cuda(cudaMemcpyAsync(staging, gguf_rows, bytes, cudaMemcpyHostToDevice, stream), "cudaMemcpyAsync(rows)");
        launch_mmq_weights(variant, static_cast<const uint8_t*>(staging), n, k, w->codes, w->scales, stream);
        check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize(mmq weights)");
        *out = hold.release();
    });
}

samq_status samq_mmq_weights_destroy_v1(samq_mmq_weights* w) {
    return guarded([&] {
        if (!w) return;
        DeviceGuard guard(w->device);
        if (w->codes) cudaFree(w->codes);
        if (w->scales) cudaFree(w->scales);
        delete w;
    });
}

samq_status samq_linear_mmq_v1(const samq_mmq_weights* w, const float* x, int64_t m, int64_t ldx, const float* bias,
                               int epilogue, float* y, int64_t ldy, void* stream_ptr) {
    return guarded([&] {
        require(w != nullptr && w->codes != nullptr, "null weights");
        require(m > 0 && m <= (int64_t(1) << 24), "row count out of range");
        require(ldx >= w->k && ldx % 4 == 0 && ldy >= w->n && ldy % 4 == 0, "leading dimensions");
        require(x && y && aligned16(x) && aligned16(y), "x and y must be 16-byte aligned device pointers");
        require(epilogue == SAMQ_EPILOGUE_NONE || epilogue == SAMQ_EPILOGUE_GELU_ERF, "unknown epilogue");
        const int device = current_device();
        require(w->device == device, "weights belong to another device");
        DeviceState& state = device_state(device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        const size_t code_bytes = static_cast<size_t>(m * w->k) * mmq_code_bytes(w->variant);
        const size_t scale_bytes = static_cast<size_t>(m * (w->k / 32)) * sizeof(float);
        Scratch& scratch = scratch_for(state, stream, code_bytes + scale_bytes + 512);
        uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(scratch.ptr) + 255) & ~uintptr_t(255));
        float* dx = reinterpret_cast<float*>(base + ((code_bytes + 255) & ~size_t(255)));
        launch_mmq_stage(w->variant, x, m, w->k, ldx, base, dx, state.status, stream);
        launch_mmq_gemm(w->variant, base, dx, w->codes, w->scales, m, w->n, w->k, bias,
                        epilogue == SAMQ_EPILOGUE_GELU_ERF ? 1 : 0, y, ldy, state, stream);
    });
}

samq_status samq_quantize_rows_v1(int type, int64_t k, int64_t n, const float* src, void* dst, size_t bytes) {
    return guarded([&] {
        require(supported_type(type), "weight type must be Q8_0, Q4_K, Q5_K or Q6_K");
        require(n > 0 && n <= (int64_t(1) << 24), "row count out of range");
        const int64_t rb = row_bytes(type, k);
        require(rb > 0 && k <= (int64_t(1) << 20), "width is not a whole number of blocks");
        require(src != nullptr && dst != nullptr && bytes == static_cast<size_t>(rb * n),
                "output size differs from n packed rows");
        quantize_rows(type, k, n, src, static_cast<uint8_t*>(dst));
    });
}

samq_status samq_sine_pe_2d_v1(int h, int w, int d, float* out) {
    return guarded([&] {
        require(h > 0 && w > 0 && h <= 4096 && w <= 4096 && d > 0 && d % 2 == 0 && d <= 8192 && out != nullptr,
                "positional encoding size out of range");
        const int half = d / 2;
        const float scale = 2.0f * 3.14159265358979323846f;
        for (int y = 0; y < h; ++y) {
            const float py = (static_cast<float>(y + 1) / static_cast<float>(h)) * scale;
            for (int x = 0; x < w; ++x) {
                const float px = (static_cast<float>(x + 1) / static_cast<float>(w)) * scale;
                float* row = out + (static_cast<int64_t>(y) * w + x) * d;
                for (int i = 0; i < half; ++i) {
                    const float dim_t = powf(10000.0f, static_cast<float>(i & ~1) / static_cast<float>(half));
                    row[i] = (i % 2 == 0) ? sinf(py / dim_t) : cosf(py / dim_t);
                    row[half + i] = (i % 2 == 0) ? sinf(px / dim_t) : cosf(px / dim_t);
                }
            }
        }
    });
}

samq_status samq_dense_create_v1(int device, int type, int kind, int kw, int kh, int64_t cin, int64_t cout,
                                 const void* data, size_t bytes, void* stream_ptr, samq_dense** out) {
    return guarded([&] {
        require(out != nullptr, "null output handle");
        *out = nullptr;
        require(type == SAMQ_TYPE_F32 || type == SAMQ_TYPE_F16, "dense weight type must be F32 or F16");
        require(cin > 0 && cout > 0 && cin <= (int64_t(1) << 20) && cout <= (int64_t(1) << 20),
                "channel counts out of range");
        int64_t n = 0, k = 0;
        switch (kind) {
            case SAMQ_DENSE_LINEAR:
                require(kw == 1 && kh == 1, "a linear has kw == kh == 1");
                require(cin % 4 == 0, "linear width must be a multiple of 4");
                n = cout;
                k = cin;
                break;
            case SAMQ_DENSE_CONV:
                require(kw == kh && (kw == 1 || kw == 3), "convolution kernels are 1x1 or 3x3");
                require(cin % 32 == 0, "convolution input channels must be a multiple of 32");
                n = cout;
                k = cin * kw * kh;
                break;
            case SAMQ_DENSE_DECONV2X2:
                require(kw == 2 && kh == 2, "the transposed convolution is 2x2");
                require(cin % 32 == 0 && cout % 32 == 0, "deconvolution channels must be multiples of 32");
                n = 4 * cout;
                k = cin;
                break;
            default: fail(SAMQ_ERR_INVALID_ARGUMENT, "unknown dense kind");
        }
        require(n * k <= (int64_t(1) << 31), "weight too large");
        const size_t elem = type == SAMQ_TYPE_F32 ? 4 : 2;
        require(data != nullptr && bytes == static_cast<size_t>(n * k) * elem, "payload size differs from the shape");
        DeviceState& state = device_state(device);
        DeviceGuard guard(device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        std::unique_ptr<samq_dense, void (*)(samq_dense*)> w(new samq_dense, release_dense);
        w->device = device;
        w->type = type;
        w->kind = kind;
        w->ks = kw;
        w->cin = cin;
        w->cout = cout;
        w->n = n;
        w->k = k;
        void* staging = nullptr;
        struct Free {
            void*& p;
            ~Free() {
                if (p) cudaFree(p);
            }
        } free_staging{staging};
        check_cuda(cudaMalloc(&staging, bytes), "cudaMalloc(dense staging)");
        check_cuda(cudaMalloc(reinterpret_cast<void**>(&w->hi), static_cast<size_t>(n * k) * 4), "cudaMalloc(dense hi)");
        check_cuda(cudaMalloc(reinterpret_cast<void**>(&w->lo), static_cast<size_t>(n * k) * 4), "cudaMalloc(dense lo)");
        check_cuda(cudaMemcpyAsync(staging, data, bytes, cudaMemcpyHostToDevice, stream), "cudaMemcpyAsync(H2D)");
        launch_dense_prep(staging, type, kind, kw, cin, cout, n, k, w->hi, w->lo, state, stream);
        check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize(dense prep)");
        *out = w.release();
    });
}

samq_status samq_dense_destroy_v1(samq_dense* weights) {
    return guarded([&] { release_dense(weights); });
}

samq_status samq_dense_linear_v1(const samq_dense* w, const float* x, int64_t m, int64_t ldx, const float* bias,
                                 int epilogue, float* y, int64_t ldy, void* stream_ptr) {
    return guarded([&] {
        require(w != nullptr && w->kind == SAMQ_DENSE_LINEAR, "weights must be a dense LINEAR handle");
        require(m >= 0 && m <= (int64_t(1) << 30), "row count out of range");
        require(epilogue == SAMQ_EPILOGUE_NONE || epilogue == SAMQ_EPILOGUE_GELU_ERF, "unknown epilogue");
        require(ldx >= w->k && ldx % 4 == 0, "input row stride must be >= k and a multiple of 4 floats");
        require(ldy >= w->n && ldy % 4 == 0, "output row stride must be >= n and a multiple of 4 floats");
        if (m == 0) return;
        require(x != nullptr && y != nullptr && aligned16(x) && aligned16(y), "pointers must be 16-byte aligned");
        require(w->device == current_device(), "dense handle belongs to another device");
        DeviceState& state = device_state(w->device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        const size_t half = static_cast<size_t>(m * w->k);
        Scratch& scratch = scratch_for(state, stream, 2 * half * sizeof(float) + 256);
        float* xh = static_cast<float*>(scratch.ptr);
        float* xl = xh + (half + 63) / 64 * 64;
        launch_split_rows(x, m, w->k, ldx, xh, xl, state, stream);
        launch_dense_gemm(xh, xl, *w, m, 0, 0, bias, epilogue, y, nullptr, ldy, state, stream);
    });
}

samq_status samq_conv2d_v1(const samq_dense* w, const float* x, int width, int height, const float* bias,
                           int epilogue, float* y, void* stream_ptr) {
    return guarded([&] {
        require(w != nullptr && (w->kind == SAMQ_DENSE_CONV || w->kind == SAMQ_DENSE_DECONV2X2),
                "weights must be a dense CONV or DECONV2X2 handle");
        require(width > 0 && height > 0 && int64_t(width) * height <= (int64_t(1) << 26), "image size out of range");
        require(epilogue == SAMQ_EPILOGUE_NONE || epilogue == SAMQ_EPILOGUE_GELU_ERF, "unknown epilogue");
        require(x != nullptr && y != nullptr && aligned16(x) && aligned16(y), "pointers must be 16-byte aligned");
        require(w->device == current_device(), "dense handle belongs to another device");
        DeviceState& state = device_state(w->device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        const int64_t pixels = int64_t(width) * height;
        const size_t half = static_cast<size_t>(pixels * w->cin);
        Scratch& scratch = scratch_for(state, stream, 2 * half * sizeof(float) + 256);
        float* xh = static_cast<float*>(scratch.ptr);
        float* xl = xh + (half + 63) / 64 * 64;
        launch_split_rows(x, pixels, w->cin, w->cin, xh, xl, state, stream);
        if (w->kind == SAMQ_DENSE_DECONV2X2)
            launch_dense_gemm(xh, xl, *w, pixels, width, 0, bias, epilogue, y, nullptr, w->cout, state, stream);
        else
            launch_dense_gemm(xh, xl, *w, pixels, width, height, bias, epilogue, y, nullptr, w->cout, state, stream);
    });
}

samq_status samq_maxpool2x2_v1(const float* x, int width, int height, int64_t channels, float* y, void* stream) {
    return guarded([&] {
        require(width > 0 && height > 0 && int64_t(width) * height <= (int64_t(1) << 26), "image size out of range");
        require(channels > 0 && channels % 4 == 0 && channels <= (int64_t(1) << 20), "channels must be a multiple of 4");
        require(x != nullptr && y != nullptr && aligned16(x) && aligned16(y), "pointers must be 16-byte aligned");
        DeviceState& state = device_state(current_device());
        launch_maxpool2x2(x, width, height, channels, y, nullptr, state, static_cast<cudaStream_t>(stream));
    });
}

samq_status samq_neck_forward_v1(const samq_neck_v1* neck, const float* x, int grid_w, int grid_h,
                                 float* const out[4], void* stream_ptr) {
    return guarded([&] {
        require(neck != nullptr && neck->version == 1, "neck descriptor must have version 1");
        require(grid_w >= 2 && grid_h >= 2 && int64_t(grid_w) * grid_h <= (int64_t(1) << 20), "grid out of range");
        require(x != nullptr && aligned16(x) && out != nullptr, "null or misaligned pointer");
        for (int i = 0; i < 4; ++i) require(out[i] != nullptr && aligned16(out[i]), "null or misaligned output");
        const int device = current_device();
        const samq_dense* layers[] = {neck->s0_deconv1, neck->s0_deconv2, neck->s0_conv1x1, neck->s0_conv3x3,
                                      neck->s1_deconv1, neck->s1_conv1x1, neck->s1_conv3x3, neck->s2_conv1x1,
                                      neck->s2_conv3x3, neck->s3_conv1x1, neck->s3_conv3x3};
        for (const samq_dense* w : layers) {
            require(w != nullptr, "neck weight missing");
            require(w->device == device, "neck weight belongs to another device");
        }
        DeviceState& state = device_state(device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        Scratch& scratch = scratch_for(state, stream, neck_scratch_bytes(*neck, grid_w, grid_h));
        launch_neck(*neck, x, grid_w, grid_h, out, scratch.ptr, state, stream);
    });
}

samq_status samq_query_v1(const samq_weights* w, struct samq_counters_v1* out) {
    return guarded([&] {
        require(w != nullptr && out != nullptr, "null argument");
        std::memset(out, 0, sizeof(*out));
        out->version = 1;
        out->path = 1;
        out->launches = w->launches.load();
        out->payload_bytes = w->payload_bytes.load();
        out->allocation_bytes = w->allocation_bytes.load();
        out->weight_bytes = w->packet_bytes + w->operand_bytes;
    });
}

samq_status samq_check_v1(int device, void* stream) {
    samq_status found = SAMQ_OK;
    const samq_status rc = guarded([&] {
        int count = 0;
        check_cuda(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
        require(device >= 0 && device < count && device < 64, "device index is not visible");
        DeviceGuard guard(device);
        check_cuda(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize(check)");
        // The library's status word (only if its device state exists: a caller
        // that only used the allocation-free path has none, and checking must
        // not create one) merged with the allocation-free path's own word.
        DeviceStatus host{};
        if (DeviceState* state = existing_device_state(device)) {
            check_cuda(cudaMemcpy(&host, state->status, sizeof(host), cudaMemcpyDeviceToHost), "cudaMemcpy(status)");
            check_cuda(cudaMemset(state->status, 0, sizeof(DeviceStatus)), "cudaMemset(status)");
        }
        DeviceStatus fixed{};
        if (take_static_status(device, &fixed)) {
            host.flags |= fixed.flags;
            host.range_blocks += fixed.range_blocks;
            if (fixed.flags & kStatusTimeout) host.timeout_site = fixed.timeout_site;
        }
        if (host.flags & kStatusTimeout) {
            found = SAMQ_ERR_TIMEOUT;
            fail(SAMQ_ERR_TIMEOUT, "a device-side wait timed out at site " + std::to_string(host.timeout_site));
        }
        if (host.flags & kStatusLayout) {
            found = SAMQ_ERR_UNSUPPORTED;
            fail(SAMQ_ERR_UNSUPPORTED, "a kernel skipped its work: dynamic shared memory base misaligned");
        }
        if (host.flags & kStatusRange) {
            found = SAMQ_ERR_RANGE;
            fail(SAMQ_ERR_RANGE, std::to_string(host.range_blocks) +
                                     " activation warps held non-finite or out-of-range values");
        }
    });
    return rc != SAMQ_OK ? rc : found;
}

}  // extern "C"
