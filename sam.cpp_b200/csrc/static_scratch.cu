// static_scratch.cu -- samq_linear_static_v1, the allocation-free variant of
// samq_linear_v1.
//
// samq_linear_v1 stages the f16 activation operand in scratch memory that the
// library grows with cudaMalloc on first use per stream.  Some callers cannot
// let a library allocate: an embedding framework whose caching allocator has
// already reserved the GPU's memory (a cudaMalloc would fail or fragment its
// pool), serving loops where cudaMalloc's implicit device synchronization
// stalls the other streams, and hosts that must not meet an out-of-memory
// error in the middle of a request.  For them this entry point keeps the
// operand in a fixed file-scope device array instead; it calls no cudaMalloc,
// cudaFree or allocating library routine.
//
// The array holds kStaticOperandElements f16 values (32 MiB), and every GPU
// that loads the library holds its own copy until the process exits.  All
// calls on a device share it and it keeps the last call's contents: nothing
// needs to start at zero, because the staging kernel overwrites every element
// of [m][k] that the GEMM then reads (rows past m and columns past k are
// zero-filled by the tensor-memory copies, not read from the array).  Calls
// whose GPU work overlaps in time (different streams, or host threads sharing
// a device without ordering) race on the array; order them on one stream.
#include <mutex>

#include "samq_internal.hpp"

namespace samq {
namespace {

constexpr int64_t kStaticOperandElements = SAMQ_STATIC_OPERAND_ELEMENTS;
constexpr int kMaxDevices = 64;

// Staged activation operand (binary16 bit patterns).  In host code this name
// is only a stand-in for the device symbol; its device address comes from
// cudaGetSymbolAddress.
static __device__ __align__(256) uint16_t g_static_operand[kStaticOperandElements];
// Findings of this path (range, timeout), read and cleared by samq_check_v1.
// Zero-initialized when the module loads.
static __device__ __align__(16) DeviceStatus g_static_status;

// Per-device launch parameters and the two device addresses, filled once per
// device with that device current.
struct StaticDevice {
    bool ready = false;
    __half* operand = nullptr;
    DeviceStatus* status = nullptr;
    DeviceState launch;  // device, sm_count, cc_major; launch.status = status
};

std::mutex g_static_mutex;
StaticDevice g_static[kMaxDevices];

// Set-up of `device` (the caller's DeviceGuard makes it current): checks the
// architecture and looks up the device addresses of the two file-scope
// variables.  Makes no allocation.
StaticDevice& static_device(int device) {
    if (device < 0 || device >= kMaxDevices) fail(SAMQ_ERR_INVALID_ARGUMENT, "device index out of range");
    std::lock_guard<std::mutex> lock(g_static_mutex);
    StaticDevice& d = g_static[device];
    if (d.ready) return d;
    int sm_count = 0, cc_major = 0, cc_minor = 0;
    check_cuda(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, device),
               "cudaDeviceGetAttribute(SM count)");
    check_cuda(cudaDeviceGetAttribute(&cc_major, cudaDevAttrComputeCapabilityMajor, device),
               "cudaDeviceGetAttribute(compute capability)");
    check_cuda(cudaDeviceGetAttribute(&cc_minor, cudaDevAttrComputeCapabilityMinor, device),
               "cudaDeviceGetAttribute(compute capability)");
    if (cc_major != 10 || cc_minor != 0) fail(SAMQ_ERR_UNSUPPORTED, "samq kernels are built for sm_100a");
    void* operand = nullptr;
    void* status = nullptr;
    check_cuda(cudaGetSymbolAddress(&operand, g_static_operand), "cudaGetSymbolAddress(static operand)");
    check_cuda(cudaGetSymbolAddress(&status, g_static_status), "cudaGetSymbolAddress(static status)");
    if (!operand || !status) fail(SAMQ_ERR_CUDA, "static operand has no device address");
    d.operand = static_cast<__half*>(operand);
    d.status = static_cast<DeviceStatus*>(status);
    d.launch.device = device;
    d.launch.sm_count = sm_count;
    d.launch.cc_major = cc_major;
    d.launch.cc_minor = cc_minor;
    d.launch.status = d.status;
    d.ready = true;
    return d;
}

}  // namespace

bool take_static_status(int device, DeviceStatus* out) {
    DeviceStatus* status = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_static_mutex);
        if (device < 0 || device >= kMaxDevices || !g_static[device].ready) return false;
        status = g_static[device].status;
    }
    DeviceGuard guard(device);
    check_cuda(cudaMemcpy(out, status, sizeof(DeviceStatus), cudaMemcpyDeviceToHost), "cudaMemcpy(static status)");
    check_cuda(cudaMemset(status, 0, sizeof(DeviceStatus)), "cudaMemset(static status)");
    return true;
}

}  // namespace samq

extern "C" samq_status samq_linear_static_v1(const samq_weights* w, const float* x, int64_t m, int64_t ldx,
                                              const float* bias, int epilogue, float* y, int64_t ldy,
                                              void* stream_ptr) {
    using namespace samq;
    try {
        check_linear_args(w, m, bias, epilogue, y, ldy);
        check_activation_args(m, w->k, ldx, x, y);
        if (m > kStaticOperandElements / w->k)
            fail(SAMQ_ERR_INVALID_ARGUMENT,
                 "m * k exceeds the static operand capacity of SAMQ_STATIC_OPERAND_ELEMENTS "
                 "(16777216) elements; split the rows across calls");
        if (m > 0) {
            DeviceGuard guard(w->device);
            StaticDevice& d = static_device(w->device);
            cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
            launch_act_f16(x, m, w->k, ldx, d.operand, nullptr, d.status, stream);
            launch_gemm_f16(d.operand, w->k, w->operand, m, w->n, w->k, bias, epilogue, y, ldy, d.launch, stream);
        }
        set_last_error("");
        return SAMQ_OK;
    } catch (const Error& e) {
        set_last_error(e.message);
        return e.status;
    } catch (...) {
        set_last_error("unexpected internal failure");
        return SAMQ_ERR_CUDA;
    }
}
