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

// Staged activation operand (binary16 bit patterns).  In host code this name
// is only a stand-in for the device symbol; its device address comes from
// cudaGetSymbolAddress.
static __device__ __align__(256) uint16_t g_static_operand[kStaticOperandElements];

std::mutex g_static_mutex;
void* g_static_address[64] = {};

// Device address of g_static_operand on `device`, looked up once per device
// with that device current (the caller's DeviceGuard makes it current).
__half* static_operand(int device) {
    std::lock_guard<std::mutex> lock(g_static_mutex);
    if (!g_static_address[device]) {
        void* address = nullptr;
        check_cuda(cudaGetSymbolAddress(&address, g_static_operand), "cudaGetSymbolAddress(static operand)");
        if (!address) fail(SAMQ_ERR_CUDA, "static operand has no device address");
        g_static_address[device] = address;
    }
    return static_cast<__half*>(g_static_address[device]);
}

void require_arg(bool condition, const char* message) {
    if (!condition) fail(SAMQ_ERR_INVALID_ARGUMENT, message);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace samq

extern "C" samq_status samq_linear_static_v1(const samq_weights* w, const float* x, int64_t m, int64_t ldx,
                                              const float* bias, int epilogue, float* y, int64_t ldy,
                                              void* stream_ptr) {
    using namespace samq;
    try {
        require_arg(w != nullptr, "null weights");
        require_arg(m >= 0, "row count out of range");
        require_arg(epilogue == SAMQ_EPILOGUE_NONE || epilogue == SAMQ_EPILOGUE_GELU_ERF, "unknown epilogue");
        require_arg(ldx >= w->k && ldx % 4 == 0, "row stride must be >= width and a multiple of 4 floats");
        require_arg(ldy >= w->n && ldy % 4 == 0, "output row stride must be >= n and a multiple of 4 floats");
        require_arg(m <= kStaticOperandElements / w->k,
                    "m * k exceeds the static operand capacity of SAMQ_STATIC_OPERAND_ELEMENTS "
                    "(16777216) elements; split the rows across calls");
        if (m > 0) {
            require_arg(x != nullptr && aligned16(x), "activation pointer must be 16-byte aligned");
            require_arg(y != nullptr && aligned16(y), "output pointer must be 16-byte aligned");
            DeviceGuard guard(w->device);
            // Launch parameters without touching the library's device state
            // (creating that state allocates its status word).
            DeviceState launch;
            launch.device = w->device;
            check_cuda(cudaDeviceGetAttribute(&launch.sm_count, cudaDevAttrMultiProcessorCount, w->device),
                       "cudaDeviceGetAttribute(SM count)");
            check_cuda(cudaDeviceGetAttribute(&launch.cc_major, cudaDevAttrComputeCapabilityMajor, w->device),
                       "cudaDeviceGetAttribute(compute capability)");
            if (launch.cc_major != 10) fail(SAMQ_ERR_UNSUPPORTED, "samq kernels are built for sm_100a");
            launch.status = nullptr;  // no findings are recorded on this path; waits stay bounded
            __half* a = static_operand(w->device);
            cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
            launch_act_f16(x, m, w->k, ldx, a, nullptr, nullptr, stream);
            launch_gemm_f16(a, w->k, w->operand, m, w->n, w->k, bias, epilogue, y, ldy, launch, stream);
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
