// quantize.cu -- K1: activation staging for the quantized linears.
//
// Restates GGML CUDA's quantize_q8_1 (MMVQ staging, 36-byte blocks) and
// quantize_mmq_q8_1 (MMQ D4 staging, 144-byte blocks) as pinned by SAM.cpp's
// verifiers (tools/validation/verify_q8_rhs_staging.py:24-83,
// tools/validation/verify_q8_mmq_rhs_staging.py:24-67) and its scale rule
// patch (cmake/patches/ggml-precise-cuda.patch:623-633: the inverse scale is
// an IEEE round-to-nearest division).  The deterministic rule used here:
//   amax = max |x| over 32 values
//   d    = amax / 127            (f32, IEEE division; stored as f16 for Q8_1)
//   q    = roundf(x * (127/amax)) (half away from zero; 0 when amax == 0)
//   sum  = f16 of the f32 sum in 32-lane xor-butterfly order
// Besides the staged bytes, the kernel writes the tensor-core A operand of the
// GEMM: f16(f32(d_f16) * q), the exact decoded Q8_1 value rounded once.
//
// Memory layout: every thread owns 8 consecutive values (two 16-byte loads,
// one 16-byte f16 store); four neighbouring lanes form one 32-value block.
#include <algorithm>
#include <climits>

#include "samq_internal.hpp"

namespace samq {
namespace {


__device__ __forceinline__ void load8(const float* __restrict__ p, float (&v)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// amax over the 4-lane group (32 values).
__device__ __forceinline__ float group_amax(const float (&v)[8]) {
    float a = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) a = fmaxf(a, fabsf(v[j]));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    return a;
}

// Sum of the 32 values in the order of a 32-lane xor butterfly with offsets
// 16, 8, 4, 2, 1.  Element e = 8 * lane_in_group + j, so offsets 16 and 8 are
// lane offsets 2 and 1, and offsets 4, 2, 1 stay inside the thread.
__device__ __forceinline__ float group_butterfly_sum(const float (&v)[8]) {
    float s[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] = __fadd_rn(v[j], __shfl_xor_sync(0xffffffffu, v[j], 2));
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j] = __fadd_rn(s[j], __shfl_xor_sync(0xffffffffu, s[j], 1));
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j] = __fadd_rn(s[j], s[j + 4]);
    s[0] = __fadd_rn(s[0], s[2]);
    s[1] = __fadd_rn(s[1], s[3]);
    return __fadd_rn(s[0], s[1]);
}

// Low byte of an integral float q with |q| <= 127 (two's complement int8):
// adding 1.5 * 2^23 places the integer in the low mantissa bits.
__device__ __forceinline__ uint32_t code_byte(float q) {
    return __float_as_uint(__fadd_rn(q, 12582912.0f)) & 0xffu;
}

// One 8-value unit: staging arithmetic and stores.  Every lane of the warp
// calls it (shuffles), inactive lanes with zeros.
__device__ __forceinline__ void stage_unit(const float (&v)[8], bool active, int64_t row, int64_t c8, int64_t k,
                                           __half* __restrict__ a, uint8_t* __restrict__ q8_1,
                                           DeviceStatus* status) {
    const float amax = group_amax(v);
    const float d = __fdiv_rn(amax, 127.0f);
    const __half dh = __float2half_rn(d);
    const float dq = __half2float(dh);
    const float inv = amax == 0.0f ? 0.0f : __fdiv_rn(127.0f, amax);
    bool bad = false;
    float q[8];
    __align__(16) __half2 out[4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        bad |= !(fabsf(v[j]) <= kOperandLimit);
        q[j] = round_half_away(__fmul_rn(v[j], inv));
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) out[j] = __floats2half2_rn(__fmul_rn(dq, q[2 * j]), __fmul_rn(dq, q[2 * j + 1]));
    record_range(bad && active, status);
    if (q8_1) {
        const float sum = group_butterfly_sum(v);
        if (active) {
            const int lane_in_group = static_cast<int>(c8 & 3);
            uint8_t* blk = q8_1 + (row * (k / 32) + c8 / 4) * 36;
            uint32_t lo = 0, hi = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                lo |= code_byte(q[j]) << (8 * j);
                hi |= code_byte(q[j + 4]) << (8 * j);
            }
            uint32_t* words = reinterpret_cast<uint32_t*>(blk);
            words[1 + 2 * lane_in_group] = lo;
            words[2 + 2 * lane_in_group] = hi;
            if (lane_in_group == 0) {
                const __half hs = __float2half_rn(sum);
                words[0] = static_cast<uint32_t>(__half_as_ushort(dh)) |
                           (static_cast<uint32_t>(__half_as_ushort(hs)) << 16);
            }
        }
    }
    if (active && a) *reinterpret_cast<uint4*>(a + row * k + c8 * 8) = *reinterpret_cast<const uint4*>(out);
}

template <int U, class Index>
__global__ void __launch_bounds__(256) act_f16_kernel(const float* __restrict__ x, int64_t rows, int64_t k,
                                                      int64_t ld, __half* __restrict__ a,
                                                      uint8_t* __restrict__ q8_1, DeviceStatus* status) {
    // Index arithmetic in `Index` (uint32_t whenever rows * k / 8 < 2^32: a
    // 64-bit division per unit costs more than the unit's quantization).
    pdl_wait();     // X may come from, and the operand buffer may still be read by, the previous kernel
    pdl_trigger();  // the GEMM that consumes this operand may start its prologue
    const Index per_row = static_cast<Index>(k / 8);
    const Index units = static_cast<Index>(rows) * per_row;
    const Index total = static_cast<Index>(gridDim.x) * blockDim.x;
    for (Index base = static_cast<Index>(blockIdx.x) * blockDim.x + threadIdx.x;
         base - threadIdx.x % 32 < units; base += total * U) {
        float v[U][8];
        bool act[U];
        Index row[U], c8[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const Index idx = base + static_cast<Index>(u) * total;
            act[u] = idx < units;
            row[u] = act[u] ? idx / per_row : 0;
            c8[u] = act[u] ? idx - row[u] * per_row : 0;
            if (act[u]) {
                load8(x + static_cast<int64_t>(row[u]) * ld + static_cast<int64_t>(c8[u]) * 8, v[u]);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[u][j] = 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) stage_unit(v[u], act[u], row[u], c8[u], k, a, q8_1, status);
    }
}

__global__ void __launch_bounds__(256) q8_1_to_f16_kernel(const uint8_t* __restrict__ q8_1, int64_t rows, int64_t k,
                                                          __half* __restrict__ a) {
    const int64_t per_row = k / 8;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= rows * per_row) return;
    const int64_t row = idx / per_row, c8 = idx % per_row;
    const uint8_t* blk = q8_1 + (row * (k / 32) + c8 / 4) * 36;
    const uint32_t* words = reinterpret_cast<const uint32_t*>(blk);
    const float dq = __half2float(__ushort_as_half(static_cast<unsigned short>(words[0] & 0xffffu)));
    const uint32_t lo = words[1 + 2 * (c8 & 3)], hi = words[2 + 2 * (c8 & 3)];
    __align__(16) __half out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t w = j < 4 ? lo : hi;
        const int q = static_cast<int8_t>((w >> (8 * (j & 3))) & 0xffu);
        out[j] = __float2half_rn(__fmul_rn(dq, static_cast<float>(q)));
    }
    *reinterpret_cast<uint4*>(a + row * k + c8 * 8) = *reinterpret_cast<const uint4*>(out);
}

// MMQ D4: 128-value blocks {f32 d[4], int8 q[128]}, width padded to 512,
// stored [block][row].  16 threads per block, 4 per 32-value sub-block.
__global__ void __launch_bounds__(256) mmq_d4_kernel(const float* __restrict__ x, int64_t rows, int64_t k,
                                                     int64_t ld, int64_t padded, uint8_t* __restrict__ out) {
    const int64_t per_row = padded / 8;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const bool active = idx < rows * per_row;
    const int64_t row = active ? idx / per_row : 0;
    const int64_t c8 = active ? idx % per_row : 0;
    float v[8];
    const int64_t col = c8 * 8;
    if (active && col < k) {
        load8(x + row * ld + col, v);
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = 0.0f;
    }
    const float amax = group_amax(v);
    const float d = __fdiv_rn(amax, 127.0f);
    const float inv = amax == 0.0f ? 0.0f : __fdiv_rn(127.0f, amax);
    if (!active) return;
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        lo |= (static_cast<uint32_t>(static_cast<int>(roundf(__fmul_rn(v[j], inv)))) & 0xffu) << (8 * j);
        hi |= (static_cast<uint32_t>(static_cast<int>(roundf(__fmul_rn(v[j + 4], inv)))) & 0xffu) << (8 * j);
    }
    const int64_t blk = c8 / 16;            // 128-value block index
    const int sub = static_cast<int>((c8 / 4) & 3), lane_in_group = static_cast<int>(c8 & 3);
    uint8_t* o = out + (blk * rows + row) * 144;
    uint32_t* words = reinterpret_cast<uint32_t*>(o);
    words[4 + 8 * sub + 2 * lane_in_group] = lo;
    words[5 + 8 * sub + 2 * lane_in_group] = hi;
    if (lane_in_group == 0) reinterpret_cast<float*>(o)[sub] = d;
}

unsigned grid_for(int64_t threads) { return static_cast<unsigned>((threads + 255) / 256); }

}  // namespace

// Units per thread (1..4): each extra unit keeps two more 16-byte loads in
// flight but costs registers, i.e. resident blocks.  The choice minimizes
// (waves of resident blocks) x (units per thread), the length of the
// critical path in units per thread.
int choose_units_per_thread(int64_t units, int device) {
    static int sms[64] = {};
    static int occupancy[64][5] = {};
    if (!sms[device & 63]) {
        check_cuda(cudaDeviceGetAttribute(&sms[device & 63], cudaDevAttrMultiProcessorCount, device),
                   "cudaDeviceGetAttribute");
        const void* kernels[5] = {nullptr, reinterpret_cast<const void*>(act_f16_kernel<1, uint32_t>),
                                  reinterpret_cast<const void*>(act_f16_kernel<2, uint32_t>),
                                  reinterpret_cast<const void*>(act_f16_kernel<3, uint32_t>),
                                  reinterpret_cast<const void*>(act_f16_kernel<4, uint32_t>)};
        for (int u = 1; u <= 4; ++u)
            check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occupancy[device & 63][u], kernels[u], 256, 0),
                       "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    }
    int best = 1;
    int64_t best_cost = INT64_MAX;
    for (int u = 1; u <= 4; ++u) {
        const int64_t blocks = (units + 256 * u - 1) / (256 * u);
        const int64_t resident = static_cast<int64_t>(sms[device & 63]) * std::max(occupancy[device & 63][u], 1);
        const int64_t cost = (blocks + resident - 1) / resident * u;
        if (cost < best_cost) {
            best_cost = cost;
            best = u;
        }
    }
    return best;
}

void launch_act_f16(const float* x, int64_t rows, int64_t k, int64_t ld, __half* a_out, uint8_t* q8_1_out,
                    DeviceStatus* status, cudaStream_t stream) {
    if (rows == 0) return;
    int device = 0;
    check_cuda(cudaGetDevice(&device), "cudaGetDevice");
    const int64_t units = rows * (k / 8);
    const int u = choose_units_per_thread(units, device);
    if (units + 4 * 256 >= (int64_t(1) << 32)) {
        // Beyond 32-bit unit indices: 64-bit index math, 4 units per thread per pass.
        const unsigned grid = grid_for(std::min<int64_t>((units + 3) / 4, int64_t(1) << 24));
        launch_pdl(act_f16_kernel<4, uint64_t>, dim3(grid), dim3(256), 0, stream, "act_f16_kernel launch", x, rows, k,
                   ld, a_out, q8_1_out, status);
        check_cuda(cudaGetLastError(), "act_f16_kernel launch");
        return;
    }
    const unsigned grid = grid_for((units + u - 1) / u);
    switch (u) {
        case 1:
            launch_pdl(act_f16_kernel<1, uint32_t>, dim3(grid), dim3(256), 0, stream, "act_f16_kernel launch", x,
                       rows, k, ld, a_out, q8_1_out, status);
            break;
        case 2:
            launch_pdl(act_f16_kernel<2, uint32_t>, dim3(grid), dim3(256), 0, stream, "act_f16_kernel launch", x,
                       rows, k, ld, a_out, q8_1_out, status);
            break;
        case 3:
            launch_pdl(act_f16_kernel<3, uint32_t>, dim3(grid), dim3(256), 0, stream, "act_f16_kernel launch", x,
                       rows, k, ld, a_out, q8_1_out, status);
            break;
        default:
            launch_pdl(act_f16_kernel<4, uint32_t>, dim3(grid), dim3(256), 0, stream, "act_f16_kernel launch", x, rows,
                       k, ld, a_out, q8_1_out, status);
            break;
    }
    check_cuda(cudaGetLastError(), "act_f16_kernel launch");
}

void launch_q8_1_to_f16(const uint8_t* q8_1, int64_t rows, int64_t k, __half* a_out, DeviceStatus*,
                        cudaStream_t stream) {
    if (rows == 0) return;
    q8_1_to_f16_kernel<<<grid_for(rows * (k / 8)), 256, 0, stream>>>(q8_1, rows, k, a_out);
    check_cuda(cudaGetLastError(), "q8_1_to_f16_kernel launch");
}

void launch_mmq_d4(const float* x, int64_t rows, int64_t k, int64_t ld, uint8_t* out, cudaStream_t stream) {
    if (rows == 0) return;
    const int64_t padded = (k + 511) / 512 * 512;
    mmq_d4_kernel<<<grid_for(rows * (padded / 8)), 256, 0, stream>>>(x, rows, k, ld, padded, out);
    check_cuda(cudaGetLastError(), "mmq_d4_kernel launch");
}

}  // namespace samq
