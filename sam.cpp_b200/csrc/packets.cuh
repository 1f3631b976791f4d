// packets.cuh -- the K4 packet layout as seen by device code.
//
// A weight matrix [n][k] is stored as packets of 128 rows x 64 columns: packet
// (t, c) (rows 128t.., columns 64c..) holds, row after row, code_bytes_of(TYPE)
// bytes of codes for those 64 columns, then one 8-byte scale record per row.
// decode8 rebuilds 8 consecutive weights of a row exactly as gguf-py's f32
// dequantization of the GGUF block they came from.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "samq.h"

namespace samq {

__host__ __device__ constexpr int block_bytes_of(int type) {
    return type == SAMQ_TYPE_Q8_0 ? 34 : type == SAMQ_TYPE_Q4_K ? 144 : type == SAMQ_TYPE_Q5_K ? 176 : 210;
}
__host__ __device__ constexpr int code_bytes_of(int type) {
    return type == SAMQ_TYPE_Q8_0 ? 64 : type == SAMQ_TYPE_Q4_K ? 32 : type == SAMQ_TYPE_Q5_K ? 40 : 48;
}


// Decode 8 consecutive columns (8j .. 8j+7 of the 64-column chunk) of one
// packet row (codes `code`, scale record `rec`) into f32, with gguf-py's
// operation order.
template <int TYPE>
__device__ __forceinline__ void decode8(const uint8_t* __restrict__ code, const uint8_t* __restrict__ rec, int j,
                                        float (&w)[8]) {
    if constexpr (TYPE == SAMQ_TYPE_Q8_0) {
        const uint2 raw = *reinterpret_cast<const uint2*>(code + 8 * j);
        const float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(rec + 2 * (j >> 2))));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t word = i < 4 ? raw.x : raw.y;
            const int q = static_cast<int8_t>((word >> (8 * (i & 3))) & 0xffu);
            w[i] = __fmul_rn(static_cast<float>(q), d);
        }
    } else {
        const uint32_t lo = *reinterpret_cast<const uint32_t*>(code + 4 * j);
        uint32_t q[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = (lo >> (4 * i)) & 15u;
        if constexpr (TYPE == SAMQ_TYPE_Q5_K) {
            const uint32_t hb = code[32 + j];
#pragma unroll
            for (int i = 0; i < 8; ++i) q[i] |= ((hb >> i) & 1u) << 4;
        }
        if constexpr (TYPE == SAMQ_TYPE_Q6_K) {
            const uint32_t hb = *reinterpret_cast<const uint16_t*>(code + 32 + 2 * j);
#pragma unroll
            for (int i = 0; i < 8; ++i) q[i] |= ((hb >> (2 * i)) & 3u) << 4;
            const float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(rec)));
            const float ds = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(rec[2 + (j >> 1)])));
#pragma unroll
            for (int i = 0; i < 8; ++i) w[i] = __fmul_rn(ds, static_cast<float>(static_cast<int>(q[i]) - 32));
        } else {
            const float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(rec)));
            const float dmin = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(rec + 2)));
            const int s = j >> 2;
            const float ds = __fmul_rn(d, static_cast<float>(rec[4 + s]));
            const float dm = __fmul_rn(dmin, static_cast<float>(rec[6 + s]));
#pragma unroll
            for (int i = 0; i < 8; ++i) w[i] = __fsub_rn(__fmul_rn(ds, static_cast<float>(q[i])), dm);
        }
    }
}


}  // namespace samq
