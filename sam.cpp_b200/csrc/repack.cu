// repack.cu -- K4: load-time weight repack and its inverse.
//
// GGUF rows (gguf-py GGML_QUANT_SIZES: Q8_0 34 B / 32, Q4_K 144 B / 256,
// Q5_K 176 B / 256, Q6_K 210 B / 256; field order as in gguf/quants.py and
// src/models/sam3/weights.hpp:405-419) are rewritten into "packets": one
// packet per 128 rows x 64 columns, holding for each row the codes of those
// 64 columns in column order (4-bit low parts two per byte, then the 5th bit
// one per bit, or the 5th/6th bits two per element) followed by one 8-byte
// scale record per row:
//   Q8_0        f16 d[2]                      (two 32-column blocks)
//   Q4_K, Q5_K  f16 d, f16 dmin, u8 sc[2], u8 m[2] (the chunk's 2 sub-blocks)
//   Q6_K        f16 d, i8 sc[4], 2 zero bytes  (the chunk's 4 sub-blocks)
// Every packet is 16-byte aligned and 128 x (code bytes + 8) long, so a
// producer reads one contiguous, aligned span per (row tile, 64 columns).  The
// layout is lossless; packets_to_gguf rebuilds the GGUF rows byte for byte.
//
// packets_to_f16 expands packets into the f16 tensor-core operand
// f16(w) with w computed in f32 exactly as gguf-py dequantizes:
//   Q8_0: q * d;  Q4_K/Q5_K: (d*sc) * q - (dmin*m);  Q6_K: (d*sc) * (q - 32).
#include "packets.cuh"
#include "samq_internal.hpp"

namespace samq {

int64_t packet_code_bytes(int type) {
    switch (type) {
        case SAMQ_TYPE_Q8_0: return 64;
        case SAMQ_TYPE_Q4_K: return 32;
        case SAMQ_TYPE_Q5_K: return 40;
        case SAMQ_TYPE_Q6_K: return 48;
        default: return -1;
    }
}

int64_t packet_bytes(int type) {
    const int64_t c = packet_code_bytes(type);
    return c < 0 ? -1 : 128 * (c + 8);
}

int64_t row_bytes(int type, int64_t k) {
    int64_t be, bb;
    switch (type) {
        case SAMQ_TYPE_Q8_0: be = 32; bb = 34; break;
        case SAMQ_TYPE_Q4_K: be = 256; bb = 144; break;
        case SAMQ_TYPE_Q5_K: be = 256; bb = 176; break;
        case SAMQ_TYPE_Q6_K: be = 256; bb = 210; break;
        default: return -1;
    }
    if (k <= 0 || k % be) return -1;
    return k / be * bb;
}

namespace {

__device__ __forceinline__ void kquant_scale_min(const uint8_t* s, int j, int& sc, int& m) {
    // 6-bit scale/min j of the 12-byte field (gguf-py Q4_K.get_scale_min).
    if (j < 4) {
        sc = s[j] & 63;
        m = s[4 + j] & 63;
    } else {
        sc = (s[8 + j - 4] & 15) | ((s[j - 4] >> 2) & 0x30);
        m = (s[8 + j - 4] >> 4) | ((s[j] >> 2) & 0x30);
    }
}

// 6-bit code of element e (0..255) of a K-quant super-block, as stored.
__device__ __forceinline__ uint32_t kquant_code(int type, const uint8_t* o, int e) {
    if (type == SAMQ_TYPE_Q6_K) {
        const int h = e >> 7, i = e & 127;
        const uint32_t lo = i < 64 ? (o[64 * h + i] & 15u) : (o[64 * h + i - 64] >> 4);
        const uint32_t hi = (o[128 + 32 * h + (i & 31)] >> (2 * (i >> 5))) & 3u;
        return lo | (hi << 4);
    }
    const uint8_t* qs = type == SAMQ_TYPE_Q5_K ? o + 48 : o + 16;
    const int p = e >> 6, l = e & 63;
    uint32_t q = l < 32 ? (qs[32 * p + l] & 15u) : (qs[32 * p + l - 32] >> 4);
    if (type == SAMQ_TYPE_Q5_K) q |= ((o[16 + (e & 31)] >> (e >> 5)) & 1u) << 4;
    return q;
}

__device__ __forceinline__ bool half_finite(uint16_t h) { return (h & 0x7c00u) != 0x7c00u; }

__global__ void gguf_to_packets_kernel(int type, int64_t k, int64_t n, const uint8_t* __restrict__ rows,
                                       uint8_t* __restrict__ packets, uint32_t* bad_scales) {
    const int64_t chunks = (k + 63) / 64;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= n * chunks) return;
    const int64_t r = idx / chunks, c = idx % chunks;
    const int cb = code_bytes_of(type);
    const int64_t rb = k / (type == SAMQ_TYPE_Q8_0 ? 32 : 256) * block_bytes_of(type);
    uint8_t* packet = packets + ((r / 128) * chunks + c) * static_cast<int64_t>(128 * (cb + 8));
    uint8_t code[64];
    uint8_t rec[8];
#pragma unroll
    for (int i = 0; i < 64; ++i) code[i] = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) rec[i] = 0;
    const uint8_t* row = rows + r * rb;
    bool bad = false;
    if (type == SAMQ_TYPE_Q8_0) {
        for (int s = 0; s < 2; ++s) {
            const int64_t blk = 2 * c + s;
            if (blk * 32 >= k) break;
            const uint8_t* o = row + blk * 34;
            rec[2 * s] = o[0];
            rec[2 * s + 1] = o[1];
            bad |= !half_finite(static_cast<uint16_t>(o[0] | (o[1] << 8)));
            for (int i = 0; i < 32; ++i) code[32 * s + i] = o[2 + i];
        }
    } else {
        const int64_t sb = c / 4;
        const int part = static_cast<int>(c % 4);
        const uint8_t* o = row + sb * block_bytes_of(type);
        for (int i = 0; i < 64; ++i) {
            const uint32_t q = kquant_code(type, o, 64 * part + i);
            code[i / 2] |= static_cast<uint8_t>((q & 15u) << (4 * (i & 1)));
            if (type == SAMQ_TYPE_Q5_K) code[32 + i / 8] |= static_cast<uint8_t>(((q >> 4) & 1u) << (i & 7));
            if (type == SAMQ_TYPE_Q6_K) code[32 + i / 4] |= static_cast<uint8_t>(((q >> 4) & 3u) << (2 * (i & 3)));
        }
        if (type == SAMQ_TYPE_Q6_K) {
            rec[0] = o[208];
            rec[1] = o[209];
            bad |= !half_finite(static_cast<uint16_t>(o[208] | (o[209] << 8)));
            for (int i = 0; i < 4; ++i) rec[2 + i] = o[192 + 4 * part + i];
        } else {
            for (int i = 0; i < 4; ++i) rec[i] = o[i];
            bad |= !half_finite(static_cast<uint16_t>(o[0] | (o[1] << 8)));
            bad |= !half_finite(static_cast<uint16_t>(o[2] | (o[3] << 8)));
            int sc, m;
            kquant_scale_min(o + 4, 2 * part, sc, m);
            rec[4] = static_cast<uint8_t>(sc);
            rec[6] = static_cast<uint8_t>(m);
            kquant_scale_min(o + 4, 2 * part + 1, sc, m);
            rec[5] = static_cast<uint8_t>(sc);
            rec[7] = static_cast<uint8_t>(m);
        }
    }
    uint8_t* dst = packet + (r % 128) * cb;
    for (int i = 0; i < cb; ++i) dst[i] = code[i];
    uint8_t* rdst = packet + 128 * cb + (r % 128) * 8;
    for (int i = 0; i < 8; ++i) rdst[i] = rec[i];
    if (bad && bad_scales) atomicAdd(bad_scales, 1u);
}

__global__ void packets_to_gguf_kernel(int type, int64_t k, int64_t n, const uint8_t* __restrict__ packets,
                                       uint8_t* __restrict__ rows) {
    const int be = type == SAMQ_TYPE_Q8_0 ? 32 : 256;
    const int64_t blocks = k / be, chunks = (k + 63) / 64;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= n * blocks) return;
    const int64_t r = idx / blocks, b = idx % blocks;
    const int cb = code_bytes_of(type), bb = block_bytes_of(type);
    uint8_t* o = rows + r * blocks * bb + b * bb;
    const int64_t pbytes = static_cast<int64_t>(128 * (cb + 8));
    if (type == SAMQ_TYPE_Q8_0) {
        const int64_t c = b / 2;
        const int s = static_cast<int>(b % 2);
        const uint8_t* packet = packets + ((r / 128) * chunks + c) * pbytes;
        const uint8_t* code = packet + (r % 128) * cb;
        const uint8_t* rec = packet + 128 * cb + (r % 128) * 8;
        o[0] = rec[2 * s];
        o[1] = rec[2 * s + 1];
        for (int i = 0; i < 32; ++i) o[2 + i] = code[32 * s + i];
        return;
    }
    for (int i = 0; i < bb; ++i) o[i] = 0;
    int sc[8], mn[8];
    for (int part = 0; part < 4; ++part) {
        const int64_t c = 4 * b + part;
        const uint8_t* packet = packets + ((r / 128) * chunks + c) * pbytes;
        const uint8_t* code = packet + (r % 128) * cb;
        const uint8_t* rec = packet + 128 * cb + (r % 128) * 8;
        for (int i = 0; i < 64; ++i) {
            uint32_t q = (code[i / 2] >> (4 * (i & 1))) & 15u;
            if (type == SAMQ_TYPE_Q5_K) q |= ((code[32 + i / 8] >> (i & 7)) & 1u) << 4;
            if (type == SAMQ_TYPE_Q6_K) q |= ((code[32 + i / 4] >> (2 * (i & 3))) & 3u) << 4;
            const int e = 64 * part + i;
            if (type == SAMQ_TYPE_Q6_K) {
                const int h = e >> 7, j = e & 127;
                if (j < 64) o[64 * h + j] |= static_cast<uint8_t>(q & 15u);
                else o[64 * h + j - 64] |= static_cast<uint8_t>((q & 15u) << 4);
                o[128 + 32 * h + (j & 31)] |= static_cast<uint8_t>(((q >> 4) & 3u) << (2 * (j >> 5)));
            } else {
                uint8_t* qs = type == SAMQ_TYPE_Q5_K ? o + 48 : o + 16;
                const int p = e >> 6, l = e & 63;
                if (l < 32) qs[32 * p + l] |= static_cast<uint8_t>(q & 15u);
                else qs[32 * p + l - 32] |= static_cast<uint8_t>((q & 15u) << 4);
                if (type == SAMQ_TYPE_Q5_K && (q & 16u)) o[16 + (e & 31)] |= static_cast<uint8_t>(1u << (e >> 5));
            }
        }
        if (type == SAMQ_TYPE_Q6_K) {
            o[208] = rec[0];
            o[209] = rec[1];
            for (int i = 0; i < 4; ++i) o[192 + 4 * part + i] = rec[2 + i];
        } else {
            for (int i = 0; i < 4; ++i) o[i] = rec[i];
            sc[2 * part] = rec[4];
            sc[2 * part + 1] = rec[5];
            mn[2 * part] = rec[6];
            mn[2 * part + 1] = rec[7];
        }
    }
    if (type != SAMQ_TYPE_Q6_K) {
        uint8_t* s = o + 4;
        for (int i = 0; i < 4; ++i) {
            s[i] = static_cast<uint8_t>((sc[i] & 63) | ((sc[i + 4] >> 4) << 6));
            s[4 + i] = static_cast<uint8_t>((mn[i] & 63) | ((mn[i + 4] >> 4) << 6));
            s[8 + i] = static_cast<uint8_t>((sc[i + 4] & 15) | ((mn[i + 4] & 15) << 4));
        }
    }
}

// The f16 B operand of K2: every weight decoded (decode8) and rounded once.
template <int TYPE>
__global__ void __launch_bounds__(256) packets_to_f16_kernel(int64_t k, int64_t n,
                                                             const uint8_t* __restrict__ packets,
                                                             __half* __restrict__ out) {
    const int64_t per_row = k / 8, chunks = (k + 63) / 64;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= n * per_row) return;
    const int64_t r = idx / per_row, c8 = idx % per_row;
    constexpr int cb = code_bytes_of(TYPE);
    const uint8_t* packet = packets + ((r / 128) * chunks + c8 / 8) * static_cast<int64_t>(128 * (cb + 8));
    float w[8];
    decode8<TYPE>(packet + (r % 128) * cb, packet + 128 * cb + (r % 128) * 8, static_cast<int>(c8 & 7), w);
    __align__(16) __half h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = __float2half_rn(w[i]);
    *reinterpret_cast<uint4*>(out + r * k + c8 * 8) = *reinterpret_cast<const uint4*>(h);
}

unsigned grid_for(int64_t threads) { return static_cast<unsigned>((threads + 255) / 256); }

}  // namespace

void launch_gguf_to_packets(int type, int64_t k, int64_t n, const uint8_t* rows, uint8_t* packets,
                            uint32_t* bad_scales, cudaStream_t stream) {
    const int64_t chunks = (k + 63) / 64;
    gguf_to_packets_kernel<<<grid_for(n * chunks), 256, 0, stream>>>(type, k, n, rows, packets, bad_scales);
    check_cuda(cudaGetLastError(), "gguf_to_packets_kernel launch");
}

void launch_packets_to_gguf(int type, int64_t k, int64_t n, const uint8_t* packets, uint8_t* rows,
                            cudaStream_t stream) {
    const int64_t blocks = k / (type == SAMQ_TYPE_Q8_0 ? 32 : 256);
    packets_to_gguf_kernel<<<grid_for(n * blocks), 256, 0, stream>>>(type, k, n, packets, rows);
    check_cuda(cudaGetLastError(), "packets_to_gguf_kernel launch");
}

void launch_packets_to_f16(int type, int64_t k, int64_t n, const uint8_t* packets, __half* out,
                           cudaStream_t stream) {
    const unsigned grid = grid_for(n * (k / 8));
    switch (type) {
        case SAMQ_TYPE_Q8_0: packets_to_f16_kernel<SAMQ_TYPE_Q8_0><<<grid, 256, 0, stream>>>(k, n, packets, out); break;
        case SAMQ_TYPE_Q4_K: packets_to_f16_kernel<SAMQ_TYPE_Q4_K><<<grid, 256, 0, stream>>>(k, n, packets, out); break;
        case SAMQ_TYPE_Q5_K: packets_to_f16_kernel<SAMQ_TYPE_Q5_K><<<grid, 256, 0, stream>>>(k, n, packets, out); break;
        case SAMQ_TYPE_Q6_K: packets_to_f16_kernel<SAMQ_TYPE_Q6_K><<<grid, 256, 0, stream>>>(k, n, packets, out); break;
        default: fail(SAMQ_ERR_INVALID_ARGUMENT, "unsupported weight type");
    }
    check_cuda(cudaGetLastError(), "packets_to_f16_kernel launch");
}

}  // namespace samq
