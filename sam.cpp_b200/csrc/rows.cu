// rows.cu -- host-side GGUF row quantizer: f32 rows -> packed Q8_0 / Q4_K /
// Q5_K / Q6_K rows in the GGUF block layouts, the role of the reference's
// tools/quantize/quantize_rows.cpp:210 (ggml_quantize_chunk).  Used to write
// synthetic models and to quantize weights a caller holds in f32.
//
// Q8_0 follows the reference converter's quantizer (gguf-py, used by
// tools/convert/sam3_gguf.py:319-324): d = amax / 127 in f32, codes
// round-half-away(x * (1 / d)), d stored as f16.  The K-quants use a plain
// min / max encoder per 32- (Q4_K, Q5_K) or 16-element (Q6_K) sub-block, not
// GGML's iterative make_qkx search: any valid encoding is a valid weight, and
// the device path's results are defined on the decoded values.
#include <cmath>
#include <cstring>

#include <cuda_fp16.h>

#include "samq_internal.hpp"

namespace samq {
namespace {

uint16_t f16_bits(float v) {
    const __half h = __float2half_rn(v);
    uint16_t bits;
    std::memcpy(&bits, &h, 2);
    return bits;
}

float f16_value(uint16_t bits) {
    __half_raw raw;
    raw.x = bits;
    return __half2float(__half(raw));
}

void put16(uint8_t* p, uint16_t v) {
    p[0] = static_cast<uint8_t>(v & 0xff);
    p[1] = static_cast<uint8_t>(v >> 8);
}

int clamp_int(long v, int lo, int hi) { return static_cast<int>(v < lo ? lo : (v > hi ? hi : v)); }

void q8_0_block(const float* x, uint8_t* out) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = std::fmax(amax, std::fabs(x[i]));
    const float d = amax / 127.0f;
    const float inv = d == 0.0f ? 0.0f : 1.0f / d;
    put16(out, f16_bits(d));
    for (int i = 0; i < 32; ++i) out[2 + i] = static_cast<uint8_t>(static_cast<int8_t>(std::round(x[i] * inv)));
}

// Q4_K / Q5_K super-block: f16 d, f16 dmin, 12 bytes of 6-bit (scale, min)
// pairs for the eight 32-element sub-blocks, [Q5_K: 32 bytes of fifth bits],
// 128 bytes of 4-bit codes (sub-blocks 2p and 2p + 1 share byte row p, low
// and high nibble).  Value = d * sc * q - dmin * m.
void q45_k_block(const float* x, uint8_t* out, bool five) {
    const int qmax = five ? 31 : 15;
    float step[8], floor_[8], max_step = 0.0f, max_floor = 0.0f;
    for (int s = 0; s < 8; ++s) {
        float lo = 0.0f, hi = 0.0f;  // the minimum is clamped to <= 0 (m >= 0)
        for (int i = 0; i < 32; ++i) {
            lo = std::fmin(lo, x[32 * s + i]);
            hi = std::fmax(hi, x[32 * s + i]);
        }
        step[s] = (hi - lo) / static_cast<float>(qmax);
        floor_[s] = -lo;
        max_step = std::fmax(max_step, step[s]);
        max_floor = std::fmax(max_floor, floor_[s]);
    }
    const uint16_t d_bits = f16_bits(max_step / 63.0f), m_bits = f16_bits(max_floor / 63.0f);
    const float d = f16_value(d_bits), dmin = f16_value(m_bits);
    int sc[8], mn[8];
    for (int s = 0; s < 8; ++s) {
        sc[s] = d > 0.0f ? clamp_int(std::lround(step[s] / d), 0, 63) : 0;
        mn[s] = dmin > 0.0f ? clamp_int(std::lround(floor_[s] / dmin), 0, 63) : 0;
    }
    put16(out, d_bits);
    put16(out + 2, m_bits);
    uint8_t* packed = out + 4;
    for (int i = 0; i < 4; ++i) {
        packed[i] = static_cast<uint8_t>((sc[i] & 63) | ((sc[i + 4] >> 4) << 6));
        packed[4 + i] = static_cast<uint8_t>((mn[i] & 63) | ((mn[i + 4] >> 4) << 6));
        packed[8 + i] = static_cast<uint8_t>((sc[i + 4] & 15) | ((mn[i + 4] & 15) << 4));
    }
    uint8_t code[256];
    for (int s = 0; s < 8; ++s) {
        const float scale = d * static_cast<float>(sc[s]), offset = dmin * static_cast<float>(mn[s]);
        for (int i = 0; i < 32; ++i)
            code[32 * s + i] = static_cast<uint8_t>(
                scale > 0.0f ? clamp_int(std::lround((x[32 * s + i] + offset) / scale), 0, qmax) : 0);
    }
    uint8_t* high = out + 16;
    uint8_t* low = five ? out + 48 : out + 16;
    if (five) std::memset(high, 0, 32);
    for (int p = 0; p < 4; ++p)
        for (int l = 0; l < 32; ++l)
            low[32 * p + l] = static_cast<uint8_t>((code[64 * p + l] & 15) | ((code[64 * p + 32 + l] & 15) << 4));
    if (five)
        for (int e = 0; e < 256; ++e)
            if (code[e] & 16) high[e % 32] |= static_cast<uint8_t>(1u << (e / 32));
}

// Q6_K super-block: 128 bytes of low nibbles, 64 bytes of 2-bit high parts,
// 16 int8 sub-block scales, f16 d at the end.  Value = d * sc * (q - 32).
void q6_k_block(const float* x, uint8_t* out) {
    float step[16], max_step = 0.0f;
    for (int s = 0; s < 16; ++s) {
        float amax = 0.0f;
        for (int i = 0; i < 16; ++i) amax = std::fmax(amax, std::fabs(x[16 * s + i]));
        step[s] = amax / 31.0f;
        max_step = std::fmax(max_step, step[s]);
    }
    const uint16_t d_bits = f16_bits(max_step / 127.0f);
    const float d = f16_value(d_bits);
    int8_t sc[16];
    for (int s = 0; s < 16; ++s) sc[s] = static_cast<int8_t>(d > 0.0f ? clamp_int(std::lround(step[s] / d), -128, 127) : 0);
    std::memset(out, 0, 192);
    for (int e = 0; e < 256; ++e) {
        const float scale = d * static_cast<float>(sc[e / 16]);
        const int v = scale != 0.0f ? clamp_int(std::lround(x[e] / scale), -32, 31) : 0;
        const uint8_t q = static_cast<uint8_t>(v + 32);
        const int half = e / 128, i = e % 128;
        if (i < 64)
            out[64 * half + i] |= static_cast<uint8_t>(q & 15);
        else
            out[64 * half + i - 64] |= static_cast<uint8_t>((q & 15) << 4);
        out[128 + 32 * half + (i % 32)] |= static_cast<uint8_t>(((q >> 4) & 3) << (2 * (i / 32)));
    }
    std::memcpy(out + 192, sc, 16);
    put16(out + 208, d_bits);
}

}  // namespace

// n rows of k f32 values -> n packed rows of row_bytes(type, k) bytes (the
// caller has checked type, k and the sizes).
void quantize_rows(int type, int64_t k, int64_t n, const float* src, uint8_t* out) {
    const int64_t rb = row_bytes(type, k);
    const int64_t block = type == SAMQ_TYPE_Q8_0 ? 32 : 256;
    const int64_t block_bytes = rb / (k / block);
    for (int64_t r = 0; r < n; ++r)
        for (int64_t b = 0; b < k / block; ++b) {
            const float* x = src + r * k + b * block;
            for (int64_t i = 0; i < block; ++i)
                if (!std::isfinite(x[i])) fail(SAMQ_ERR_INVALID_ARGUMENT, "non-finite weight");
            uint8_t* o = out + r * rb + b * block_bytes;
            switch (type) {
                case SAMQ_TYPE_Q8_0: q8_0_block(x, o); break;
                case SAMQ_TYPE_Q4_K: q45_k_block(x, o, false); break;
                case SAMQ_TYPE_Q5_K: q45_k_block(x, o, true); break;
                default: q6_k_block(x, o); break;
            }
        }
}

}  // namespace samq
