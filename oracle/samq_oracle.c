/*
 * samq_oracle.c -- CPU restatement of SAM.cpp's quantized-linear path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline); the
 * product library never links or calls it.  See samq_oracle.h for what each
 * function restates and which reference file/line it follows.
 *
 * Compiled with -ffp-contract=off so that every f32 expression rounds exactly
 * as written (the bit-exact comparisons depend on it).
 */
#include "samq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#if defined(__x86_64__) && defined(__GNUC__)
#include <immintrin.h>
#define ORACLE_X86 1
#endif

/* ------------------------------------------------------------------ f16 */

uint16_t oracle_f32_to_f16(float value) {
    uint32_t x;
    memcpy(&x, &value, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t a = x & 0x7fffffffu;
    if (a >= 0x7f800000u) return (uint16_t)(sign | (a > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
    if (a < 0x38800000u) {                                   /* half subnormal or zero */
        float v;
        memcpy(&v, &a, 4);
        const float scaled = v * 16777216.0f;                /* exact: power of two */
        const uint32_t mant = (uint32_t)rintf(scaled);       /* ties to even */
        return (uint16_t)(sign | mant);
    }
    const uint32_t exponent = (a >> 23) - 127u + 15u;
    const uint32_t mant = a & 0x7fffffu;
    uint32_t h = (exponent << 10) | (mant >> 13);
    const uint32_t rest = mant & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

float oracle_f16_to_f32(uint16_t bits) {
    const uint32_t sign = ((uint32_t)bits & 0x8000u) << 16;
    const uint32_t exponent = (bits >> 10) & 0x1fu;
    const uint32_t mant = bits & 0x3ffu;
    uint32_t out;
    if (exponent == 0) {
        if (mant == 0) {
            out = sign;
        } else {
            const float v = (float)mant * (1.0f / 16777216.0f);
            memcpy(&out, &v, 4);
            out |= sign;
        }
    } else if (exponent == 31) {
        out = sign | 0x7f800000u | (mant << 13);
    } else {
        out = sign | ((exponent - 15u + 127u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &out, 4);
    return f;
}

static inline uint16_t load_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline void store_u16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

/* --------------------------------------------------------------- sizes */

int64_t oracle_block_elements(int type) {
    switch (type) {
        case ORACLE_TYPE_Q8_0: case ORACLE_TYPE_Q8_1: return 32;
        case ORACLE_TYPE_Q4_K: case ORACLE_TYPE_Q5_K: case ORACLE_TYPE_Q6_K: case ORACLE_TYPE_Q8_K: return 256;
        default: return -1;
    }
}

int64_t oracle_block_bytes(int type) {
    switch (type) {
        case ORACLE_TYPE_Q8_0: return 34;
        case ORACLE_TYPE_Q8_1: return 36;   /* GGML CUDA block_q8_1 (cuda_q8_rhs_probe.cu:16,91) */
        case ORACLE_TYPE_Q4_K: return 144;
        case ORACLE_TYPE_Q5_K: return 176;
        case ORACLE_TYPE_Q6_K: return 210;
        case ORACLE_TYPE_Q8_K: return 4 + 256 + 32; /* cpu_quantized_matmul.hpp:26-42 */
        default: return -1;
    }
}

int64_t oracle_row_bytes(int type, int64_t k) {
    const int64_t be = oracle_block_elements(type);
    if (be <= 0 || k <= 0 || k % be) return -1;
    return k / be * oracle_block_bytes(type);
}

/* ------------------------------------------------ Q8_0 (gguf-py, exact) */

int oracle_quantize_q8_0(const float* x, int64_t n, uint8_t* out) {
    if (n % 32) return -1;
    for (int64_t b = 0; b < n / 32; ++b) {
        const float* v = x + b * 32;
        uint8_t* o = out + b * 34;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) { const float a = fabsf(v[i]); if (a > amax) amax = a; }
        const float d = amax / 127.0f;
        const float id = d == 0.0f ? 0.0f : 1.0f / d;
        store_u16(o, oracle_f32_to_f16(d));
        for (int i = 0; i < 32; ++i) {
            const float q = roundf(v[i] * id);   /* np_roundf: half away from zero */
            o[2 + i] = (uint8_t)(int8_t)q;
        }
    }
    return 0;
}

/* ----------------------------------------------- own K-quant packer */

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

static void pack_kquant_scales(const int sc[8], const int m[8], uint8_t s[12]) {
    /* Inverse of gguf-py Q4_K.get_scale_min (gguf/quants.py). */
    for (int i = 0; i < 4; ++i) {
        s[i] = (uint8_t)((sc[i] & 63) | ((sc[i + 4] >> 4) << 6));
        s[4 + i] = (uint8_t)((m[i] & 63) | ((m[i + 4] >> 4) << 6));
        s[8 + i] = (uint8_t)((sc[i + 4] & 15) | ((m[i + 4] & 15) << 4));
    }
}

static void unpack_kquant_scales(const uint8_t s[12], int sc[8], int m[8]) {
    for (int i = 0; i < 4; ++i) {
        sc[i] = s[i] & 63;
        m[i] = s[4 + i] & 63;
        sc[4 + i] = (s[8 + i] & 15) | ((s[i] >> 2) & 0x30);
        m[4 + i] = (s[8 + i] >> 4) | ((s[4 + i] >> 2) & 0x30);
    }
}

static void quantize_q45k_block(const float* x, uint8_t* o, int five_bit) {
    const int qmax = five_bit ? 31 : 15;
    float lo[8], scale[8];
    float dmax = 0.0f, mmax = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float mn = 0.0f, mx = 0.0f;
        for (int i = 0; i < 32; ++i) {
            const float v = x[32 * j + i];
            if (v < mn) mn = v;
            if (v > mx) mx = v;
        }
        lo[j] = mn;
        scale[j] = (mx - mn) / (float)qmax;
        if (scale[j] > dmax) dmax = scale[j];
        if (-mn > mmax) mmax = -mn;
    }
    const uint16_t d16 = oracle_f32_to_f16(dmax / 63.0f);
    const uint16_t dm16 = oracle_f32_to_f16(mmax / 63.0f);
    const float d = oracle_f16_to_f32(d16), dmin = oracle_f16_to_f32(dm16);
    int sc[8], m[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = d > 0.0f ? clampi((int)lrintf(scale[j] / d), 0, 63) : 0;
        m[j] = dmin > 0.0f ? clampi((int)lrintf(-lo[j] / dmin), 0, 63) : 0;
    }
    store_u16(o, d16);
    store_u16(o + 2, dm16);
    pack_kquant_scales(sc, m, o + 4);
    uint8_t q[256];
    for (int j = 0; j < 8; ++j) {
        const float s = d * (float)sc[j];
        const float off = dmin * (float)m[j];
        for (int i = 0; i < 32; ++i)
            q[32 * j + i] = (uint8_t)(s > 0.0f ? clampi((int)lrintf((x[32 * j + i] + off) / s), 0, qmax) : 0);
    }
    uint8_t* qh = o + 16;
    uint8_t* qs = five_bit ? o + 48 : o + 16;
    if (five_bit) memset(qh, 0, 32);
    for (int p = 0; p < 4; ++p)
        for (int l = 0; l < 32; ++l)
            qs[32 * p + l] = (uint8_t)((q[64 * p + l] & 15) | ((q[64 * p + 32 + l] & 15) << 4));
    if (five_bit)
        for (int e = 0; e < 256; ++e)
            if (q[e] & 16) qh[e % 32] |= (uint8_t)(1u << (e / 32));
}

static void quantize_q6k_block(const float* x, uint8_t* o) {
    float scale[16];
    float smax = 0.0f;
    for (int j = 0; j < 16; ++j) {
        float amax = 0.0f;
        for (int i = 0; i < 16; ++i) { const float a = fabsf(x[16 * j + i]); if (a > amax) amax = a; }
        scale[j] = amax / 31.0f;
        if (scale[j] > smax) smax = scale[j];
    }
    const uint16_t d16 = oracle_f32_to_f16(smax / 127.0f);
    const float d = oracle_f16_to_f32(d16);
    int8_t sc[16];
    for (int j = 0; j < 16; ++j) sc[j] = (int8_t)(d > 0.0f ? clampi((int)lrintf(scale[j] / d), -128, 127) : 0);
    uint8_t q[256];
    for (int e = 0; e < 256; ++e) {
        const float s = d * (float)sc[e / 16];
        const int v = s != 0.0f ? clampi((int)lrintf(x[e] / s), -32, 31) : 0;
        q[e] = (uint8_t)(v + 32);
    }
    uint8_t* ql = o;
    uint8_t* qh = o + 128;
    memset(ql, 0, 128);
    memset(qh, 0, 64);
    for (int e = 0; e < 256; ++e) {
        const int h = e / 128, i = e % 128;
        if (i < 64) ql[64 * h + i] |= (uint8_t)(q[e] & 15);
        else ql[64 * h + i - 64] |= (uint8_t)((q[e] & 15) << 4);
        qh[32 * h + (i % 32)] |= (uint8_t)(((q[e] >> 4) & 3) << (2 * (i / 32)));
    }
    memcpy(o + 192, sc, 16);
    store_u16(o + 208, d16);
}

int oracle_quantize_kquant(int type, const float* x, int64_t n, uint8_t* out) {
    if (n % 256) return -1;
    for (int64_t b = 0; b < n / 256; ++b) {
        switch (type) {
            case ORACLE_TYPE_Q4_K: quantize_q45k_block(x + 256 * b, out + 144 * b, 0); break;
            case ORACLE_TYPE_Q5_K: quantize_q45k_block(x + 256 * b, out + 176 * b, 1); break;
            case ORACLE_TYPE_Q6_K: quantize_q6k_block(x + 256 * b, out + 210 * b); break;
            default: return -1;
        }
    }
    return 0;
}

/* ---------------------------------------- dequantizers (gguf-py, exact) */

/* 6-bit codes of one super-block (values stored as they appear in GGUF). */
static void decode_codes(int type, const uint8_t* o, uint8_t q[256]) {
    if (type == ORACLE_TYPE_Q4_K || type == ORACLE_TYPE_Q5_K) {
        const uint8_t* qs = type == ORACLE_TYPE_Q5_K ? o + 48 : o + 16;
        for (int p = 0; p < 4; ++p)
            for (int l = 0; l < 32; ++l) {
                q[64 * p + l] = qs[32 * p + l] & 15;
                q[64 * p + 32 + l] = qs[32 * p + l] >> 4;
            }
        if (type == ORACLE_TYPE_Q5_K)
            for (int e = 0; e < 256; ++e) q[e] |= (uint8_t)(((o[16 + e % 32] >> (e / 32)) & 1) << 4);
    } else { /* Q6_K */
        for (int e = 0; e < 256; ++e) {
            const int h = e / 128, i = e % 128;
            const uint8_t lo = i < 64 ? (o[64 * h + i] & 15) : (o[64 * h + i - 64] >> 4);
            const uint8_t hi = (o[128 + 32 * h + (i % 32)] >> (2 * (i / 32))) & 3;
            q[e] = (uint8_t)(lo | (hi << 4));
        }
    }
}

int oracle_dequantize(int type, const uint8_t* blocks, int64_t n, float* out) {
    const int64_t be = oracle_block_elements(type), bb = oracle_block_bytes(type);
    if (be <= 0 || n % be || type == ORACLE_TYPE_Q8_1 || type == ORACLE_TYPE_Q8_K) return -1;
    for (int64_t b = 0; b < n / be; ++b) {
        const uint8_t* o = blocks + b * bb;
        float* y = out + b * be;
        if (type == ORACLE_TYPE_Q8_0) {
            const float d = oracle_f16_to_f32(load_u16(o));
            for (int i = 0; i < 32; ++i) y[i] = (float)(int8_t)o[2 + i] * d;
            continue;
        }
        uint8_t q[256];
        decode_codes(type, o, q);
        if (type == ORACLE_TYPE_Q6_K) {
            const float d = oracle_f16_to_f32(load_u16(o + 208));
            for (int e = 0; e < 256; ++e) {
                const float ds = d * (float)(int8_t)o[192 + e / 16];
                y[e] = ds * (float)((int)q[e] - 32);
            }
        } else {
            const float d = oracle_f16_to_f32(load_u16(o));
            const float dmin = oracle_f16_to_f32(load_u16(o + 2));
            int sc[8], m[8];
            unpack_kquant_scales(o + 4, sc, m);
            for (int e = 0; e < 256; ++e) {
                const float ds = d * (float)sc[e / 32];
                const float dm = dmin * (float)m[e / 32];
                y[e] = ds * (float)q[e] - dm;
            }
        }
    }
    return 0;
}

/* ------------------------------------------------- activation staging */

/* f32 sum in the order of a 32-lane xor butterfly (offsets 16, 8, 4, 2, 1),
 * as read on lane 0 (verify_q8_rhs_staging.py:69-76). */
static float butterfly_sum32(const float* v) {
    float r[32], t[32];
    memcpy(r, v, sizeof(r));
    for (int off = 16; off >= 1; off >>= 1) {
        for (int i = 0; i < 32; ++i) t[i] = r[i] + r[i ^ off];
        memcpy(r, t, sizeof(r));
    }
    return r[0];
}

static float block_amax(const float* v, int count) {
    float amax = 0.0f;
    for (int i = 0; i < count; ++i) { const float a = fabsf(v[i]); if (a > amax) amax = a; }
    return amax;
}

int oracle_quantize_q8_1(const float* x, int64_t rows, int64_t k, int64_t ld, uint8_t* out) {
    if (k <= 0 || k % 32 || ld < k || rows < 0) return -1;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b = 0; b < k / 32; ++b) {
            const float* v = x + r * ld + b * 32;
            uint8_t* o = out + (r * (k / 32) + b) * 36;
            const float amax = block_amax(v, 32);
            const float d = amax / 127.0f;
            const float inv = amax == 0.0f ? 0.0f : 127.0f / amax;
            store_u16(o, oracle_f32_to_f16(d));
            store_u16(o + 2, oracle_f32_to_f16(butterfly_sum32(v)));
            for (int i = 0; i < 32; ++i) o[4 + i] = (uint8_t)(int8_t)roundf(v[i] * inv);
        }
    return 0;
}

int64_t oracle_mmq_d4_bytes(int64_t rows, int64_t k) {
    const int64_t padded = (k + 511) / 512 * 512;
    return rows * (padded / 128) * 144;
}

int oracle_quantize_mmq_d4(const float* x, int64_t rows, int64_t k, int64_t ld, uint8_t* out) {
    if (k <= 0 || k % 32 || ld < k || rows < 0) return -1;
    const int64_t padded = (k + 511) / 512 * 512, blocks = padded / 128;
    for (int64_t blk = 0; blk < blocks; ++blk)
        for (int64_t r = 0; r < rows; ++r) {
            uint8_t* o = out + (blk * rows + r) * 144;
            for (int s = 0; s < 4; ++s) {
                float v[32];
                for (int i = 0; i < 32; ++i) {
                    const int64_t col = blk * 128 + s * 32 + i;
                    v[i] = col < k ? x[r * ld + col] : 0.0f;
                }
                const float amax = block_amax(v, 32);
                const float d = amax / 127.0f;
                const float inv = amax == 0.0f ? 0.0f : 127.0f / amax;
                memcpy(o + 4 * s, &d, 4);
                for (int i = 0; i < 32; ++i) o[16 + 32 * s + i] = (uint8_t)(int8_t)roundf(v[i] * inv);
            }
        }
    return 0;
}

int oracle_q8_1_decode(const uint8_t* q8_1, int64_t rows, int64_t k, float* out) {
    if (k % 32) return -1;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b = 0; b < k / 32; ++b) {
            const uint8_t* o = q8_1 + (r * (k / 32) + b) * 36;
            const float d = oracle_f16_to_f32(load_u16(o));
            for (int i = 0; i < 32; ++i) out[r * k + b * 32 + i] = d * (float)(int8_t)o[4 + i];
        }
    return 0;
}

int oracle_act_f16(const float* x, int64_t rows, int64_t k, int64_t ld, uint16_t* out) {
    if (k <= 0 || k % 32 || ld < k) return -1;
    uint8_t blk[36];
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t b = 0; b < k / 32; ++b) {
            if (oracle_quantize_q8_1(x + r * ld + b * 32, 1, 32, 32, blk)) return -1;
            const float d = oracle_f16_to_f32(load_u16(blk));
            for (int i = 0; i < 32; ++i)
                out[r * k + b * 32 + i] = oracle_f32_to_f16(d * (float)(int8_t)blk[4 + i]);
        }
    return 0;
}

int oracle_quantize_q8_k(const float* x, int64_t n, uint8_t* out) {
    if (n % 256) return -1;
    for (int64_t b = 0; b < n / 256; ++b) {
        const float* v = x + 256 * b;
        uint8_t* o = out + 292 * b;
        const float amax = block_amax(v, 256);
        const float d = amax / 127.0f;
        const float inv = amax == 0.0f ? 0.0f : 127.0f / amax;
        memcpy(o, &d, 4);
        int8_t* q = (int8_t*)(o + 4);
        for (int i = 0; i < 256; ++i) q[i] = (int8_t)roundf(v[i] * inv);
        for (int j = 0; j < 16; ++j) {
            int s = 0;
            for (int i = 0; i < 16; ++i) s += q[16 * j + i];
            const int16_t s16 = (int16_t)s;
            memcpy(o + 260 + 2 * j, &s16, 2);
        }
    }
    return 0;
}

/* ------------------------------------------------------- packet layout */

int64_t oracle_packet_code_bytes(int type) {
    switch (type) {
        case ORACLE_TYPE_Q8_0: return 64;
        case ORACLE_TYPE_Q4_K: return 32;
        case ORACLE_TYPE_Q5_K: return 40;
        case ORACLE_TYPE_Q6_K: return 48;
        default: return -1;
    }
}

int64_t oracle_packet_bytes(int type) {
    const int64_t c = oracle_packet_code_bytes(type);
    return c < 0 ? -1 : 128 * (c + 8);
}

static int64_t chunks_of(int64_t k) { return (k + 63) / 64; }

int64_t oracle_packets_size(int type, int64_t k, int64_t n) {
    if (oracle_row_bytes(type, k) < 0 || n <= 0) return -1;
    return (n + 127) / 128 * chunks_of(k) * oracle_packet_bytes(type);
}

/* Codes of 64 columns (chunk c) of one GGUF row, as stored in a packet. */
static void row_chunk_to_packet(int type, const uint8_t* row, int64_t k, int64_t c,
                                uint8_t* code, uint8_t* rec) {
    const int64_t cb = oracle_packet_code_bytes(type);
    memset(code, 0, (size_t)cb);
    memset(rec, 0, 8);
    if (type == ORACLE_TYPE_Q8_0) {
        for (int s = 0; s < 2; ++s) {
            const int64_t blk = 2 * c + s;
            if (blk * 32 >= k) break;
            const uint8_t* o = row + blk * 34;
            memcpy(rec + 2 * s, o, 2);
            memcpy(code + 32 * s, o + 2, 32);
        }
        return;
    }
    const int64_t sb = c / 4, part = c % 4;   /* super-block, quarter of it */
    const uint8_t* o = row + sb * oracle_block_bytes(type);
    uint8_t q[256];
    decode_codes(type, o, q);
    const uint8_t* qc = q + 64 * part;
    for (int i = 0; i < 32; ++i) code[i] = (uint8_t)((qc[2 * i] & 15) | ((qc[2 * i + 1] & 15) << 4));
    if (type == ORACLE_TYPE_Q5_K) {
        for (int i = 0; i < 64; ++i) code[32 + i / 8] |= (uint8_t)(((qc[i] >> 4) & 1) << (i % 8));
    } else if (type == ORACLE_TYPE_Q6_K) {
        for (int i = 0; i < 64; ++i) code[32 + i / 4] |= (uint8_t)(((qc[i] >> 4) & 3) << (2 * (i % 4)));
    }
    if (type == ORACLE_TYPE_Q6_K) {
        memcpy(rec, o + 208, 2);
        memcpy(rec + 2, o + 192 + 4 * part, 4);
    } else {
        int sc[8], m[8];
        unpack_kquant_scales(o + 4, sc, m);
        memcpy(rec, o, 4);                 /* d, dmin */
        rec[4] = (uint8_t)sc[2 * part];
        rec[5] = (uint8_t)sc[2 * part + 1];
        rec[6] = (uint8_t)m[2 * part];
        rec[7] = (uint8_t)m[2 * part + 1];
    }
}

int oracle_pack_packets(int type, int64_t k, int64_t n, const uint8_t* gguf_rows, uint8_t* packets) {
    const int64_t rb = oracle_row_bytes(type, k);
    const int64_t total = oracle_packets_size(type, k, n);
    if (rb < 0 || total < 0) return -1;
    memset(packets, 0, (size_t)total);
    const int64_t cb = oracle_packet_code_bytes(type), pb = oracle_packet_bytes(type), nc = chunks_of(k);
    for (int64_t r = 0; r < n; ++r)
        for (int64_t c = 0; c < nc; ++c) {
            uint8_t* p = packets + ((r / 128) * nc + c) * pb;
            row_chunk_to_packet(type, gguf_rows + r * rb, k, c, p + (r % 128) * cb, p + 128 * cb + (r % 128) * 8);
        }
    return 0;
}

int oracle_unpack_packets(int type, int64_t k, int64_t n, const uint8_t* packets, uint8_t* gguf_rows) {
    const int64_t rb = oracle_row_bytes(type, k);
    if (rb < 0 || n <= 0) return -1;
    const int64_t cb = oracle_packet_code_bytes(type), pb = oracle_packet_bytes(type), nc = chunks_of(k);
    for (int64_t r = 0; r < n; ++r) {
        uint8_t* row = gguf_rows + r * rb;
        memset(row, 0, (size_t)rb);
        for (int64_t c = 0; c < nc; ++c) {
            const uint8_t* p = packets + ((r / 128) * nc + c) * pb;
            const uint8_t* code = p + (r % 128) * cb;
            const uint8_t* rec = p + 128 * cb + (r % 128) * 8;
            if (type == ORACLE_TYPE_Q8_0) {
                for (int s = 0; s < 2; ++s) {
                    const int64_t blk = 2 * c + s;
                    if (blk * 32 >= k) break;
                    memcpy(row + blk * 34, rec + 2 * s, 2);
                    memcpy(row + blk * 34 + 2, code + 32 * s, 32);
                }
                continue;
            }
            const int64_t sb = c / 4, part = c % 4;
            uint8_t* o = row + sb * oracle_block_bytes(type);
            uint8_t q[64];
            for (int i = 0; i < 64; ++i) q[i] = (uint8_t)((code[i / 2] >> (4 * (i % 2))) & 15);
            if (type == ORACLE_TYPE_Q5_K)
                for (int i = 0; i < 64; ++i) q[i] |= (uint8_t)(((code[32 + i / 8] >> (i % 8)) & 1) << 4);
            if (type == ORACLE_TYPE_Q6_K)
                for (int i = 0; i < 64; ++i) q[i] |= (uint8_t)(((code[32 + i / 4] >> (2 * (i % 4))) & 3) << 4);
            for (int i = 0; i < 64; ++i) {
                const int e = (int)(64 * part + i);
                if (type == ORACLE_TYPE_Q6_K) {
                    const int h = e / 128, j = e % 128;
                    if (j < 64) o[64 * h + j] |= (uint8_t)(q[i] & 15);
                    else o[64 * h + j - 64] |= (uint8_t)((q[i] & 15) << 4);
                    o[128 + 32 * h + (j % 32)] |= (uint8_t)(((q[i] >> 4) & 3) << (2 * (j / 32)));
                } else {
                    uint8_t* qs = type == ORACLE_TYPE_Q5_K ? o + 48 : o + 16;
                    const int p = e / 64, l = e % 64;
                    if (l < 32) qs[32 * p + l] |= (uint8_t)(q[i] & 15);
                    else qs[32 * p + l - 32] |= (uint8_t)((q[i] & 15) << 4);
                    if (type == ORACLE_TYPE_Q5_K && (q[i] & 16)) o[16 + e % 32] |= (uint8_t)(1u << (e / 32));
                }
            }
            if (type == ORACLE_TYPE_Q6_K) {
                memcpy(o + 208, rec, 2);
                memcpy(o + 192 + 4 * part, rec + 2, 4);
            } else {
                memcpy(o, rec, 4);
                /* Scales: rebuild the 12-byte field from the quarter records. */
                int sc[8], m[8];
                unpack_kquant_scales(o + 4, sc, m);
                sc[2 * part] = rec[4];
                sc[2 * part + 1] = rec[5];
                m[2 * part] = rec[6];
                m[2 * part + 1] = rec[7];
                pack_kquant_scales(sc, m, o + 4);
            }
        }
    }
    return 0;
}

int oracle_weight_f16(int type, int64_t k, int64_t n, const uint8_t* gguf_rows, uint16_t* out) {
    const int64_t rb = oracle_row_bytes(type, k);
    if (rb < 0) return -1;
    float* row = (float*)malloc((size_t)k * sizeof(float));
    if (!row) return -1;
    for (int64_t r = 0; r < n; ++r) {
        oracle_dequantize(type, gguf_rows + r * rb, k, row);
        for (int64_t i = 0; i < k; ++i) out[r * k + i] = oracle_f32_to_f16(row[i]);
    }
    free(row);
    return 0;
}

/* ------------------------------------------------------ GEMM references */

static double gelu_erf_f64(double v) { return 0.5 * v * (1.0 + erf(v * 0.70710678118654752440)); }

int oracle_gemm_f64(const float* w, const float* x, int64_t m, int64_t n, int64_t k,
                    const float* bias, int epilogue, float* y, int threads) {
    if (m < 0 || n <= 0 || k <= 0) return -1;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 4) num_threads(threads > 0 ? threads : 1)
#endif
    for (int64_t i = 0; i < m; ++i)
        for (int64_t j = 0; j < n; ++j) {
            double acc = 0.0;
            for (int64_t t = 0; t < k; ++t) acc += (double)w[j * k + t] * (double)x[i * k + t];
            if (bias) acc += bias[j];
            if (epilogue == ORACLE_EPILOGUE_GELU_ERF) acc = gelu_erf_f64(acc);
            y[i * n + j] = (float)acc;
        }
    (void)threads;
    return 0;
}

int oracle_gemm_f16_f64(const uint16_t* w, const uint16_t* x, int64_t m, int64_t n, int64_t k,
                        const float* bias, int epilogue, float* y, int threads) {
    if (m < 0 || n <= 0 || k <= 0) return -1;
    float* wf = (float*)malloc((size_t)(n * k) * sizeof(float));
    float* xf = (float*)malloc((size_t)((m ? m : 1) * k) * sizeof(float));
    if (!wf || !xf) { free(wf); free(xf); return -1; }
    for (int64_t i = 0; i < n * k; ++i) wf[i] = oracle_f16_to_f32(w[i]);
    for (int64_t i = 0; i < m * k; ++i) xf[i] = oracle_f16_to_f32(x[i]);
    const int rc = oracle_gemm_f64(wf, xf, m, n, k, bias, epilogue, y, threads);
    free(wf);
    free(xf);
    return rc;
}

/* ------------------------------------------------------ ViT attention */

static void rope_pair_f64(const float* x, const float* freq_row, int half, double* outv) {
    for (int i = 0; i < half; ++i) {
        const double a = x[2 * i], b = x[2 * i + 1];
        const double c = freq_row[2 * i], sn = freq_row[2 * i + 1];
        outv[2 * i] = a * c - b * sn;
        outv[2 * i + 1] = a * sn + b * c;
    }
}

int oracle_vit_attention(const float* qkv, int64_t ldq, int grid_w, int grid_h, int heads, int head_dim,
                         int window, const float* freqs, const int64_t* rows, int64_t nrows, float* out,
                         int64_t ldo, int threads) {
    const int64_t tokens = (int64_t)grid_w * grid_h, E = (int64_t)heads * head_dim;
    if (head_dim % 2 || ldq < 3 * E || ldo < E || grid_w <= 0 || grid_h <= 0) return -1;
    if (window > 0 && (grid_w % window || grid_h % window)) return -1;
    const int64_t group = window > 0 ? (int64_t)window * window : tokens;
    const int half = head_dim / 2;
    if (!rows) nrows = tokens;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1)
#endif
    for (int64_t r = 0; r < nrows; ++r) {
        const int64_t t = rows ? rows[r] : r;
        const int ty = (int)(t / grid_w), tx = (int)(t % grid_w);
        /* tokens of the query's attention group, in window-local raster order */
        int64_t* members = (int64_t*)malloc((size_t)group * sizeof(int64_t));
        double* qv = (double*)malloc((size_t)head_dim * sizeof(double));
        double* kv = (double*)malloc((size_t)head_dim * sizeof(double));
        double* sc = (double*)malloc((size_t)group * sizeof(double));
        int64_t qpos;
        if (window > 0) {
            const int wy = ty / window, wx = tx / window;
            for (int y = 0; y < window; ++y)
                for (int x = 0; x < window; ++x)
                    members[y * window + x] = (int64_t)(wy * window + y) * grid_w + (wx * window + x);
            qpos = (int64_t)(ty % window) * window + (tx % window);
        } else {
            for (int64_t u = 0; u < tokens; ++u) members[u] = u;
            qpos = t;
        }
        for (int h = 0; h < heads; ++h) {
            rope_pair_f64(qkv + t * ldq + (int64_t)h * head_dim, freqs + qpos * head_dim, half, qv);
            double mx = -1e300;
            for (int64_t j = 0; j < group; ++j) {
                const int64_t u = members[j];
                rope_pair_f64(qkv + u * ldq + E + (int64_t)h * head_dim, freqs + j * head_dim, half, kv);
                double d = 0.0;
                for (int i = 0; i < head_dim; ++i) d += qv[i] * kv[i];
                sc[j] = d / sqrt((double)head_dim);
                if (sc[j] > mx) mx = sc[j];
            }
            double sum = 0.0;
            for (int64_t j = 0; j < group; ++j) { sc[j] = exp(sc[j] - mx); sum += sc[j]; }
            for (int i = 0; i < head_dim; ++i) {
                double o = 0.0;
                for (int64_t j = 0; j < group; ++j) o += sc[j] * qkv[members[j] * ldq + 2 * E + (int64_t)h * head_dim + i];
                out[r * ldo + (int64_t)h * head_dim + i] = (float)(o / sum);
            }
        }
        free(members); free(qv); free(kv); free(sc);
    }
    (void)threads;
    return 0;
}

/* ------------------------------------------- restated GGML CPU path
 *
 * Weights are decoded once ("prepared", as GGML's CPU repack does at load)
 * into 16-row groups: for every 4 columns, 16 rows x 4 unsigned codes
 * (Q8_0: q+128, Q4_K: q, Q5_K: q, Q6_K: q as stored, i.e. q+32).  Scales stay
 * in their GGUF integer/f16 form.  Activations are packed per call into Q8_0
 * (Q8_0 weights) or Q8_K (K-quant weights) exactly as the CPU backend pairs
 * them (backends/cpu.hpp:13-22); the dot products are integer per block with
 * f32 scale arithmetic. */

typedef struct {
    int type;
    int64_t k, n, groups, blocks;   /* blocks = 32-blocks (Q8_0) or 256-blocks */
    uint8_t* codes;                 /* [groups][k/4][16][4] */
    float* d;                       /* [groups][blocks][16] */
    float* dmin;                    /* [groups][blocks][16]   (Q4_K/Q5_K) */
    int32_t* sc;                    /* [groups][blocks][nsub][16] */
    int32_t* mn;                    /* [groups][blocks][8][16] (Q4_K/Q5_K) */
    int nsub;
} cpu_weights;

static void cpu_weights_free(cpu_weights* w) {
    free(w->codes); free(w->d); free(w->dmin); free(w->sc); free(w->mn);
    memset(w, 0, sizeof(*w));
}

static int cpu_weights_prepare(cpu_weights* w, int type, const uint8_t* rows, int64_t k, int64_t n) {
    memset(w, 0, sizeof(*w));
    const int64_t rb = oracle_row_bytes(type, k);
    if (rb < 0 || n <= 0) return -1;
    w->type = type; w->k = k; w->n = n;
    w->groups = (n + 15) / 16;
    w->blocks = k / oracle_block_elements(type);
    w->nsub = type == ORACLE_TYPE_Q6_K ? 16 : 8;
    w->codes = (uint8_t*)calloc((size_t)(w->groups * k * 16), 1);
    w->d = (float*)calloc((size_t)(w->groups * w->blocks * 16), sizeof(float));
    if (type != ORACLE_TYPE_Q8_0) {
        w->sc = (int32_t*)calloc((size_t)(w->groups * w->blocks * w->nsub * 16), sizeof(int32_t));
        if (type != ORACLE_TYPE_Q6_K) {
            w->dmin = (float*)calloc((size_t)(w->groups * w->blocks * 16), sizeof(float));
            w->mn = (int32_t*)calloc((size_t)(w->groups * w->blocks * 8 * 16), sizeof(int32_t));
        }
    }
    if (!w->codes || !w->d || (type != ORACLE_TYPE_Q8_0 && !w->sc) ||
        (type != ORACLE_TYPE_Q8_0 && type != ORACLE_TYPE_Q6_K && (!w->dmin || !w->mn))) {
        cpu_weights_free(w);
        return -1;
    }
    uint8_t q[256];
    for (int64_t r = 0; r < n; ++r) {
        const int64_t g = r / 16, lane = r % 16;
        const uint8_t* row = rows + r * rb;
        for (int64_t b = 0; b < w->blocks; ++b) {
            const int64_t be = oracle_block_elements(type);
            const uint8_t* o = row + b * oracle_block_bytes(type);
            float* dd = w->d + (g * w->blocks + b) * 16;
            if (type == ORACLE_TYPE_Q8_0) {
                dd[lane] = oracle_f16_to_f32(load_u16(o));
                for (int i = 0; i < 32; ++i) q[i] = (uint8_t)((int)(int8_t)o[2 + i] + 128);
            } else {
                decode_codes(type, o, q);
                int32_t* s = w->sc + ((g * w->blocks + b) * w->nsub) * 16;
                if (type == ORACLE_TYPE_Q6_K) {
                    dd[lane] = oracle_f16_to_f32(load_u16(o + 208));
                    for (int j = 0; j < 16; ++j) s[j * 16 + lane] = (int8_t)o[192 + j];
                } else {
                    int sc[8], m[8];
                    unpack_kquant_scales(o + 4, sc, m);
                    dd[lane] = oracle_f16_to_f32(load_u16(o));
                    w->dmin[(g * w->blocks + b) * 16 + lane] = oracle_f16_to_f32(load_u16(o + 2));
                    int32_t* mm = w->mn + ((g * w->blocks + b) * 8) * 16;
                    for (int j = 0; j < 8; ++j) { s[j * 16 + lane] = sc[j]; mm[j * 16 + lane] = m[j]; }
                }
            }
            for (int64_t i = 0; i < be; ++i) {
                const int64_t col = b * be + i;
                w->codes[((g * (k / 4) + col / 4) * 16 + lane) * 4 + col % 4] = q[i];
            }
        }
    }
    return 0;
}

/* Packed activation row: int8 codes plus per-block scale and sums. */
typedef struct {
    int8_t* q;          /* [m][k] */
    float* d;           /* [m][blocks] */
    int32_t* sums;      /* [m][k/16]: sums of 16 codes (Q8_K bsums; Q8_0 uses pairs) */
} cpu_acts;

static int pack_acts(const cpu_weights* w, const float* x, int64_t m, int64_t ldx, cpu_acts* a, int threads) {
    const int64_t k = w->k;
    a->q = (int8_t*)malloc((size_t)(m * k));
    a->d = (float*)malloc((size_t)(m * w->blocks) * sizeof(float));
    a->sums = (int32_t*)malloc((size_t)(m * (k / 16)) * sizeof(int32_t));
    if (!a->q || !a->d || !a->sums) return -1;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
#endif
    for (int64_t r = 0; r < m; ++r) {
        const float* v = x + r * ldx;
        if (w->type == ORACLE_TYPE_Q8_0) {
            uint8_t blk[34];
            for (int64_t b = 0; b < w->blocks; ++b) {
                oracle_quantize_q8_0(v + 32 * b, 32, blk);
                a->d[r * w->blocks + b] = oracle_f16_to_f32(load_u16(blk));
                memcpy(a->q + r * k + 32 * b, blk + 2, 32);
            }
        } else {
            uint8_t blk[292];
            for (int64_t b = 0; b < w->blocks; ++b) {
                oracle_quantize_q8_k(v + 256 * b, 256, blk);
                memcpy(&a->d[r * w->blocks + b], blk, 4);
                memcpy(a->q + r * k + 256 * b, blk + 4, 256);
            }
        }
        for (int64_t j = 0; j < k / 16; ++j) {
            int32_t s = 0;
            for (int i = 0; i < 16; ++i) s += a->q[r * k + 16 * j + i];
            a->sums[r * (k / 16) + j] = s;
        }
    }
    (void)threads;
    return 0;
}

/* Integer dot of 4 codes of lane `l` over columns [c0, c0+cnt). */
static inline int32_t dot_lane(const cpu_weights* w, int64_t g, int l, const int8_t* xq, int64_t c0, int cnt) {
    int32_t s = 0;
    for (int i = 0; i < cnt; ++i) {
        const int64_t col = c0 + i;
        s += (int32_t)w->codes[((g * (w->k / 4) + col / 4) * 16 + l) * 4 + col % 4] * xq[col];
    }
    return s;
}

/* Scalar kernel: 16 weight rows (one group) x one activation row. */
static void group_row_scalar(const cpu_weights* w, int64_t g, const cpu_acts* a, int64_t r, float out[16]) {
    const int64_t k = w->k;
    const int8_t* xq = a->q + r * k;
    const float* xd = a->d + r * w->blocks;
    const int32_t* xs = a->sums + r * (k / 16);
    for (int l = 0; l < 16; ++l) {
        float acc = 0.0f;
        for (int64_t b = 0; b < w->blocks; ++b) {
            const int64_t gb = g * w->blocks + b;
            if (w->type == ORACLE_TYPE_Q8_0) {
                const int32_t p = dot_lane(w, g, l, xq, 32 * b, 32) - 128 * (xs[2 * b] + xs[2 * b + 1]);
                acc += (float)p * (w->d[gb * 16 + l] * xd[b]);
            } else if (w->type == ORACLE_TYPE_Q6_K) {
                int32_t isum = 0;
                for (int j = 0; j < 16; ++j) {
                    const int32_t p = dot_lane(w, g, l, xq, 256 * b + 16 * j, 16) - 32 * xs[16 * b + j];
                    isum += p * w->sc[(gb * 16 + j) * 16 + l];
                }
                acc += (float)isum * (w->d[gb * 16 + l] * xd[b]);
            } else {
                int32_t isum = 0, msum = 0;
                for (int j = 0; j < 8; ++j) {
                    isum += dot_lane(w, g, l, xq, 256 * b + 32 * j, 32) * w->sc[(gb * 8 + j) * 16 + l];
                    msum += w->mn[(gb * 8 + j) * 16 + l] * (xs[16 * b + 2 * j] + xs[16 * b + 2 * j + 1]);
                }
                acc += (float)isum * (w->d[gb * 16 + l] * xd[b]) - (float)msum * (w->dmin[gb * 16 + l] * xd[b]);
            }
        }
        out[l] = acc;
    }
}

#ifdef ORACLE_X86
#define VNNI_TARGET __attribute__((target("avx512f,avx512bw,avx512vl,avx512vnni")))

/* 16 weight rows x 4 activation rows with VPDPBUSD: every 64-byte load of
 * weight codes (16 lanes x 4 columns) feeds 4 rows of broadcast activations. */
VNNI_TARGET static void group_rows4_vnni(const cpu_weights* w, int64_t g, const cpu_acts* a, int64_t r0,
                                         int nr, float out[4][16]) {
    const int64_t k = w->k, kq = k / 4;
    const uint8_t* wc = w->codes + g * kq * 64;
    __m512 acc[4];
    for (int i = 0; i < 4; ++i) acc[i] = _mm512_setzero_ps();
    const int8_t* xq[4];
    for (int i = 0; i < 4; ++i) xq[i] = a->q + (r0 + (i < nr ? i : 0)) * k;
    for (int64_t b = 0; b < w->blocks; ++b) {
        const int64_t gb = g * w->blocks + b;
        if (w->type == ORACLE_TYPE_Q8_0) {
            __m512i p[4];
            for (int i = 0; i < 4; ++i) p[i] = _mm512_setzero_si512();
            for (int c = 0; c < 8; ++c) {
                const int64_t quad = 8 * b + c;
                const __m512i wv = _mm512_loadu_si512((const void*)(wc + quad * 64));
                for (int i = 0; i < 4; ++i) {
                    int32_t xv;
                    memcpy(&xv, xq[i] + 4 * quad, 4);
                    p[i] = _mm512_dpbusd_epi32(p[i], wv, _mm512_set1_epi32(xv));
                }
            }
            const __m512 dw = _mm512_loadu_ps(w->d + gb * 16);
            for (int i = 0; i < 4; ++i) {
                const int64_t r = r0 + (i < nr ? i : 0);
                const int32_t sx = a->sums[r * (k / 16) + 2 * b] + a->sums[r * (k / 16) + 2 * b + 1];
                const __m512i pi = _mm512_sub_epi32(p[i], _mm512_set1_epi32(128 * sx));
                const __m512 scale = _mm512_mul_ps(dw, _mm512_set1_ps(a->d[r * w->blocks + b]));
                acc[i] = _mm512_fmadd_ps(_mm512_cvtepi32_ps(pi), scale, acc[i]);
            }
        } else {
            const int nsub = w->nsub, sub = 256 / nsub;
            __m512i isum[4], msum[4];
            for (int i = 0; i < 4; ++i) { isum[i] = _mm512_setzero_si512(); msum[i] = _mm512_setzero_si512(); }
            for (int j = 0; j < nsub; ++j) {
                __m512i p[4];
                for (int i = 0; i < 4; ++i) p[i] = _mm512_setzero_si512();
                for (int c = 0; c < sub / 4; ++c) {
                    const int64_t quad = 64 * b + (sub / 4) * j + c;
                    const __m512i wv = _mm512_loadu_si512((const void*)(wc + quad * 64));
                    for (int i = 0; i < 4; ++i) {
                        int32_t xv;
                        memcpy(&xv, xq[i] + 4 * quad, 4);
                        p[i] = _mm512_dpbusd_epi32(p[i], wv, _mm512_set1_epi32(xv));
                    }
                }
                const __m512i scv = _mm512_loadu_si512((const void*)(w->sc + (gb * nsub + j) * 16));
                for (int i = 0; i < 4; ++i) {
                    const int64_t r = r0 + (i < nr ? i : 0);
                    const int32_t* xs = a->sums + r * (k / 16) + 16 * b;
                    __m512i pi = p[i];
                    if (w->type == ORACLE_TYPE_Q6_K) pi = _mm512_sub_epi32(pi, _mm512_set1_epi32(32 * xs[j]));
                    isum[i] = _mm512_add_epi32(isum[i], _mm512_mullo_epi32(pi, scv));
                    if (w->type != ORACLE_TYPE_Q6_K) {
                        const __m512i mv = _mm512_loadu_si512((const void*)(w->mn + (gb * 8 + j) * 16));
                        msum[i] = _mm512_add_epi32(msum[i], _mm512_mullo_epi32(mv, _mm512_set1_epi32(xs[2 * j] + xs[2 * j + 1])));
                    }
                }
            }
            const __m512 dw = _mm512_loadu_ps(w->d + gb * 16);
            for (int i = 0; i < 4; ++i) {
                const int64_t r = r0 + (i < nr ? i : 0);
                const __m512 xd = _mm512_set1_ps(a->d[r * w->blocks + b]);
                acc[i] = _mm512_fmadd_ps(_mm512_cvtepi32_ps(isum[i]), _mm512_mul_ps(dw, xd), acc[i]);
                if (w->type != ORACLE_TYPE_Q6_K) {
                    const __m512 dm = _mm512_loadu_ps(w->dmin + gb * 16);
                    acc[i] = _mm512_fnmadd_ps(_mm512_cvtepi32_ps(msum[i]), _mm512_mul_ps(dm, xd), acc[i]);
                }
            }
        }
    }
    for (int i = 0; i < 4; ++i) _mm512_storeu_ps(out[i], acc[i]);
}
#endif

int oracle_cpu_has_vnni(void) {
#ifdef ORACLE_X86
    __builtin_cpu_init();
    return __builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512bw") ? 1 : 0;
#else
    return 0;
#endif
}

int oracle_cpu_linear(int type, const uint8_t* w_rows, int64_t k, int64_t n,
                      const float* x, int64_t m, int64_t ldx, const float* bias, int epilogue,
                      float* y, int64_t ldy, int threads) {
    if (m < 0 || ldx < k || ldy < n) return -1;
    if (type != ORACLE_TYPE_Q8_0 && type != ORACLE_TYPE_Q4_K && type != ORACLE_TYPE_Q5_K &&
        type != ORACLE_TYPE_Q6_K) return -1;
    if (k % 16) return -1;
    cpu_weights w;
    if (cpu_weights_prepare(&w, type, w_rows, k, n)) return -1;
    cpu_acts a = {0};
    if (pack_acts(&w, x, m, ldx, &a, threads)) {
        free(a.q); free(a.d); free(a.sums);
        cpu_weights_free(&w);
        return -1;
    }
    const int vnni = oracle_cpu_has_vnni();
    const int64_t mblocks = (m + 3) / 4;
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(dynamic, 8) num_threads(threads > 0 ? threads : 1)
#endif
    for (int64_t g = 0; g < w.groups; ++g)
        for (int64_t mb = 0; mb < mblocks; ++mb) {
            const int64_t r0 = mb * 4;
            const int nr = (int)(m - r0 < 4 ? m - r0 : 4);
            float out[4][16];
#ifdef ORACLE_X86
            if (vnni) {
                group_rows4_vnni(&w, g, &a, r0, nr, out);
            } else
#endif
            {
                for (int i = 0; i < nr; ++i) group_row_scalar(&w, g, &a, r0 + i, out[i]);
            }
            for (int i = 0; i < nr; ++i)
                for (int l = 0; l < 16; ++l) {
                    const int64_t col = g * 16 + l;
                    if (col >= n) break;
                    float v = out[i][l];
                    if (bias) v += bias[col];
                    if (epilogue == ORACLE_EPILOGUE_GELU_ERF) v = 0.5f * v * (1.0f + erff(v * 0.70710678f));
                    y[(r0 + i) * ldy + col] = v;
                }
        }
    (void)vnni;
    free(a.q); free(a.d); free(a.sums);
    cpu_weights_free(&w);
    return 0;
}

/* ------------------------------------------------- CPU flash attention */

#ifdef ORACLE_X86
#define AVX512_TARGET __attribute__((target("avx512f")))
AVX512_TARGET static float dot_f32_avx512(const float* a, const float* b, int n) {
    __m512 acc = _mm512_setzero_ps();
    int i = 0;
    for (; i + 16 <= n; i += 16) acc = _mm512_fmadd_ps(_mm512_loadu_ps(a + i), _mm512_loadu_ps(b + i), acc);
    float s = _mm512_reduce_add_ps(acc);
    for (; i < n; ++i) s += a[i] * b[i];
    return s;
}
AVX512_TARGET static void mad_f32_avx512(float* y, const float* x, float w, int n) {
    const __m512 wv = _mm512_set1_ps(w);
    int i = 0;
    for (; i + 16 <= n; i += 16)
        _mm512_storeu_ps(y + i, _mm512_fmadd_ps(_mm512_loadu_ps(x + i), wv, _mm512_loadu_ps(y + i)));
    for (; i < n; ++i) y[i] += x[i] * w;
}
AVX512_TARGET static void scale_f32_avx512(float* y, float w, int n) {
    const __m512 wv = _mm512_set1_ps(w);
    int i = 0;
    for (; i + 16 <= n; i += 16) _mm512_storeu_ps(y + i, _mm512_mul_ps(_mm512_loadu_ps(y + i), wv));
    for (; i < n; ++i) y[i] *= w;
}
#endif

static float dot_f32_scalar(const float* a, const float* b, int n) {
    float s = 0.0f;
    for (int i = 0; i < n; ++i) s += a[i] * b[i];
    return s;
}

static void flash_row(const float* q, const float* k, int64_t ldk, const float* v, int64_t ldv, int64_t n_kv, int hd,
                      float scale, float* acc, int wide) {
    float m = -INFINITY, sum = 0.0f;
    for (int i = 0; i < hd; ++i) acc[i] = 0.0f;
    for (int64_t j = 0; j < n_kv; ++j) {
        const float* kj = k + j * ldk;
        const float* vj = v + j * ldv;
#ifdef ORACLE_X86
        const float s = (wide ? dot_f32_avx512(q, kj, hd) : dot_f32_scalar(q, kj, hd)) * scale;
#else
        const float s = dot_f32_scalar(q, kj, hd) * scale;
#endif
        float ms = 1.0f, vs = 1.0f;
        if (s > m) {
            const float m_old = m;
            m = s;
            ms = expf(m_old - m);
#ifdef ORACLE_X86
            if (wide) scale_f32_avx512(acc, ms, hd);
            else
#endif
                for (int i = 0; i < hd; ++i) acc[i] *= ms;
        } else {
            vs = expf(s - m);
        }
#ifdef ORACLE_X86
        if (wide) mad_f32_avx512(acc, vj, vs, hd);
        else
#endif
            for (int i = 0; i < hd; ++i) acc[i] += vj[i] * vs;
        sum = sum * ms + vs;
    }
    const float inv = sum == 0.0f ? 0.0f : 1.0f / sum;
    for (int i = 0; i < hd; ++i) acc[i] *= inv;
    (void)wide;
}

int oracle_flash_attn_f32(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                          int64_t n_q, int64_t n_kv, int head_dim, float scale, float* out, int64_t ldo,
                          int threads) {
    if (!q || !k || !v || !out || n_q < 0 || n_kv <= 0 || head_dim <= 0 || ldq < head_dim || ldk < head_dim ||
        ldv < head_dim || ldo < head_dim)
        return -1;
    int wide = 0;
#ifdef ORACLE_X86
    wide = __builtin_cpu_supports("avx512f") ? 1 : 0;
#endif
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
#endif
    for (int64_t r = 0; r < n_q; ++r)
        flash_row(q + r * ldq, k, ldk, v, ldv, n_kv, head_dim, scale, out + r * ldo, wide);
    (void)threads;
    return 0;
}
