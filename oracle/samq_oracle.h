/*
 * samq_oracle.h -- CPU restatement of SAM.cpp's quantized-linear path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the B200 path
 * (tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm).  The product library never links, loads or calls it.
 *
 * What it restates (reference paths are relative to the SAM.cpp tree):
 *   - GGUF block formats Q8_0 / Q4_K / Q5_K / Q6_K.  The arithmetic lives in
 *     GGML (pinned d7cb5741, v0.26.0, cmake/ggml.cmake:10-15), which is not
 *     vendored.  The executable spec used here is gguf-py 0.19.0
 *     (gguf/quants.py), the version the reference CI pins
 *     (.github/workflows/quick-checks.yml:22) and whose Q8_0 quantizer the
 *     reference converter calls (tools/convert/sam3_gguf.py:319-324).
 *   - GGML CUDA activation staging: Q8_1 36-byte MMVQ blocks
 *     (tools/validation/verify_q8_rhs_staging.py:24-83) and MMQ-D4 144-byte
 *     blocks (tools/validation/verify_q8_mmq_rhs_staging.py:24-67,
 *     cmake/patches/ggml-precise-cuda.patch:623-633,
 *     tests/runtime/ggml/test_cuda_q8_mmq_scale.cpp:33-93).
 *   - GGML CPU activation packing Q8_K (wire layout pinned by
 *     tools/benchmark/cpu_quantized_matmul.hpp:26-42) and the CPU dot pairing
 *     Q8_0 x Q8_0 / K-quant x Q8_K (src/runtime/ggml/backends/cpu.hpp:13-22).
 *   - Decoded-operand scalar references in f64
 *     (tests/runtime/ggml/test_quantization.cpp:469-494,
 *     tools/benchmark/cpu_quantized_matmul.hpp:195-222,
 *     tools/validation/verify_q8_mmq_dots.py:54-105).
 *
 * Parity pinning: formats and the Q8_0 quantizer are pinned byte-for-byte to
 * gguf-py outputs (tests/golden).  Q8_1 / D4 staging is pinned to the
 * reference verifier rules and the MMQ scale known-answer test.  Q8_K byte
 * rounding inside GGML is unpinned (only its layout and output tolerance are
 * published by the reference).
 */
#ifndef SAMQ_ORACLE_H
#define SAMQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids (ggml.h enum ggml_type): kept so callers speak GGUF ids. */
enum {
    ORACLE_TYPE_F32 = 0,
    ORACLE_TYPE_F16 = 1,
    ORACLE_TYPE_Q8_0 = 8,
    ORACLE_TYPE_Q8_1 = 9,
    ORACLE_TYPE_Q4_K = 12,
    ORACLE_TYPE_Q5_K = 13,
    ORACLE_TYPE_Q6_K = 14,
    ORACLE_TYPE_Q8_K = 15,
};

/* Elements per block and bytes per block (gguf-py GGML_QUANT_SIZES). */
int64_t oracle_block_elements(int type);
int64_t oracle_block_bytes(int type);
/* Bytes of one packed row of `k` elements, or -1 when k is not block aligned. */
int64_t oracle_row_bytes(int type, int64_t k);

/* IEEE binary16 conversions, round to nearest even. */
uint16_t oracle_f32_to_f16(float value);
float oracle_f16_to_f32(uint16_t bits);

/* gguf-py Q8_0.quantize_blocks (gguf/quants.py), bit exact. */
int oracle_quantize_q8_0(const float* x, int64_t n, uint8_t* out);

/* Own K-quant packer (GGML's make_qkx search is not available; any valid
 * packing is acceptable because GEMM parity is defined on decoded weights). */
int oracle_quantize_kquant(int type, const float* x, int64_t n, uint8_t* out);

/* gguf-py dequantize for Q8_0 / Q4_K / Q5_K / Q6_K, bit exact in f32. */
int oracle_dequantize(int type, const uint8_t* blocks, int64_t n, float* out);

/* Q8_1 MMVQ staging: per 32 values {f16 d, f16 sum, int8 q[32]} (36 B).
 * d = f16(amax/127), q = roundf(x * (127/amax)) with IEEE division,
 * sum = f16 of the 32-lane xor-butterfly f32 sum of the source values.
 * x is [rows][ld] f32, k % 32 == 0; out is [rows][k/32] blocks. */
int oracle_quantize_q8_1(const float* x, int64_t rows, int64_t k, int64_t ld, uint8_t* out);

/* MMQ-D4 staging: per 128 values {f32 d[4], int8 q[128]} (144 B); width
 * padded with zeros to a multiple of 512; blocks stored [k_block][row]. */
int64_t oracle_mmq_d4_bytes(int64_t rows, int64_t k);
int oracle_quantize_mmq_d4(const float* x, int64_t rows, int64_t k, int64_t ld, uint8_t* out);

/* Tensor-core A operand of the B200 path: f16(f32(d_half) * q) for every
 * element of the Q8_1 blocks of x.  out is [rows][k] binary16. */
int oracle_act_f16(const float* x, int64_t rows, int64_t k, int64_t ld, uint16_t* out);
/* Decoded Q8_1 activations f32(d_half) * q, [rows][k]. */
int oracle_q8_1_decode(const uint8_t* q8_1, int64_t rows, int64_t k, float* out);

/* GGML CPU Q8_K activation packing (f32 d, int8 q[256], int16 bsums[16]). */
int oracle_quantize_q8_k(const float* x, int64_t n, uint8_t* out);

/* ---- device weight layout ("packets") produced by the GPU repack -------
 * The B200 path stores each weight matrix [n][k] as packets of 128 rows x 64
 * columns.  packet (t, c) covers rows 128t..128t+127 and columns 64c..64c+63
 * and holds, row after row, the codes of that chunk followed by one 8-byte
 * scale record per row.  Rows past n are zero.  The layout is lossless:
 * oracle_unpack_packets() rebuilds the GGUF rows byte for byte. */
int64_t oracle_packet_code_bytes(int type);   /* per row per 64 columns */
int64_t oracle_packet_bytes(int type);        /* one 128 x 64 packet */
int64_t oracle_packets_size(int type, int64_t k, int64_t n);
int oracle_pack_packets(int type, int64_t k, int64_t n, const uint8_t* gguf_rows, uint8_t* packets);
int oracle_unpack_packets(int type, int64_t k, int64_t n, const uint8_t* packets, uint8_t* gguf_rows);

/* Tensor-core B operand of the B200 path: f16 of the f32 dequantized
 * weights, [n][k] binary16. */
int oracle_weight_f16(int type, int64_t k, int64_t n, const uint8_t* gguf_rows, uint16_t* out);

/* ---- GEMM references ----------------------------------------------------
 * Y[m][n] = sum_k W[n][k] * X[m][k] (GGML mul_mat(W, X), ops.hpp:40-45).
 * f64 accumulation over the given f32 operands, optional bias and erf-GELU
 * (vision.hpp:234-236), result rounded to f32. */
enum { ORACLE_EPILOGUE_NONE = 0, ORACLE_EPILOGUE_GELU_ERF = 1 };
int oracle_gemm_f64(const float* w, const float* x, int64_t m, int64_t n, int64_t k,
                    const float* bias, int epilogue, float* y, int threads);
/* Same over binary16 operands (the exact inputs of the tensor-core MMA). */
int oracle_gemm_f16_f64(const uint16_t* w, const uint16_t* x, int64_t m, int64_t n, int64_t k,
                        const float* bias, int epilogue, float* y, int threads);

/* ViT attention of one block (src/models/sam3/vision.hpp:152-243): qkv is the
 * f32 output of the qkv linear, [tokens][ldq] with columns Q | K | V, each
 * head-major (head h at 64h..64h+63); tokens are the raster grid W x H.  RoPE
 * (vision.hpp:100-148) rotates channel pairs (2i, 2i+1) of Q and K by
 * (cos, sin) = freqs[pos][i][0..1], pos = window-local raster position (or the
 * global one when window == 0).  Softmax(Q K^T / sqrt(hd)) V over the tokens of
 * the same window (24x24 windows of the grid, vision.hpp:170-173) or of the
 * whole grid.  f64 arithmetic.  Computes the query tokens listed in `rows`
 * (raster indices; NULL = all) into out[r][ldo] for r = 0..nrows-1. */
int oracle_vit_attention(const float* qkv, int64_t ldq, int grid_w, int grid_h, int heads, int head_dim,
                         int window, const float* freqs, const int64_t* rows, int64_t nrows, float* out,
                         int64_t ldo, int threads);

/* Restated GGML CPU path (the timed CPU baseline): pack X rows to Q8_0
 * (Q8_0 weights) or Q8_K (K-quant weights), integer block dots, f32 scales,
 * f32 output, OpenMP over `threads` host threads; AVX-512 VNNI when the host
 * has it.  Returns 0 on success. */
int oracle_cpu_linear(int type, const uint8_t* w_rows, int64_t k, int64_t n,
                      const float* x, int64_t m, int64_t ldx, const float* bias, int epilogue,
                      float* y, int64_t ldy, int threads);
/* 1 when the AVX-512 VNNI kernel is in use on this host. */
int oracle_cpu_has_vnni(void);

/* Restated GGML CPU flash attention for F32 Q / K / V (the timed CPU baseline's
 * attention; ggml_flash_attn_ext as sam3_vit_block_forward calls it,
 * src/models/sam3/vision.hpp:216, no mask): one head, each query row on its
 * own with an online softmax in f32 -- s = (q . k_j) * scale; when s exceeds
 * the running maximum M the f32 accumulator and the running sum are rescaled
 * by expf(M_old - s), otherwise v_j is added with weight expf(s - M); the row
 * ends divided by the running sum.  q [n_q][ldq], k / v [n_kv][ldk / ldv],
 * out [n_q][ldo]; OpenMP over the query rows.  Returns 0 on success. */
int oracle_flash_attn_f32(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                          int64_t n_q, int64_t n_kv, int head_dim, float scale, float* out, int64_t ldo,
                          int threads);

#ifdef __cplusplus
}
#endif
#endif
