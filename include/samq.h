/*
 * samq.h -- C ABI of the B200 (sm_100a) quantized-linear path of SAM.cpp.
 *
 * This library replaces, for the quantized linears of SAM 3, the GGML CUDA
 * backend that SAM.cpp reaches through ggml_backend_sched_graph_compute
 * (src/runtime/ggml/workspace.hpp:163) -> ggml_cuda_mul_mat -> MMQ/MMVQ with
 * Q8_1 activation staging (cmake/patches/ggml-native-activation.patch:78-86).
 * The ABI follows the convention of SAM.cpp's private Q8-RHS extension
 * (cmake/patches/ggml-native-activation.patch:12-26, looked up by name in
 * src/runtime/ggml/backends/cuda_activation.hpp:22-25): plain extern "C",
 * versioned `_v1` symbols, info structs whose first field is `version`.
 * Differences: every call returns a status code instead of bool, and a
 * thread-local message explains the last failure.
 *
 * Conventions
 *   - GGML mul_mat(W, X) semantics (src/models/sam3/ops.hpp:40-45): W is
 *     [n][k] packed GGUF rows (one row per output channel), X is [m][k] f32
 *     row-major with row stride ldx (elements), Y is [m][n] f32 row-major with
 *     row stride ldy: Y[i][j] = sum_t W[j][t] * X[i][t] (+ bias[j]).
 *   - Type ids are GGML's (ggml_type): Q8_0 = 8, Q4_K = 12, Q5_K = 13,
 *     Q6_K = 14; activation staging Q8_1 = 9.
 *   - Device pointers are owned by the caller, as is the CUDA stream
 *     (`stream` is a cudaStream_t; NULL is the legacy default stream).  The
 *     library owns repacked weights and per-stream scratch memory.
 *   - Calls that share a stream are ordered by it; calls on one weights
 *     handle from several host threads must be serialized by the caller (the
 *     reference serializes sessions with execution_mutex,
 *     src/models/sam3/image_session.hpp:34,57).
 *   - No C++ exception crosses this boundary.
 */
#ifndef SAMQ_H
#define SAMQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SAMQ_ABI_VERSION 1

typedef enum samq_status {
    SAMQ_OK = 0,
    SAMQ_ERR_INVALID_ARGUMENT = 1, /* shape, stride, alignment or type rejected */
    SAMQ_ERR_UNSUPPORTED = 2,      /* device is not sm_100 or the library lacks its code */
    SAMQ_ERR_CUDA = 3,             /* a CUDA runtime call failed (message has the name) */
    SAMQ_ERR_OUT_OF_MEMORY = 4,
    SAMQ_ERR_RANGE = 5,            /* activations non-finite or beyond the f16 operand range */
    SAMQ_ERR_TIMEOUT = 6,          /* a bounded device-side wait gave up */
    SAMQ_ERR_PAYLOAD = 7           /* packed weight block has a non-finite scale */
} samq_status;

enum {
    SAMQ_TYPE_Q8_0 = 8,
    SAMQ_TYPE_Q8_1 = 9,
    SAMQ_TYPE_Q4_K = 12,
    SAMQ_TYPE_Q5_K = 13,
    SAMQ_TYPE_Q6_K = 14
};

enum {
    SAMQ_EPILOGUE_NONE = 0,
    SAMQ_EPILOGUE_GELU_ERF = 1 /* ggml_gelu_erf after the bias (src/models/sam3/vision.hpp:234-236) */
};

/* Arithmetic of the ViT attention and patch embedding: sam::CudaComputeMode
 * (include/sam/types.hpp:13,21; default F32).  F32 is the reference's default
 * precise mode (GGML_PREC_F32 attention, F32 convolution columns); F16 is its
 * opt-in reduced mode (src/runtime/ggml/backends/cuda.hpp:82-92,177-186: f16
 * Q / K / V / P on the tensor cores, f16 convolution columns).  Quantized
 * linears compute the same way in both modes, as in the reference (MMQ over
 * Q8_1-staged activations). */
enum {
    SAMQ_COMPUTE_F32 = 0,
    SAMQ_COMPUTE_F16 = 1
};

typedef struct samq_weights samq_weights;

/* Replaces the device checks of make_cuda_backend
 * (src/runtime/ggml/backends/cuda.hpp:156-189). */
struct samq_capabilities_v1 {
    uint32_t version;            /* = 1 */
    int32_t device;
    int32_t cc_major, cc_minor;  /* sm_100 required */
    int32_t sm_count;
    uint64_t global_memory_bytes;
    uint64_t max_shared_memory_per_block;
    char name[256];
};

/* Mirrors ggml_sam_q8_rhs_info (cmake/patches/ggml-native-activation.patch:10-16). */
struct samq_counters_v1 {
    uint32_t version;            /* = 1 */
    uint32_t path;               /* 1: tcgen05 GEMM over packet weights */
    uint64_t launches;           /* GEMM launches recorded on this handle */
    uint64_t payload_bytes;      /* bytes of the last activation staging buffer */
    uint64_t allocation_bytes;   /* bytes of the scratch allocation that held it */
    uint64_t weight_bytes;       /* device bytes owned by the handle */
};

/* Thread-local text of the last failure on the calling thread ("" if none). */
const char* samq_last_error_v1(void);

/* Select and check `device`; fails with SAMQ_ERR_UNSUPPORTED unless it is an
 * sm_100 part.  Replaces ggml_backend_reg_by_name("CUDA") + device init
 * (src/runtime/ggml/backends/cuda.hpp:159-165). */
samq_status samq_init_v1(int device);
samq_status samq_capabilities_v1(int device, struct samq_capabilities_v1* info);

/* K4: load-time repack.  `gguf_rows` is HOST memory holding n packed rows of
 * k elements in GGUF layout (Q8_0 34 B / 32, Q4_K 144 B / 256, Q5_K 176 B /
 * 256, Q6_K 210 B / 256).  Validates every block scale is finite
 * (src/models/sam3/weights.hpp:384-425) and repacks on the device into the
 * library's packet layout.  Replaces ggml_backend_alloc_ctx_tensors +
 * ggml_backend_tensor_set of a WEIGHTS buffer (src/models/sam3/model.hpp:114-133). */
samq_status samq_weights_create_v1(int device, int type, int64_t k, int64_t n,
                                   const void* gguf_rows, size_t bytes, void* stream,
                                   samq_weights** out);
samq_status samq_weights_destroy_v1(samq_weights* weights);
/* Inverse repack into host GGUF rows (bit-exact round trip), synchronous. */
samq_status samq_weights_export_v1(const samq_weights* weights, void* gguf_rows, size_t bytes);
/* Device address and size of the packet layout (read-only). */
samq_status samq_weights_packets_v1(const samq_weights* weights, const void** packets, size_t* bytes);

/* K1: GGML CUDA quantize_q8_1 staging (MMVQ, 36 B per 32 values: f16 d,
 * f16 sum, int8[32]); x is [rows][ld] f32 on the device, out holds
 * rows * k/32 blocks.  Contract: tools/validation/verify_q8_rhs_staging.py:24-83. */
samq_status samq_quantize_q8_1_v1(const float* x, int64_t rows, int64_t k, int64_t ld,
                                  void* out, void* stream);
/* K1: GGML CUDA quantize_mmq_q8_1 D4 staging (144 B per 128 values: f32 d[4],
 * int8[128]; width zero-padded to 512; blocks stored [k/128][rows]).
 * Contract: tools/validation/verify_q8_mmq_rhs_staging.py:24-67,
 * tests/runtime/ggml/test_cuda_q8_mmq_scale.cpp:33-93. */
size_t samq_mmq_d4_bytes_v1(int64_t rows, int64_t k);
samq_status samq_quantize_mmq_q8_1_v1(const float* x, int64_t rows, int64_t k, int64_t ld,
                                      void* out, void* stream);

/* K1 + K2: Y = gelu?(X . W^T + bias).  Activations are staged exactly as the
 * Q8_1 rule above, then multiplied on the tcgen05 tensor cores with f32
 * accumulation.  Replaces the GGML_OP_MUL_MAT node of sam3_channel_projection
 * (src/models/sam3/ops.hpp:40-45) and the text/decoder linears.  bias may be
 * NULL.  ldx % 4 == 0 and ldy % 4 == 0 (16-byte rows). */
samq_status samq_linear_v1(const samq_weights* weights, const float* x, int64_t m, int64_t ldx,
                           const float* bias, int epilogue, float* y, int64_t ldy, void* stream);
/* K2 over already-staged activations: `x_q8_1` holds m * k/32 Q8_1 blocks as
 * written by samq_quantize_q8_1_v1. */
samq_status samq_linear_q8_1_v1(const samq_weights* weights, const void* x_q8_1, int64_t m,
                                const float* bias, int epilogue, float* y, int64_t ldy, void* stream);

/* K1 alone: stage f32 activations into the tensor-core A operand, f16
 * [rows][k] row-major, each value f16(f32(d) * q) of its Q8_1 block (the
 * rule of samq_quantize_q8_1_v1).  samq_linear_v1 == this + samq_linear_f16_v1. */
samq_status samq_stage_f16_v1(const float* x, int64_t rows, int64_t k, int64_t ld, void* out_f16, void* stream);
/* K2 alone over f16 activations [m][ldx] (ldx % 8 == 0, 16-byte aligned rows).
 * Same product as the reference's F16 compute mode for a quantized weight
 * (src/runtime/ggml/backends/cuda.hpp:177-186 selects F16 operands). */
samq_status samq_linear_f16_v1(const samq_weights* weights, const void* x_f16, int64_t m, int64_t ldx,
                               const float* bias, int epilogue, float* y, int64_t ldy, void* stream);

/* K3: RoPE + self-attention of one SAM 3 ViT block.  qkv is the device f32
 * output of the block's qkv linear (+bias), [grid_h * grid_w][ldq] in raster
 * token order, columns Q | K | V, each head-major with head_dim = 64.  RoPE
 * rotates channel pairs of Q and K by freqs_cis[pos][i] = (cos, sin)
 * ([positions][32][2] f32; positions = window * window for windowed blocks,
 * grid_w * grid_h for global ones).  Attention is softmax(Q K^T / 8) V within
 * each window x window tile of the grid (window > 0; the grid must divide) or
 * over the whole grid (window == 0).  out is [tokens][ldo] f32 in raster order
 * (head h at columns 64h..64h+63).  Replaces the RoPE, win_part, flash_attn_ext
 * and win_unpart nodes of sam3_vit_block_forward
 * (src/models/sam3/vision.hpp:100-148,170-227) and the precise F32 attention
 * of cmake/patches/ggml-precise-cuda.patch:448-606.  Operands are f16 on the
 * tensor cores with f32 accumulation and an f32 online softmax. */
samq_status samq_vit_attention_v1(const float* qkv, int64_t ldq, int grid_w, int grid_h, int heads, int head_dim,
                                  int window, const float* freqs_cis, float* out, int64_t ldo, void* stream);
/* samq_vit_attention_v1 with the compute mode chosen: SAMQ_COMPUTE_F16 is
 * exactly samq_vit_attention_v1; SAMQ_COMPUTE_F32 keeps Q, K, V and P in f32
 * (RoPE with GGML's rounding, f32 products and expf softmax on the FP32 pipe),
 * the reference's GGML_PREC_F32 attention checked at 1e-5 by
 * tests/runtime/ggml/test_precision.cpp:68-126. */
samq_status samq_vit_attention_v2(const float* qkv, int64_t ldq, int grid_w, int grid_h, int heads, int head_dim,
                                  int window, const float* freqs_cis, float* out, int64_t ldo, int compute,
                                  void* stream);

/* sam3_apply_rope (src/models/sam3/vision.hpp:113-148) on its own: x and out
 * are device f32 [head_batches][tokens][head_dim] (GGML [head_dim, N,
 * heads * B]), freqs_cis [tokens][head_dim / 2][2] (cos, sin); channel pairs
 * (2i, 2i+1) become (re cos - im sin, re sin + im cos), each product and the
 * sum rounded to f32 as GGML's mul / sub / add nodes do.  head_dim == 64;
 * out may equal x. */
samq_status samq_vit_rope_v1(const float* x, int64_t tokens, int64_t head_batches, int head_dim,
                             const float* freqs_cis, float* out, void* stream);

/* One SAM 3 ViT block, pre-LN (src/models/sam3/vision.hpp:152-243):
 *   x = x + proj(attn(RoPE(qkv(LN1(x)))))   (windowed or global attention)
 *   x = x + fc2(GELU_erf(fc1(LN2(x))))
 * Every linear consumes its input through the Q8_1 staging rule of
 * samq_quantize_q8_1_v1, as GGML's CUDA path does for quantized weights.
 * Parameters are device f32 arrays of the reference tensors
 * (src/models/sam3/tensors.hpp:108-126): LayerNorm weight / bias [E], linear
 * biases [N], freqs_cis [positions][32][2].  Linears are weight handles:
 * qkv E -> 3E, proj E -> E, fc1 E -> MLP, fc2 MLP -> E, with E = 64 * heads
 * and E in {256, 512, 1024}; MLP % 32 == 0. */
typedef struct samq_vit_block_v1 {
    uint32_t version;  /* 1, or 2 with the compute field */
    int32_t window;    /* 24: windowed blocks (grid divisible by it), 0: global */
    const float* norm1_w;
    const float* norm1_b;
    const samq_weights* qkv;
    const float* qkv_b;
    const samq_weights* proj;
    const float* proj_b;
    const float* norm2_w;
    const float* norm2_b;
    const samq_weights* fc1;
    const float* fc1_b;
    const samq_weights* fc2;
    const float* fc2_b;
    const float* freqs_cis;
    /* version >= 2 only: SAMQ_COMPUTE_F32 (the reference's default) or
     * SAMQ_COMPUTE_F16.  A version-1 descriptor (which ends before this field)
     * runs SAMQ_COMPUTE_F16.  In F32 mode the qkv linear's output stays f32 and
     * the attention is samq_vit_attention_v2's F32 path. */
    int32_t compute;
} samq_vit_block_v1;

/* Runs one block in place on the residual stream x, device f32
 * [grid_h * grid_w][E] in raster token order (the reference's [E, W, H, 1]). */
samq_status samq_vit_block_forward_v1(const samq_vit_block_v1* block, float* x, int grid_w, int grid_h,
                                      void* stream);

/* The same block over `batch` images at once (config 5's per-GPU batches):
 * x is [batch][grid_h * grid_w][E], image after image.  Each image's result is
 * bit-identical to samq_vit_block_forward_v1 on that image alone; one call
 * launches the block's kernels once for the whole batch. */
samq_status samq_vit_block_forward_batch_v1(const samq_vit_block_v1* block, float* x, int batch, int grid_w,
                                            int grid_h, void* stream);

/* Backbone prefix (src/models/sam3/vision.hpp:252-282): patch embedding (an
 * unpadded patch x patch convolution without bias, weight [E][3][patch][patch]
 * f32), + pos_embed ([pos_grid][pos_grid][E] f32, tiled over the token grid),
 * then ln_pre (weight / bias [E]).  image is device f32 [3][height][width]
 * (normalized, channel planes); x receives [tokens][E] f32, tokens =
 * (height / patch) * (width / patch) in raster order.  The convolution runs on
 * the tensor cores with f16 operands and f32 accumulation. */
samq_status samq_vit_prefix_v1(const float* image, int width, int height, int patch, const float* patch_w,
                               int64_t embed, const float* pos_embed, int pos_grid, const float* ln_w,
                               const float* ln_b, float* x, void* stream);
/* samq_vit_prefix_v1 with the compute mode chosen: SAMQ_COMPUTE_F16 is
 * samq_vit_prefix_v1 (f16 convolution columns, as the reference's F16 mode
 * sets convolution_columns_type, src/runtime/ggml/backends/cuda.hpp:182-185);
 * SAMQ_COMPUTE_F32 keeps F32 columns and runs the convolution with F32
 * semantics (the three-term TF32 split of the dense modules below). */
samq_status samq_vit_prefix_v2(const float* image, int width, int height, int patch, const float* patch_w,
                               int64_t embed, const float* pos_embed, int pos_grid, const float* ln_w,
                               const float* ln_b, float* x, int compute, void* stream);

/* ---- Text encoder and general attention ------------------------------------
 * The SAM 3 text encoder (src/models/sam3/text_encoder.hpp:68-180):
 *   x = token_embed[ids] + pos_embed                       (samq_token_embed_v1)
 *   24 x pre-LN block with a causal mask                   (samq_text_block_forward_v1)
 *   features = resizer(LN_final(x))                        (samq_layer_norm_v1 + samq_linear_v1)
 * The block's linears are quantized weight handles (Q8_0 in the reference's
 * full-linear and mixed profiles) and stage their inputs to Q8_1 like every
 * quantized linear here; its attention keeps F32 operands (the reference runs
 * masked attention at GGML_PREC_F32 in both compute modes,
 * src/runtime/ggml/backends/cuda.hpp:86-91). */
typedef struct samq_text_block_v1 {
    uint32_t version;  /* 1 */
    const float* norm1_w;   /* text.blocks.N.ln_1.weight [E] */
    const float* norm1_b;
    const samq_weights* in_proj;   /* attn.in_proj.weight, E -> 3E (Q | K | V, heads of 64) */
    const float* in_proj_b;
    const samq_weights* out_proj;  /* attn.out_proj.weight, E -> E */
    const float* out_proj_b;
    const float* norm2_w;   /* ln_2 */
    const float* norm2_b;
    const samq_weights* fc1;       /* mlp.fc1.weight, E -> MLP, erf-GELU after the bias */
    const float* fc1_b;
    const samq_weights* fc2;       /* mlp.fc2.weight, MLP -> E */
    const float* fc2_b;
} samq_text_block_v1;

/* One block in place on x, device f32 [tokens][E] (E = 64 * heads). */
samq_status samq_text_block_forward_v1(const samq_text_block_v1* block, float* x, int tokens, void* stream);

/* ggml_get_rows + ggml_add: out[i] = table[ids[i]] + pos[i] (pos may be NULL).
 * table is device f32 [vocab][width], ids HOST int32 [count] (each checked to
 * lie in [0, vocab); the reference's tokenizer validates ids before this node,
 * src/models/sam3/tokenizer.hpp:103-118), pos / out device f32 [count][width]. */
samq_status samq_token_embed_v1(const float* table, int64_t vocab, int width, const int32_t* ids, int count,
                                const float* pos, float* out, void* stream);

/* sam3_layer_norm in f32 (ggml_norm with eps, then * w + b; b may be NULL),
 * rows of `width` values: x [rows][ldx] -> out [rows][ldo] (may alias). */
samq_status samq_layer_norm_v1(const float* x, int64_t rows, int width, int64_t ldx, const float* w, const float* b,
                               float eps, float* out, int64_t ldo, void* stream);

/* ggml_flash_attn_ext at GGML_PREC_F32 for the fusion / decoder / text
 * attentions: per head h, out = softmax(scale Q_h K_h^T + bias) V_h with F32
 * operands.  q [lq][ldq], k and v [lk][ldk / ldv], out [lq][ldo], head h at
 * columns h*head_dim (head_dim 32 or 64, all strides multiples of 4 floats,
 * pointers 16-byte aligned).  bias (nullable) is additive,
 * bias[h * bias_h + q * bias_q + k] (a key padding mask: bias_h = bias_q = 0,
 * -INFINITY at masked keys); causal != 0 masks keys k > q.  A query whose
 * keys are all masked gets 0. */
samq_status samq_attention_v1(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                              int lq, int lk, int heads, int head_dim, float scale, int causal, const float* bias,
                              int64_t bias_h, int64_t bias_q, float* out, int64_t ldo, void* stream);

/* ---- Fusion encoder -----------------------------------------------------------
 * A linear of the fusion / decoder modules is either a quantized weight handle
 * (the full-linear Q8_0 profiles) or a dense F32 / F16 handle of kind
 * SAMQ_DENSE_LINEAR (the mixed profile's fusion=f32, decoder=f32): exactly one
 * of the two is non-NULL. */
struct samq_dense;
typedef struct samq_linear_ref_v1 {
    const samq_weights* quantized;
    const struct samq_dense* dense;
    const float* bias;  /* [n] or NULL */
} samq_linear_ref_v1;

/* One fusion-encoder layer (src/models/sam3/fusion_encoder.hpp:38-150), tensor
 * names fenc.layers.N.* (src/models/sam3/tensors.hpp:218-243), width D:
 *   x = x + sa.out_proj(attn(Q, K from LN1(x) + pos; V from LN1(x)))
 *   x = x + ca.out_proj(attn(Q from LN2(x); K, V from prompt; + prompt_bias))
 *   x = x + linear2(ReLU(linear1(LN3(x))))
 * in_proj weights are [3D][D] (Q | K | V rows, D % 128 == 0); heads of D / heads
 * channels (32 or 64), attention with F32 operands. */
typedef struct samq_fusion_layer_v1 {
    uint32_t version;  /* 1 */
    int32_t heads;     /* 8 in SAM 3 */
    const float *norm1_w, *norm1_b, *norm2_w, *norm2_b, *norm3_w, *norm3_b;
    samq_linear_ref_v1 sa_in_proj, sa_out_proj, ca_in_proj, ca_out_proj, linear1, linear2;
} samq_fusion_layer_v1;

/* x: device f32 [tokens][D] image tokens (in place), pos [tokens][D] their
 * positional encoding, prompt [prompt_tokens][D] the prompt tokens (text
 * features and the geometry token), prompt_bias [prompt_tokens] additive key
 * bias (0 or a large negative value at padding tokens; NULL: none). */
samq_status samq_fusion_layer_forward_v1(const samq_fusion_layer_v1* layer, float* x, const float* pos, int tokens,
                                         const float* prompt, const float* prompt_bias, int prompt_tokens,
                                         void* stream);

/* ---- DETR decoder, scoring and presence head ----------------------------------
 * src/models/sam3/detector.hpp:67-713, tensor names ddec.*, scoring.*
 * (src/models/sam3/tensors.hpp:245-351).  One layer's weights (post-norm
 * sublayers in this order): self-attention -> norm2, text cross-attention ->
 * norm_ca_text, image cross-attention with the box relative-position bias ->
 * norm1, ReLU FFN -> norm3.  in_proj weights are [3D][D] (Q | K | V rows). */
typedef struct samq_decoder_layer_v1 {
    samq_linear_ref_v1 sa_in_proj, sa_out_proj, ca_text_in_proj, ca_text_out_proj, ca_in_proj, ca_out_proj,
        linear1, linear2;
    const float *norm1_w, *norm1_b, *norm2_w, *norm2_b, *norm_ca_text_w, *norm_ca_text_b, *norm3_w, *norm3_b;
} samq_decoder_layer_v1;

typedef struct samq_decoder_v1 {
    uint32_t version;  /* 1 */
    int32_t heads;     /* 8 */
    int32_t layers;    /* 6 */
    int32_t queries;   /* 200 */
    const samq_decoder_layer_v1* layer;  /* [layers], host memory */
    const float* query_embed;       /* ddec.query_embed.weight [queries][D] */
    const float* presence_token;    /* ddec.presence_token.weight [D] */
    const float* reference_points;  /* ddec.reference_points.weight [queries][4], f32 */
    samq_linear_ref_v1 ref_point_head[2];  /* 512 -> D (ReLU) -> D */
    samq_linear_ref_v1 bbox_embed[3];      /* D -> D (ReLU) -> D (ReLU) -> 4 */
    const float *rpb_x0_w, *rpb_x0_b, *rpb_y0_w, *rpb_y0_b;  /* boxRPB layers.0: [256][2], [256] f32 */
    samq_linear_ref_v1 rpb_x1, rpb_y1;     /* boxRPB layers.1: 256 -> heads */
    const float *norm_w, *norm_b;          /* ddec.norm */
    const float *presence_norm_w, *presence_norm_b;  /* ddec.presence_token_out_norm */
    samq_linear_ref_v1 presence_head[3];   /* D -> D (ReLU) -> D (ReLU) -> 1 */
    samq_linear_ref_v1 prompt_mlp[2];      /* scoring.prompt_mlp: D -> FFN (ReLU) -> D */
    const float *prompt_mlp_norm_w, *prompt_mlp_norm_b;
    samq_linear_ref_v1 prompt_proj, hs_proj;  /* D -> D */
} samq_decoder_v1;

/* enc, enc_pos: device f32 [grid * grid][D] (the fusion output and the image
 * positional encoding); prompt [prompt_tokens][D], prompt_bias [prompt_tokens]
 * (additive key bias), prompt_valid [prompt_tokens] (the scoring pool weights,
 * T / n_valid at valid tokens and 0 at padding, execution.hpp:160-175).
 * Outputs (device): queries_out [queries + 1][D] (the presence query, then the
 * normalized object queries: the mask head's input), boxes [queries][4]
 * (cx, cy, w, h in [0, 1]), scores [queries], presence [1] (raw logit). */
samq_status samq_decoder_forward_v1(const samq_decoder_v1* decoder, const float* enc, const float* enc_pos, int grid,
                                    const float* prompt, const float* prompt_bias, const float* prompt_valid,
                                    int prompt_tokens, float* queries_out, float* boxes, float* scores,
                                    float* presence, void* stream);

/* ---- Geometry encoder (text-only prompt form) ---------------------------------
 * src/models/sam3/prompt_encoder.hpp:44-160, tensor names geom.*
 * (src/models/sam3/tensors.hpp:357-410): the learned CLS token through
 * final_proj and norm, `layers` pre-norm layers (self-attention over the
 * token, cross-attention to the image with keys image + pos, ReLU FFN),
 * encode_norm.  The result is the geometry prompt token appended after the
 * text tokens (src/models/sam3/execution.hpp:157-175). */
typedef struct samq_geometry_layer_v1 {
    samq_linear_ref_v1 sa_in_proj, sa_out_proj, ca_in_proj, ca_out_proj, linear1, linear2;
    const float *norm1_w, *norm1_b, *norm2_w, *norm2_b, *norm3_w, *norm3_b;
} samq_geometry_layer_v1;

typedef struct samq_geometry_encoder_v1 {
    uint32_t version;  /* 1 */
    int32_t heads;     /* 8 */
    int32_t layers;    /* 3 */
    const samq_geometry_layer_v1* layer;  /* [layers], host memory */
    const float* cls_token;               /* geom.cls_embed.weight [D], device */
    samq_linear_ref_v1 final_proj;        /* D -> D */
    const float *norm_w, *norm_b, *encode_norm_w, *encode_norm_b;
} samq_geometry_encoder_v1;

/* image, pos: device f32 [tokens][D] (the 1x neck map and the image positional
 * encoding); out: device f32 [D]. */
samq_status samq_geometry_encoder_forward_v1(const samq_geometry_encoder_v1* encoder, const float* image,
                                             const float* pos, int tokens, float* out, void* stream);

/* ---- Segmentation head ----------------------------------------------------------
 * src/models/sam3/mask_decoder.hpp:57-202, tensor names seg.*
 * (src/models/sam3/tensors.hpp:405-442).  Convolutions are samq_dense handles
 * (CONV, 3x3 for conv[i], 1x1 for instance); products have F32 semantics. */
typedef struct samq_seg_head_v1 {
    uint32_t version;  /* 1 */
    int32_t heads;     /* 8 */
    const float *cross_attn_norm_w, *cross_attn_norm_b;
    samq_linear_ref_v1 ca_in_proj, ca_out_proj;  /* seg.cross_attend_prompt */
    const struct samq_dense* conv[2];            /* seg.pixel_decoder.conv_layers.{0,1} */
    const float* conv_b[2];
    const float* norm_w[2];                      /* seg.pixel_decoder.norms.{0,1} (GroupNorm 8) */
    const float* norm_b[2];
    const struct samq_dense* instance;           /* seg.instance_seg_head (1x1) */
    const float* instance_b;
    samq_linear_ref_v1 mask_embed[3];            /* seg.mask_predictor.mask_embed.layers.{0,1,2} */
} samq_seg_head_v1;

/* enc: the fusion output [grid^2][D]; fpn1 [(2 grid)^2][D], fpn0
 * [(4 grid)^2][D] (the neck's 2x and 4x maps, NHWC); queries [nq][D] (the
 * decoder's object queries); prompt [prompt_tokens][D] with key bias
 * prompt_bias; mask_logits [nq][(4 grid)^2] raw logits.  All device. */
samq_status samq_seg_head_forward_v1(const samq_seg_head_v1* head, const float* enc, int grid, const float* fpn0,
                                     const float* fpn1, const float* queries, int nq, const float* prompt,
                                     const float* prompt_bias, int prompt_tokens, float* mask_logits, void* stream);

/* ---- Quantized linear with GGML MMQ's exact arithmetic -------------------------
 * Y = sum_b d_w[n][b] d_x[m][b] (q_w . q_x)_b + bias over 32-value blocks: the
 * integer block dots exact on the tensor cores, the per-block rescale in f32
 * (GGML CUDA mul_mat_q over Q8_0 weights and MMQ-D4 staged activations,
 * verify_q8_mmq_dots.py:54-105).  No activation range limit beyond finiteness.
 * The codes are held as f16 (tcgen05 kind::f16) or int8 (kind::i8). */
enum { SAMQ_MMQ_CODES_F16 = 0, SAMQ_MMQ_CODES_I8 = 1 };
typedef struct samq_mmq_weights samq_mmq_weights;

/* Q8_0 GGUF rows (n rows of k values, k % 128 == 0) -> device codes + scales. */
samq_status samq_mmq_weights_create_v1(int device, int type, int variant, int64_t k, int64_t n, const void* gguf_rows,
                                       size_t bytes, void* stream, samq_mmq_weights** out);
samq_status samq_mmq_weights_destroy_v1(samq_mmq_weights* weights);
/* x [m][ldx] f32 (device) staged with the MMQ-D4 rule, then the exact GEMM;
 * epilogue SAMQ_EPILOGUE_NONE or _GELU_ERF; y [m][ldy] f32. */
samq_status samq_linear_mmq_v1(const samq_mmq_weights* weights, const float* x, int64_t m, int64_t ldx,
                               const float* bias, int epilogue, float* y, int64_t ldy, void* stream);

/* Host GGUF row quantizer (the role of tools/quantize/quantize_rows.cpp:210,
 * ggml_quantize_chunk): n rows of k f32 values (host) -> n packed rows (host,
 * bytes = n * row bytes).  Q8_0 is the reference converter's quantizer
 * (gguf-py); the K-quants use a min / max encoder per sub-block. */
samq_status samq_quantize_rows_v1(int type, int64_t k, int64_t n, const float* src, void* dst, size_t bytes);

/* The image positional encoding sam3_sinusoidal_pe_2d
 * (src/models/sam3/vision.hpp:39-75), computed on the host in f32 as the
 * reference does: out [h * w][d] host floats. */
samq_status samq_sine_pe_2d_v1(int h, int w, int d, float* out);

/* ---- Dense (F32 / F16) modules with F32 semantics -------------------------
 * The tensors the reference keeps unquantized (neck convolutions, fusion /
 * decoder / mask-head linears in the F32 profiles: "only ViT linear weights
 * are quantized, while text, neck, fusion, detector, mask head, and other
 * tensors remain original F32", tests/data/sam3-vision-quantization-gates.json:8)
 * are multiplied with F32 semantics:
 * ggml_cuda_mul_mat routes F32/F16 weights x F32 activations at GGML_PREC_F32
 * to cuBLAS with CUBLAS_COMPUTE_32F_PEDANTIC (no TF32 narrowing,
 * cmake/patches/ggml-precise-cuda.patch:288-356), and convolutions keep F32
 * im2col columns (src/models/sam3/ops.hpp:67-84).  Here both run on the
 * tcgen05 tensor cores as a three-term TF32 split: each F32 operand x is
 * hi = rna_tf32(x), lo = rna_tf32(x - hi), and hi*hi + hi*lo + lo*hi is
 * accumulated in F32 (relative error ~2^-22 per product, F32 level).  F16
 * weights are promoted exactly.  Layouts are channel-innermost (NHWC, the
 * reference's [C, W, H] tensors): pixel (x, y) of a width x height image with
 * C channels is row y * width + x of a [pixels][C] f32 array. */
enum {
    SAMQ_TYPE_F32 = 0,
    SAMQ_TYPE_F16 = 1
};

enum {
    SAMQ_DENSE_LINEAR = 0,     /* GGML [k, n] matrix: W[n][k] */
    SAMQ_DENSE_CONV = 1,       /* GGML conv kernel [kw, kh, cin, cout], kw == kh in {1, 3}: stride 1, pad kw/2 */
    SAMQ_DENSE_DECONV2X2 = 2   /* GGML ConvTranspose2d kernel [2, 2, cout, cin]: stride 2, no padding */
};

typedef struct samq_dense samq_dense;

/* Uploads HOST weights (`type` F32 or F16, `bytes` = element count x size) in
 * the GGML layout of `kind` and splits them on the device.  kind LINEAR:
 * cin = k, cout = n, kw = kh = 1.  cin % 32 == 0 for CONV and DECONV2X2,
 * cout % 32 == 0 for DECONV2X2, cin % 4 == 0 for LINEAR. */
samq_status samq_dense_create_v1(int device, int type, int kind, int kw, int kh, int64_t cin, int64_t cout,
                                 const void* data, size_t bytes, void* stream, samq_dense** out);
samq_status samq_dense_destroy_v1(samq_dense* weights);

/* Dense calls run on the current device, which must own the handles (else
 * SAMQ_ERR_INVALID_ARGUMENT).
 * Y[m][n] = X[m][k] W[n][k]^T (+ bias[n]) (then erf-GELU), F32 semantics;
 * `weights` of kind LINEAR.  ldx % 4 == 0, ldy % 4 == 0, pointers 16-byte
 * aligned.  Replaces ggml_mul_mat on F32/F16 weights at GGML_PREC_F32. */
samq_status samq_dense_linear_v1(const samq_dense* weights, const float* x, int64_t m, int64_t ldx,
                                 const float* bias, int epilogue, float* y, int64_t ldy, void* stream);

/* Convolution of an NHWC image x [height * width][cin] into y (+ bias[cout],
 * then optional erf-GELU).  CONV: y is [height * width][cout]
 * (sam3_conv_2d_s1_ph / sam3_conv_2d_sk_p0 with a 1x1 kernel,
 * src/models/sam3/ops.hpp:86-94).  DECONV2X2: y is [(2 height) * (2 width)][cout],
 * y(2i + ky, 2j + kx) = sum_c x(i, j)[c] W[c][co][ky][kx] (sam3_deconv_2x2,
 * ops.hpp:96-117). */
samq_status samq_conv2d_v1(const samq_dense* weights, const float* x, int width, int height, const float* bias,
                           int epilogue, float* y, void* stream);

/* 2x2 max pooling with stride 2 of an NHWC image (ggml_pool_2d MAX 2,2,2,2,0,0;
 * output floor(width / 2) x floor(height / 2)); channels % 4 == 0. */
samq_status samq_maxpool2x2_v1(const float* x, int width, int height, int64_t channels, float* y, void* stream);

/* The SimpleFPN neck of one path (src/models/sam3/vision.hpp:307-366), tensor
 * names of src/models/sam3/tensors.hpp:131-160 (E = ViT width, D = 256):
 *   out[0] (4x):   deconv E->mid, +b, GELU, deconv mid->D, +b, conv1x1, +b, conv3x3, +b
 *   out[1] (2x):   deconv E->mid, +b, conv1x1 mid->D, +b, conv3x3, +b
 *   out[2] (1x):   conv1x1 E->D, +b, conv3x3, +b
 *   out[3] (0.5x): maxpool 2x2, conv1x1 E->D, +b, conv3x3, +b
 * with mid = 512 in SAM 3 (any multiple of 32 here). */
typedef struct samq_neck_v1 {
    uint32_t version;  /* 1 */
    const samq_dense* s0_deconv1; const float* s0_deconv1_b;
    const samq_dense* s0_deconv2; const float* s0_deconv2_b;
    const samq_dense* s0_conv1x1; const float* s0_conv1x1_b;
    const samq_dense* s0_conv3x3; const float* s0_conv3x3_b;
    const samq_dense* s1_deconv1; const float* s1_deconv1_b;
    const samq_dense* s1_conv1x1; const float* s1_conv1x1_b;
    const samq_dense* s1_conv3x3; const float* s1_conv3x3_b;
    const samq_dense* s2_conv1x1; const float* s2_conv1x1_b;
    const samq_dense* s2_conv3x3; const float* s2_conv3x3_b;
    const samq_dense* s3_conv1x1; const float* s3_conv1x1_b;
    const samq_dense* s3_conv3x3; const float* s3_conv3x3_b;
} samq_neck_v1;

/* x: the ViT output, device f32 [grid_h * grid_w][E] (raster tokens = NHWC).
 * out[i]: device f32 NHWC [(grid_h * 2^(2-i)) * (grid_w * 2^(2-i))][D]
 * (out[3] is floor(grid / 2) on each side).  Replaces sam3_build_neck_graph. */
samq_status samq_neck_forward_v1(const samq_neck_v1* neck, const float* x, int grid_w, int grid_h,
                                 float* const out[4], void* stream);

/* Counters of a handle.  Mirrors ggml_cuda_sam_q8_rhs_query_v1
 * (cmake/patches/ggml-native-activation.patch:34-42). */
samq_status samq_query_v1(const samq_weights* weights, struct samq_counters_v1* out);

/* Synchronize `stream` and report device-side findings recorded since the
 * last call on `device`: SAMQ_ERR_RANGE for non-finite / out-of-range
 * activations, SAMQ_ERR_TIMEOUT for a bounded wait that gave up.  Clears them.
 * Replaces the reference's post-compute RHS range check
 * (cmake/patches/ggml-native-activation.patch:148-171). */
samq_status samq_check_v1(int device, void* stream);

/* Allocation-free variant of samq_linear_v1 (same arguments; the same result
 * for m > 64, and within the linear tolerance for m <= 64, where
 * samq_linear_v1 streams the packed weights with split-K accumulation).
 * It has no counterpart in the reference.  It serves callers that cannot let a
 * library call cudaMalloc: a framework whose caching allocator already owns the
 * device memory (a library cudaMalloc would fail or fragment its pool), serving
 * loops that cannot absorb cudaMalloc's implicit device synchronization, and
 * hosts that must not meet an out-of-memory error in the middle of a request.
 * The staged activation operand lives in a file-scope device array of
 * SAMQ_STATIC_OPERAND_ELEMENTS f16 values (32 MiB, held by every GPU that loads
 * the library until the process exits) instead of library scratch; the call
 * makes no cudaMalloc, cudaFree or other allocating call.  m * k above
 * SAMQ_STATIC_OPERAND_ELEMENTS is rejected with SAMQ_ERR_INVALID_ARGUMENT
 * (split the rows across calls).  The first call on a device looks up the
 * array's device address once (cudaGetSymbolAddress with that device current);
 * make that first call before any stream capture.  All calls on a device share
 * the array and it keeps the last call's contents (nothing in it needs to start
 * at zero): calls whose GPU work overlaps in time race on it, so order them on
 * one stream.  Range and timeout findings go to a second file-scope device
 * word and are reported by samq_check_v1 like those of samq_linear_v1
 * (samq_check_v1 itself allocates nothing on a device where only this entry
 * point has run). */
#define SAMQ_STATIC_OPERAND_ELEMENTS 16777216
samq_status samq_linear_static_v1(const samq_weights* weights, const float* x, int64_t m, int64_t ldx,
                                  const float* bias, int epilogue, float* y, int64_t ldy, void* stream);

#ifdef __cplusplus
}
#endif
#endif
