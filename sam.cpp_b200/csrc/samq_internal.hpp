// samq_internal.hpp -- host-side internals shared by the samq translation
// units: error reporting, per-device state, scratch memory, tensor maps.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>

#include "samq.h"
#include "samq_device.cuh"

namespace samq {

// Internal exception type; converted to a status at the C boundary.
struct Error {
    samq_status status;
    std::string message;
};

[[noreturn]] void fail(samq_status status, const std::string& message);
void check_cuda(cudaError_t err, const char* what);
void set_last_error(const std::string& message);

// Per-stream scratch buffer, grown on demand (growth is a cudaMalloc and
// therefore synchronizes the device).
struct Scratch {
    void* ptr = nullptr;
    size_t bytes = 0;
};

struct DeviceState {
    int device = -1;
    int sm_count = 0;
    int cc_major = 0, cc_minor = 0;
    DeviceStatus* status = nullptr;  // device memory
    std::mutex mutex;
    std::unordered_map<cudaStream_t, Scratch> scratch;
};

// Checks the device once and returns its state (throws Error otherwise).
// The first call on a device allocates its status word.
DeviceState& device_state(int device);
// The state of `device` if device_state() has created it, else nullptr
// (never allocates).
DeviceState* existing_device_state(int device);
// Argument checks shared by the linear entry points (throw Error).
void check_activation_args(int64_t rows, int64_t k, int64_t ld, const void* x, const void* out);
void check_linear_args(const samq_weights* w, int64_t m, const float* bias, int epilogue, const float* y,
                       int64_t ldy);
// Findings of samq_linear_static_v1 on `device` since the last call (its
// status word is a file-scope device variable, static_scratch.cu); clears
// them.  Returns false, touching nothing, when that path never ran on the
// device.  Makes no allocation.
bool take_static_status(int device, DeviceStatus* out);
// Scratch of at least `bytes` bytes for work ordered on `stream`.
Scratch& scratch_for(DeviceState& state, cudaStream_t stream, size_t bytes);
// Raises `kernel`'s dynamic shared memory limit to `bytes` on state.device the
// first time it is asked for there (thread-safe; later calls return at once).
void set_smem_limit_once(DeviceState& state, const void* kernel, int bytes, const char* what);


// RAII device switch.
struct DeviceGuard {
    int previous = -1;
    explicit DeviceGuard(int device);
    ~DeviceGuard();
};

// Launch `kernel` on `stream` with programmatic stream serialization (the
// kernel must call pdl_wait() before touching dependent memory).
template <class... KernelArgs, class... Args>
void launch_pdl(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                const char* what, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    check_cuda(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...), what);
}

// launch_pdl for a kernel of CTA pairs: clusters of two CTAs along x.
template <class... KernelArgs, class... Args>
void launch_pdl_pairs(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      const char* what, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    check_cuda(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...), what);
}

// How many clusters of two CTAs of `kernel` (block threads, smem bytes of
// dynamic shared memory) can be resident on state.device at once; queried
// once per (kernel, device) and cached.
int pair_clusters_resident(DeviceState& state, const void* kernel, int threads, int smem, const char* what);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on libcuda).
void encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                          uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                          CUtensorMapSwizzle swizzle);
void encode_tensor_map_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t d0, uint64_t d1,
                          uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1,
                          CUtensorMapSwizzle swizzle);
// 3-D map whose box spans box2 planes (encode_tensor_map_3d takes one).
void encode_tensor_map_3d_box(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t d0,
                              uint64_t d1, uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                              uint32_t box1, uint32_t box2, CUtensorMapSwizzle swizzle);

}  // namespace samq

// Weight handle (opaque in the C ABI).
struct samq_weights {
    int device = -1;
    int type = 0;
    int64_t k = 0, n = 0;
    void* packets = nullptr;      // K4 packet layout (canonical device form)
    size_t packet_bytes = 0;
    __half* operand = nullptr;    // f16 [n][k] tensor-core B operand expanded from the packets
    size_t operand_bytes = 0;
    std::atomic<uint64_t> launches{0};
    std::atomic<uint64_t> payload_bytes{0};
    std::atomic<uint64_t> allocation_bytes{0};
};

// Dense (F32 / F16) weights: the GEMM operand B = W split into TF32 hi / lo
// (dense.cu).
struct samq_dense {
    int device = -1;
    int type = 0, kind = 0, ks = 1;  // SAMQ_TYPE_F32 / F16, SAMQ_DENSE_*, kernel size
    int64_t cin = 0, cout = 0;
    int64_t n = 0, k = 0;            // B is [n][k]: n = cout (x 4 for DECONV2X2), k = cin (x ks^2 for CONV)
    float* hi = nullptr;
    float* lo = nullptr;
};

// Weights of the exact MMQ path: codes [n][k] (f16 or int8), scales [k / 32][n].
struct samq_mmq_weights {
    int device = -1;
    int variant = 0;
    int64_t k = 0, n = 0;
    void* codes = nullptr;
    float* scales = nullptr;
};

// ---- launchers implemented in the .cu files -------------------------------
namespace samq {

// K1 quantize.cu
void launch_act_f16(const float* x, int64_t rows, int64_t k, int64_t ld, __half* a_out, uint8_t* q8_1_out,
                    DeviceStatus* status, cudaStream_t stream);
void launch_q8_1_to_f16(const uint8_t* q8_1, int64_t rows, int64_t k, __half* a_out, DeviceStatus* status,
                        cudaStream_t stream);
void launch_mmq_d4(const float* x, int64_t rows, int64_t k, int64_t ld, uint8_t* out, cudaStream_t stream);

// K4 repack.cu
int64_t packet_code_bytes(int type);
int64_t packet_bytes(int type);
int64_t row_bytes(int type, int64_t k);
// rows.cu: host GGUF row quantizer (Q8_0 as gguf-py; K-quants min / max).
void quantize_rows(int type, int64_t k, int64_t n, const float* src, uint8_t* out);
void launch_gguf_to_packets(int type, int64_t k, int64_t n, const uint8_t* rows, uint8_t* packets,
                            uint32_t* bad_scales, cudaStream_t stream);
void launch_packets_to_gguf(int type, int64_t k, int64_t n, const uint8_t* packets, uint8_t* rows,
                            cudaStream_t stream);
void launch_packets_to_f16(int type, int64_t k, int64_t n, const uint8_t* packets, __half* out,
                           cudaStream_t stream);

// K3 attention.cu: RoPE + windowed/global attention of one ViT block.
// qkv [tokens][ldq] f32 (Q | K | V), out [tokens][ldo] f32; `packed` is
// scratch of attention_scratch_bytes() bytes.
size_t attention_scratch_bytes(int grid_w, int grid_h, int heads);
void launch_vit_attention(const float* qkv, int64_t ldq, int grid_w, int grid_h, int heads, int window,
                          const float* freqs, float* out, int64_t ldo, void* packed, DeviceState& state,
                          cudaStream_t stream);
// Attention over already packed f16 inputs (Q x 1/8 and K RoPE'd,
// [group * heads + head][group_n][64]; V^T [group * heads + head][64][group_n]),
// output in raster token order: f32 `out`, or, when out_h is given, the
// Q8_1-staged f16 operand of the proj linear.
// `batch` images of grid_w x grid_h tokens each, stored image after image.
void launch_attention_packed(const __half* q, const __half* k, const __half* vt, int grid_w, int grid_h, int heads,
                             int window, int batch, float* out, __half* out_h, int64_t ldo, DeviceState& state,
                             cudaStream_t stream);

// attention_f32.cu: F32-precise RoPE + attention (CudaComputeMode::F32).
// qkv [rows][ldq] f32 (Q | K | V); rows are window-major (g * group_n + n)
// when qkv_window_major, else raster.  Output f32 raster `out`, or (out_h) the
// proj linear's Q8_1-staged f16 operand, [tokens][ldo].
void launch_attention_f32(const float* qkv, int64_t ldq, bool qkv_window_major, int grid_w, int grid_h, int heads,
                          int window, int batch, const float* freqs, float* out, __half* out_h, int64_t ldo,
                          DeviceState& state, cudaStream_t stream);
// General F32 attention (attention_f32.cu): Q [lq][ldq], K / V [lk][ld],
// head h at columns h*head_dim (head_dim 32 or 64), additive bias
// bias[h*bias_h + q*bias_q + k] (nullable), causal mask, out [lq][ldo].
// With few query tiles and many keys the keys are split over CTAs when the
// caller provides `partials` of attention_partial_floats(...) floats.
size_t attention_partial_floats(int lq, int lk, int heads, int head_dim, int causal, int sms);
// attention_tc.cu: the same attention on the tensor cores (three-term TF32),
// for many queries and keys without a mask.
bool attention_tc_eligible(int lq, int lk, int head_dim, int causal, const float* bias, const float* out,
                           int64_t ldo);
// `scratch` (attention_tc_scratch_bytes, 256-byte aligned; nullptr: the
// loader-fed kernel over all keys) holds the K / V^T TF32 planes and the
// key-split partials merged by launch_attention_combine.
size_t attention_tc_scratch_bytes(int lq, int lk, int heads, int head_dim);
void launch_attention_tc(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                         int lq, int lk, int heads, int head_dim, float scale, float* out, int64_t ldo, float* scratch,
                         DeviceState& state, cudaStream_t stream);
// Grouped form for the ViT: qkv rows [groups * group_n][ldq] (Q, K, V at
// column 0, embed, 2 embed), one attention per group; output rows in raster
// token order when out_window > 0 (windows of a grid out_grid_w wide).  With
// `planes` (attention_tc_plane_bytes of device memory, 16-byte aligned) and
// group_n % 4 == 0, K and V^T are first split into TF32 hi / lo planes there
// and the kernel loads them by TMA; otherwise its loader warps split the rows.
size_t attention_tc_plane_bytes(int groups, int group_n, int heads, int head_dim);
void launch_attention_tc_groups(const float* qkv, int64_t ldq, int64_t embed, int groups, int group_n, int heads,
                                int head_dim, float scale, float* out, int64_t ldo, int out_window, int out_grid_w,
                                float* planes, DeviceState& state, cudaStream_t stream);
// RoPE (GGML rounding) in place on the Q and K columns of f32 qkv rows, token
// position r % group_n.
void launch_rope_rows(float* qkv, int64_t ldq, int64_t embed, int64_t rows, int group_n, const float* freqs,
                      cudaStream_t stream);
void launch_attention_gen(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                          int lq, int lk, int heads, int head_dim, float scale, int causal, const float* bias,
                          int64_t bias_h, int64_t bias_q, float* out, int64_t ldo, DeviceState& state,
                          cudaStream_t stream, float* partials = nullptr, size_t partial_floats = 0,
                          float* tc_planes = nullptr);
// Merge of key-split partials [splits][heads][lq][head_dim + 2] (unnormalized
// O, the row maximum in natural-log units, the row sum) into out rows.
void launch_attention_combine(const float* part, int splits, int heads, int lq, int head_dim, float* out,
                              int64_t ldo, cudaStream_t stream);
// Scratch a launch_attention_gen caller may pass as `tc_planes`: the K / V^T
// TF32 planes of the tensor-core path when the shape takes it (plus the
// key-split partials it may use), else 0.
size_t attention_gen_plane_bytes(int lq, int lk, int heads, int head_dim, int causal, const float* bias,
                                 const float* out, int64_t ldo);
// sam3_apply_rope on [head_batches][tokens][64] f32 with GGML's rounding.
void launch_rope_f32(const float* x, const float* freqs, int64_t tokens, int64_t head_batches, float* out,
                     cudaStream_t stream);

// K2 gemm.cu
// What the GEMM epilogue writes.  Rows of the output are rows of A.
enum OutMode : int {
    kOutF32 = 0,          // y = act(acc + bias), f32 [m][ldy]
    kOutF32Residual = 1,  // y = residual + (acc + bias), f32 (y may alias residual)
    kOutF16Staged = 2,    // h = Q8_1 operand of act(acc + bias), f16 [m][ldh] (n % 32 == 0)
    kOutQkvPack = 3,      // acc + bias split into RoPE'd f16 Q (x 1/8), K and V^T (attention layout)
};
struct Epilogue {
    int mode = kOutF32;
    int gelu = 0;                   // erf-GELU after the bias
    const float* bias = nullptr;    // [n] or null
    float* y = nullptr;             // kOutF32 / kOutF32Residual
    int64_t ldy = 0;
    const float* residual = nullptr;
    int64_t ldr = 0;
    __half* h = nullptr;            // kOutF16Staged
    int64_t ldh = 0;
    // kOutQkvPack: A rows are window-major (row = group * group_n + n), the
    // columns Q | K | V with heads of 64 channels; Q, K are
    // [group * heads + head][group_n][64], V^T is [group * heads + head][64][group_n].
    __half* q = nullptr;
    __half* k = nullptr;
    __half* vt = nullptr;
    const float* freqs = nullptr;   // [group_n][32][2] (cos, sin) of position n
    int heads = 0, group_n = 0;
};
void launch_gemm(const __half* a, int64_t lda, const __half* b, int64_t m, int64_t n, int64_t k, const Epilogue& ep,
                 DeviceState& state, cudaStream_t stream);
// f32 output with bias and optional erf-GELU (epilogue = SAMQ_EPILOGUE_*).
void launch_gemm_f16(const __half* a, int64_t lda, const __half* b, int64_t m, int64_t n, int64_t k,
                     const float* bias, int epilogue, float* y, int64_t ldy, DeviceState& state,
                     cudaStream_t stream);


// stream.cu: small-M linears streaming the K4 packets (dequant in the producer).
constexpr int kStreamMaxRows = 64;
bool stream_eligible(const samq_weights* w, int64_t m);
// Bytes of f32 split-K partial sums the streaming path needs (0 when unsplit).
size_t stream_partial_bytes(const samq_weights* w, int64_t m, int sms);
void launch_linear_stream(const samq_weights* w, const __half* x16, int64_t ldx, int64_t m, const float* bias,
                          int epilogue, float* y, int64_t ldy, float* partials, DeviceState& state,
                          cudaStream_t stream);

// vit.cu: the ViT block / backbone prefix around K2 and K3.
struct VitBlockArgs {
    int window = 0;
    int compute = SAMQ_COMPUTE_F16;  // SAMQ_COMPUTE_F32: f32 qkv and F32-precise attention
    const float *norm1_w = nullptr, *norm1_b = nullptr, *norm2_w = nullptr, *norm2_b = nullptr;
    const samq_weights *qkv = nullptr, *proj = nullptr, *fc1 = nullptr, *fc2 = nullptr;
    const float *qkv_b = nullptr, *proj_b = nullptr, *fc1_b = nullptr, *fc2_b = nullptr;
    const float* freqs = nullptr;
};
size_t vit_block_scratch_bytes(int64_t tokens, int64_t embed, int64_t mlp, int compute);
// x: `batch` images of grid_w x grid_h tokens, image after image.
void launch_vit_block(const VitBlockArgs& blk, float* x, int batch, int grid_w, int grid_h, void* scratch,
                      DeviceState& state, cudaStream_t stream);
void launch_ln_stage(const float* x, int64_t rows, int64_t embed, int grid_w, int window, const float* w,
                     const float* b, __half* a, DeviceState& state, cudaStream_t stream);
size_t vit_prefix_scratch_bytes(int64_t tokens, int64_t embed, int patch, int compute);
void launch_vit_prefix(const float* image, int width, int height, int patch, const float* patch_w, int64_t embed,
                       const float* pos, int pos_grid, const float* ln_w, const float* ln_b, float* x, int compute,
                       void* scratch, DeviceState& state, cudaStream_t stream);

// text.cu: the text encoder's pieces.
struct TextBlockArgs {
    const float *norm1_w = nullptr, *norm1_b = nullptr, *norm2_w = nullptr, *norm2_b = nullptr;
    const samq_weights *in_proj = nullptr, *out_proj = nullptr, *fc1 = nullptr, *fc2 = nullptr;
    const float *in_proj_b = nullptr, *out_proj_b = nullptr, *fc1_b = nullptr, *fc2_b = nullptr;
};
size_t text_block_scratch_bytes(const TextBlockArgs& blk, int64_t tokens, int sms);
void launch_text_block(const TextBlockArgs& blk, float* x, int64_t tokens, void* scratch, DeviceState& state,
                       cudaStream_t stream);
void launch_layer_norm_f32(const float* x, int64_t rows, int width, int64_t ldx, const float* w, const float* b,
                           float* out, int64_t ldo, float eps, cudaStream_t stream);
void launch_add_rows(float* x, int64_t ldx, const float* y, int64_t ldy, int64_t rows, int width, cudaStream_t stream);
void launch_embed_rows(const float* table, const int32_t* ids, const float* pos, int count, int width, float* out,
                       cudaStream_t stream);
void linear_from_staged(const samq_weights* w, const __half* a, int64_t lda, int64_t m, const float* bias,
                        int epilogue, float* y, int64_t ldy, float* partials, DeviceState& state,
                        cudaStream_t stream);

// fusion.cu: fusion-encoder layer and the linear helper of the F32 modules.
void launch_add2(const float* a, const float* b, float* out, int64_t rows, int width, cudaStream_t stream);
void launch_relu(float* x, int64_t count, cudaStream_t stream);
int64_t linear_in(const samq_linear_ref_v1& l);
int64_t linear_out(const samq_linear_ref_v1& l);
size_t linear_scratch_bytes(const samq_linear_ref_v1& l, int64_t m, int sms);
void apply_linear(const samq_linear_ref_v1& l, int64_t row0, int64_t rows, const float* x, int64_t ldx, int64_t m,
                  int epilogue, float* y, int64_t ldy, void* scratch, DeviceState& state, cudaStream_t stream);
size_t fusion_layer_scratch_bytes(const samq_fusion_layer_v1& ly, int64_t tokens, int64_t prompt_tokens, int sms);
void launch_fusion_layer(const samq_fusion_layer_v1& ly, float* x, const float* pos, int64_t tokens,
                         const float* prompt, const float* prompt_bias, int64_t prompt_tokens, void* scratch,
                         DeviceState& state, cudaStream_t stream);

// decoder.cu: the DETR decoder, scoring and presence head.
size_t decoder_scratch_bytes(const samq_decoder_v1& dec, int64_t enc_tokens, int64_t prompt_tokens, int grid, int sms);
void launch_decoder(const samq_decoder_v1& dec, const float* enc, const float* enc_pos, int64_t enc_tokens, int grid,
                    const float* prompt, const float* prompt_bias, const float* prompt_valid, int64_t prompt_tokens,
                    float* queries_out, float* boxes, float* scores, float* presence, void* scratch,
                    DeviceState& state, cudaStream_t stream);

// gemm_mmq.cu: quantized linear with GGML MMQ's exact arithmetic.
size_t mmq_code_bytes(int variant);
void launch_mmq_weights(int variant, const uint8_t* rows, int64_t n, int64_t k, void* codes, float* scales,
                        cudaStream_t stream);
void launch_mmq_stage(int variant, const float* x, int64_t rows, int64_t k, int64_t ld, void* codes, float* scales,
                      DeviceStatus* status, cudaStream_t stream);
void launch_mmq_gemm(int variant, const void* a_codes, const float* dx, const void* b_codes, const float* dw,
                     int64_t m, int64_t n, int64_t k, const float* bias, int gelu, float* y, int64_t ldy,
                     DeviceState& state, cudaStream_t stream);

// seg.cu: the segmentation head and the geometry encoder.
size_t seg_head_scratch_bytes(const samq_seg_head_v1& sh, int grid, int64_t queries, int64_t prompt_tokens, int sms);
void launch_seg_head(const samq_seg_head_v1& sh, const float* enc, int grid, const float* fpn0, const float* fpn1,
                     const float* queries, int64_t nq, const float* prompt, const float* prompt_bias,
                     int64_t prompt_tokens, float* logits, void* scratch, DeviceState& state, cudaStream_t stream);
size_t geometry_scratch_bytes(const samq_geometry_encoder_v1& ge, int64_t tokens, int sms);
void launch_geometry_encoder(const samq_geometry_encoder_v1& ge, const float* image, const float* pos, int64_t tokens,
                             float* out, void* scratch, DeviceState& state, cudaStream_t stream);

// dense.cu: F32-semantics linears / convolutions (three-term TF32 split).
void launch_dense_prep(const void* src, int type, int kind, int ks, int64_t cin, int64_t cout, int64_t n, int64_t k,
                       float* hi, float* lo, DeviceState& state, cudaStream_t stream);
// x [rows][ld] -> hi / lo [rows][k].
void launch_split_rows(const float* x, int64_t rows, int64_t k, int64_t ld, float* hi, float* lo, DeviceState& state,
                       cudaStream_t stream);
// y (and lo != nullptr: the hi / lo split) = 2x2 max pooling of NHWC x.
void launch_maxpool2x2(const float* x, int width, int height, int64_t channels, float* y, float* lo,
                       DeviceState& state, cudaStream_t stream);
// A = split activations: [m][k] rows (LINEAR, 1x1 CONV, DECONV2X2 with
// conv_width = input width) or an NHWC image conv_width x conv_height (CONV);
// output f32 (y_lo == nullptr) or split, [rows][ldy].
void launch_dense_gemm(const float* a_hi, const float* a_lo, const samq_dense& w, int64_t m, int conv_width,
                       int conv_height, const float* bias, int gelu, float* y, float* y_lo, int64_t ldy,
                       DeviceState& state, cudaStream_t stream);
size_t neck_scratch_bytes(const samq_neck_v1& neck, int grid_w, int grid_h);
void launch_neck(const samq_neck_v1& neck, const float* x, int grid_w, int grid_h, float* const out[4], void* scratch,
                 DeviceState& state, cudaStream_t stream);

}  // namespace samq
