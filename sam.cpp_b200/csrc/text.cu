// text.cu -- the SAM 3 text encoder on the device: token embedding, 24
// pre-LN transformer blocks with a causal mask, the final LayerNorm (the
// 1024 -> 256 resizer is a plain quantized linear).
//
// Graph (src/models/sam3/text_encoder.hpp:68-180):
//   x = token_embed[ids] + pos_embed
//   per block: x = x + out_proj(attn_causal(in_proj(LN1(x))))
//              x = x + fc2(GELU_erf(fc1(LN2(x))))
//   features = resizer(LN_final(x))
// The quantized linears stage their inputs to Q8_1 exactly as the ViT path
// does (the LayerNorm kernel emits the staged operand directly; the attention
// output and the GELU output go through K1); at M = 32 tokens they stream the
// packed weights (gemm_stream_kernel).  The causal attention is the general
// F32 attention (the reference keeps masked attention at GGML_PREC_F32 in both
// compute modes, src/runtime/ggml/backends/cuda.hpp:86-91).
#include "samq_internal.hpp"

namespace samq {
namespace {

unsigned blocks_of(int64_t work) { return static_cast<unsigned>(std::max<int64_t>(1, (work + 255) / 256)); }

// ggml_norm (eps 1e-5) then * w + b over rows of `width` f32 values, one warp
// per row: mean, centred variance, 1/sqrt(var + eps) as in ggml_compute_forward_norm.
__global__ void __launch_bounds__(256) layer_norm_f32_kernel(const float* __restrict__ x, int64_t rows, int width,
                                                             int64_t ldx, const float* __restrict__ w,
                                                             const float* __restrict__ b, float* __restrict__ out,
                                                             int64_t ldo, float eps) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (r >= rows) return;
    const float* row = x + r * ldx;
    float sum = 0.0f;
    for (int c = lane; c < width; c += 32) sum += row[c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum / static_cast<float>(width);
    float var = 0.0f;
    for (int c = lane; c < width; c += 32) {
        const float d = row[c] - mean;
        var = fmaf(d, d, var);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
    const float inv = 1.0f / sqrtf(var / static_cast<float>(width) + eps);
    float* dst = out + r * ldo;
    for (int c = lane; c < width; c += 32) {
        const float v = (row[c] - mean) * inv * w[c];
        dst[c] = b ? v + b[c] : v;
    }
}

// x += y (the residual adds, ggml_add in f32).
__global__ void __launch_bounds__(256) add_rows_kernel(float* __restrict__ x, int64_t ldx,
                                                       const float* __restrict__ y, int64_t ldy, int64_t rows,
                                                       int width) {
    pdl_wait();
    pdl_trigger();
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= rows * width) return;
    const int64_t r = idx / width, c = idx - r * width;
    x[r * ldx + c] += y[r * ldy + c];
}

// out[i] = table[ids[i]] + pos[i] (ggml_get_rows then ggml_add).
__global__ void __launch_bounds__(256) embed_rows_kernel(const float* __restrict__ table, const int32_t* __restrict__ ids,
                                                         const float* __restrict__ pos, int count, int width,
                                                         float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<int64_t>(count) * width) return;
    const int64_t i = idx / width, c = idx - i * width;
    const float v = table[static_cast<int64_t>(ids[i]) * width + c];
    out[idx] = pos ? v + pos[idx] : v;
}

}  // namespace

void launch_layer_norm_f32(const float* x, int64_t rows, int width, int64_t ldx, const float* w, const float* b,
                           float* out, int64_t ldo, float eps, cudaStream_t stream) {
    if (rows == 0) return;
    launch_pdl(layer_norm_f32_kernel, dim3(blocks_of(rows * 32)), dim3(256), 0, stream, "layer_norm_f32_kernel launch",
               x, rows, width, ldx, w, b, out, ldo, eps);
}

void launch_add_rows(float* x, int64_t ldx, const float* y, int64_t ldy, int64_t rows, int width,
                     cudaStream_t stream) {
    if (rows == 0) return;
    launch_pdl(add_rows_kernel, dim3(blocks_of(rows * width)), dim3(256), 0, stream, "add_rows_kernel launch", x, ldx,
               y, ldy, rows, width);
}

void launch_embed_rows(const float* table, const int32_t* ids, const float* pos, int count, int width, float* out,
                       cudaStream_t stream) {
    if (count == 0) return;
    launch_pdl(embed_rows_kernel, dim3(blocks_of(int64_t(count) * width)), dim3(256), 0, stream,
               "embed_rows_kernel launch", table, ids, pos, count, width, out);
}

// A quantized linear over an already staged f16 operand: packet streaming for
// M <= 64, the tcgen05 GEMM otherwise (the routing of samq_linear_v1).
void linear_from_staged(const samq_weights* w, const __half* a, int64_t lda, int64_t m, const float* bias,
                        int epilogue, float* y, int64_t ldy, float* partials, DeviceState& state,
                        cudaStream_t stream) {
    if (stream_eligible(w, m))
        launch_linear_stream(w, a, lda, m, bias, epilogue, y, ldy, partials, state, stream);
    else
        launch_gemm_f16(a, lda, w->operand, m, w->n, w->k, bias, epilogue, y, ldy, state, stream);
}

size_t text_block_scratch_bytes(const TextBlockArgs& blk, int64_t tokens, int sms) {
    const int64_t E = blk.in_proj->k, mlp = blk.fc1->n;
    size_t partial = 0;
    for (const samq_weights* w : {blk.in_proj, blk.out_proj, blk.fc1, blk.fc2})
        if (stream_eligible(w, tokens)) partial = std::max(partial, stream_partial_bytes(w, tokens, sms));
    // staged operand [T][MLP] f16, qkv [T][3E], attention [T][E], linear output [T][MLP] f32, partials
    return static_cast<size_t>(tokens) * (mlp * 2 + (3 * E + E + mlp) * 4) + partial + 5 * 256;
}

void launch_text_block(const TextBlockArgs& blk, float* x, int64_t tokens, void* scratch, DeviceState& state,
                       cudaStream_t stream) {
    const int64_t E = blk.in_proj->k, mlp = blk.fc1->n;
    const int heads = static_cast<int>(E / 64);
    auto align = [](uintptr_t p) { return (p + 255) & ~uintptr_t(255); };
    uintptr_t cursor = align(reinterpret_cast<uintptr_t>(scratch));
    auto take = [&](size_t bytes) {
        void* p = reinterpret_cast<void*>(cursor);
        cursor = align(cursor + bytes);
        return p;
    };
    __half* a = static_cast<__half*>(take(tokens * mlp * sizeof(__half)));
    float* qkv = static_cast<float*>(take(tokens * 3 * E * sizeof(float)));
    float* att = static_cast<float*>(take(tokens * E * sizeof(float)));
    float* y = static_cast<float*>(take(tokens * mlp * sizeof(float)));
    float* partials = static_cast<float*>(take(0));

    launch_ln_stage(x, tokens, E, static_cast<int>(tokens), 0, blk.norm1_w, blk.norm1_b, a, state, stream);
    linear_from_staged(blk.in_proj, a, E, tokens, blk.in_proj_b, SAMQ_EPILOGUE_NONE, qkv, 3 * E, partials, state,
                       stream);
    launch_attention_gen(qkv, 3 * E, qkv + E, 3 * E, qkv + 2 * E, 3 * E, static_cast<int>(tokens),
                         static_cast<int>(tokens), heads, 64, 0.125f, 1, nullptr, 0, 0, att, E, state, stream);
    launch_act_f16(att, tokens, E, E, a, nullptr, state.status, stream);
    linear_from_staged(blk.out_proj, a, E, tokens, blk.out_proj_b, SAMQ_EPILOGUE_NONE, y, E, partials, state, stream);
    launch_add_rows(x, E, y, E, tokens, static_cast<int>(E), stream);
    launch_ln_stage(x, tokens, E, static_cast<int>(tokens), 0, blk.norm2_w, blk.norm2_b, a, state, stream);
    linear_from_staged(blk.fc1, a, E, tokens, blk.fc1_b, SAMQ_EPILOGUE_GELU_ERF, y, mlp, partials, state, stream);
    launch_act_f16(y, tokens, mlp, mlp, a, nullptr, state.status, stream);
    linear_from_staged(blk.fc2, a, mlp, tokens, blk.fc2_b, SAMQ_EPILOGUE_NONE, y, E, partials, state, stream);
    launch_add_rows(x, E, y, E, tokens, static_cast<int>(E), stream);
}

}  // namespace samq
