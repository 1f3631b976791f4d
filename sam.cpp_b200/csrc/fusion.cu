// fusion.cu -- one SAM 3 fusion-encoder layer (src/models/sam3/fusion_encoder.hpp:38-150)
// on the device:
//   x = x + sa_out(attn(Q = Wq (LN1(x) + pos), K = Wk (LN1(x) + pos), V = Wv LN1(x)))
//   x = x + ca_out(attn(Q = Wq LN2(x), K = Wk prompt, V = Wv prompt; + prompt key bias))
//   x = x + linear2(ReLU(linear1(LN3(x))))
// The fused in-projections are used as row slices (Q | K | V rows), as the
// reference's ggml_view_2d of in_proj_weight does.  Every linear is either a
// quantized handle (Q8_1-staged input, tcgen05 GEMM: the full-linear Q8_0
// profiles) or a dense F32 / F16 handle (F32 semantics, three-term TF32
// split: the mixed profile's fusion=f32).  Attention is the general F32
// attention (head dim 32: the reference keeps head-32 attention precise in
// both compute modes, src/runtime/ggml/backends/cuda.hpp:86-91).
#include <cmath>

#include "samq_internal.hpp"

namespace samq {
namespace {

unsigned blocks_of(int64_t work) { return static_cast<unsigned>(std::max<int64_t>(1, (work + 255) / 256)); }

// out = a + b over rows of `width` (out may alias a).
__global__ void __launch_bounds__(256) add2_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                                   float* __restrict__ out, int64_t rows, int width) {
    pdl_wait();
    pdl_trigger();
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= rows * width) return;
    out[idx] = a[idx] + b[idx];
}

// ggml_relu in place.
__global__ void __launch_bounds__(256) relu_kernel(float* __restrict__ x, int64_t count) {
    pdl_wait();
    pdl_trigger();
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= count) return;
    x[idx] = fmaxf(x[idx], 0.0f);
}

}  // namespace

void launch_add2(const float* a, const float* b, float* out, int64_t rows, int width, cudaStream_t stream) {
    if (rows == 0) return;
    launch_pdl(add2_kernel, dim3(blocks_of(rows * width)), dim3(256), 0, stream, "add2_kernel launch", a, b, out, rows,
               width);
}

void launch_relu(float* x, int64_t count, cudaStream_t stream) {
    if (count == 0) return;
    launch_pdl(relu_kernel, dim3(blocks_of(count)), dim3(256), 0, stream, "relu_kernel launch", x, count);
}

int64_t linear_in(const samq_linear_ref_v1& l) { return l.quantized ? l.quantized->k : l.dense->k; }
int64_t linear_out(const samq_linear_ref_v1& l) { return l.quantized ? l.quantized->n : l.dense->n; }

// Bytes of scratch apply_linear needs for m rows of width k.
size_t linear_scratch_bytes(const samq_linear_ref_v1& l, int64_t m, int sms) {
    const int64_t k = linear_in(l);
    if (l.quantized) {
        size_t partial = stream_eligible(l.quantized, m) ? stream_partial_bytes(l.quantized, m, sms) : 0;
        return static_cast<size_t>(m * k) * sizeof(__half) + partial + 512;
    }
    return 2 * static_cast<size_t>(m * k) * sizeof(float) + 512;
}

// y[m][ldy] = act(x[m][ldx] W[row0 : row0 + rows]^T + bias[row0 : ...]), act
// none or erf-GELU (ReLU is applied by the caller).  row0 % 128 == 0.
void apply_linear(const samq_linear_ref_v1& l, int64_t row0, int64_t rows, const float* x, int64_t ldx, int64_t m,
                  int epilogue, float* y, int64_t ldy, void* scratch, DeviceState& state, cudaStream_t stream) {
    if (m == 0) return;
    const float* bias = l.bias ? l.bias + row0 : nullptr;
    auto align = [](uintptr_t p) { return (p + 255) & ~uintptr_t(255); };
    const uintptr_t base = align(reinterpret_cast<uintptr_t>(scratch));
    if (l.quantized) {
        const samq_weights& w = *l.quantized;
        samq_weights view;
        view.device = w.device;
        view.type = w.type;
        view.k = w.k;
        view.n = rows;
        view.operand = w.operand + row0 * w.k;
        view.packets = static_cast<uint8_t*>(w.packets) + (row0 / 128) * ((w.k + 63) / 64) * packet_bytes(w.type);
        __half* a = reinterpret_cast<__half*>(base);
        float* partials = reinterpret_cast<float*>(align(base + static_cast<size_t>(m * w.k) * sizeof(__half)));
        launch_act_f16(x, m, w.k, ldx, a, nullptr, state.status, stream);
        linear_from_staged(&view, a, w.k, m, bias, epilogue, y, ldy, partials, state, stream);
        return;
    }
    const samq_dense& w = *l.dense;
    samq_dense view = w;
    view.n = rows;
    view.cout = rows;
    view.hi = w.hi + row0 * w.k;
    view.lo = w.lo + row0 * w.k;
    float* xh = reinterpret_cast<float*>(base);
    float* xl = reinterpret_cast<float*>(align(base + static_cast<size_t>(m * w.k) * sizeof(float)));
    launch_split_rows(x, m, w.k, ldx, xh, xl, state, stream);
    launch_dense_gemm(xh, xl, view, m, 0, 0, bias, epilogue == SAMQ_EPILOGUE_GELU_ERF ? 1 : 0, y, nullptr, ldy, state,
                      stream);
    view.hi = view.lo = nullptr;  // a view, not owned
}

size_t fusion_layer_scratch_bytes(const samq_fusion_layer_v1& ly, int64_t tokens, int64_t prompt_tokens, int sms) {
    const int64_t D = linear_in(ly.sa_in_proj), F = linear_out(ly.linear1);
    size_t linear = 0;
    for (const samq_linear_ref_v1* l : {&ly.sa_in_proj, &ly.sa_out_proj, &ly.ca_in_proj, &ly.ca_out_proj, &ly.linear1})
        linear = std::max(linear, linear_scratch_bytes(*l, tokens, sms));
    linear = std::max(linear, linear_scratch_bytes(ly.linear2, tokens, sms));
    linear = std::max(linear, linear_scratch_bytes(ly.ca_in_proj, prompt_tokens, sms));
    // h, qk_in [T][D]; q|k [T][2D]; v, att, y [T][D]; ffn [T][F]; prompt k|v [P][2D];
    // the self-attention's tensor-core scratch (K / V^T TF32 planes, key-split partials)
    const size_t floats = static_cast<size_t>(tokens) * (D * 2 + 2 * D + 3 * D + F) + prompt_tokens * 2 * D;
    return floats * sizeof(float) + attention_tc_scratch_bytes(static_cast<int>(tokens), static_cast<int>(tokens), ly.heads,
                                                               static_cast<int>(D / ly.heads)) +
           linear + 16 * 256;
}

void launch_fusion_layer(const samq_fusion_layer_v1& ly, float* x, const float* pos, int64_t tokens,
                         const float* prompt, const float* prompt_bias, int64_t prompt_tokens, void* scratch,
                         DeviceState& state, cudaStream_t stream) {
    const int64_t D = linear_in(ly.sa_in_proj), F = linear_out(ly.linear1);
    const int heads = ly.heads, hd = static_cast<int>(D / ly.heads);
    const float scale = 1.0f / sqrtf(static_cast<float>(hd));
    auto align = [](uintptr_t p) { return (p + 255) & ~uintptr_t(255); };
    uintptr_t cursor = align(reinterpret_cast<uintptr_t>(scratch));
    auto take = [&](int64_t floats) {
        float* p = reinterpret_cast<float*>(cursor);
        cursor = align(cursor + static_cast<size_t>(floats) * sizeof(float));
        return p;
    };
    float* h = take(tokens * D);
    float* qk_in = take(tokens * D);
    float* qk = take(tokens * 2 * D);
    float* v = take(tokens * D);
    float* att = take(tokens * D);
    float* y = take(tokens * D);
    float* ffn = take(tokens * F);
    float* pkv = take(prompt_tokens * 2 * D);
    float* planes = take(static_cast<int64_t>(
        attention_tc_scratch_bytes(static_cast<int>(tokens), static_cast<int>(tokens), heads, hd) / sizeof(float)));
    void* lin = reinterpret_cast<void*>(cursor);

    // Self-attention: positions added to the queries' and keys' input only.
    launch_layer_norm_f32(x, tokens, static_cast<int>(D), D, ly.norm1_w, ly.norm1_b, h, D, 1e-5f, stream);
    launch_add2(h, pos, qk_in, tokens, static_cast<int>(D), stream);
    apply_linear(ly.sa_in_proj, 0, 2 * D, qk_in, D, tokens, SAMQ_EPILOGUE_NONE, qk, 2 * D, lin, state, stream);
    apply_linear(ly.sa_in_proj, 2 * D, D, h, D, tokens, SAMQ_EPILOGUE_NONE, v, D, lin, state, stream);
    launch_attention_gen(qk, 2 * D, qk + D, 2 * D, v, D, static_cast<int>(tokens), static_cast<int>(tokens), heads, hd,
                         scale, 0, nullptr, 0, 0, att, D, state, stream, nullptr, 0, planes);
    apply_linear(ly.sa_out_proj, 0, D, att, D, tokens, SAMQ_EPILOGUE_NONE, y, D, lin, state, stream);
    launch_add_rows(x, D, y, D, tokens, static_cast<int>(D), stream);
    // Cross-attention to the prompt tokens (key padding bias).
    launch_layer_norm_f32(x, tokens, static_cast<int>(D), D, ly.norm2_w, ly.norm2_b, h, D, 1e-5f, stream);
    apply_linear(ly.ca_in_proj, 0, D, h, D, tokens, SAMQ_EPILOGUE_NONE, qk, D, lin, state, stream);
    apply_linear(ly.ca_in_proj, D, 2 * D, prompt, D, prompt_tokens, SAMQ_EPILOGUE_NONE, pkv, 2 * D, lin, state, stream);
    launch_attention_gen(qk, D, pkv, 2 * D, pkv + D, 2 * D, static_cast<int>(tokens), static_cast<int>(prompt_tokens),
                         heads, hd, scale, 0, prompt_bias, 0, 0, att, D, state, stream);
    apply_linear(ly.ca_out_proj, 0, D, att, D, tokens, SAMQ_EPILOGUE_NONE, y, D, lin, state, stream);
    launch_add_rows(x, D, y, D, tokens, static_cast<int>(D), stream);
    // FFN with ReLU.
    launch_layer_norm_f32(x, tokens, static_cast<int>(D), D, ly.norm3_w, ly.norm3_b, h, D, 1e-5f, stream);
    apply_linear(ly.linear1, 0, F, h, D, tokens, SAMQ_EPILOGUE_NONE, ffn, F, lin, state, stream);
    launch_relu(ffn, tokens * F, stream);
    apply_linear(ly.linear2, 0, D, ffn, F, tokens, SAMQ_EPILOGUE_NONE, y, D, lin, state, stream);
    launch_add_rows(x, D, y, D, tokens, static_cast<int>(D), stream);
}

}  // namespace samq
