// decoder.cu -- the SAM 3 DETR decoder, its dot-product scoring and presence
// head on the device (src/models/sam3/detector.hpp:67-713).
//
// Per layer (6): query positions from the current reference boxes (sine
// embedding, detector.hpp:67-104, through ref_point_head), the box relative
// position bias of the image cross-attention (:160-305), then post-norm
// self-attention, text cross-attention, image cross-attention and ReLU FFN
// (:307-478), then box refinement sigmoid(inverse_sigmoid(ref) + bbox_embed(
// LN(queries))) (:660-690).  After the layers: the final LayerNorm of the
// object queries, the dot-product scoring against the pooled prompt (:507-582)
// and the presence head.  The linears are samq_linear_ref_v1 (quantized or
// dense); attention is the general F32 attention; the small element-wise
// steps are the kernels below, each written to GGML's f32 op order.
#include <cmath>

#include "samq_internal.hpp"

namespace samq {
namespace {

unsigned blocks_of(int64_t work) { return static_cast<unsigned>(std::max<int64_t>(1, (work + 255) / 256)); }

struct DimT {
    float v[64];
};

// out[q][c*128 + 2i + {0,1}] = sin / cos(ref[q][order[c]] * dim_t[i]), order (cy, cx, w, h).
__global__ void __launch_bounds__(256) sine_embed_kernel(const float* __restrict__ ref, int nq, DimT dim_t,
                                                         float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= int64_t(nq) * 256) return;
    const int q = static_cast<int>(idx / 256), r = static_cast<int>(idx % 256);
    const int c = r / 64, i = r % 64;
    const int order[4] = {1, 0, 2, 3};
    const float a = __fmul_rn(ref[q * 4 + order[c]], dim_t.v[i]);
    out[int64_t(q) * 512 + c * 128 + 2 * i] = sinf(a);
    out[int64_t(q) * 512 + c * 128 + 2 * i + 1] = cosf(a);
}

// The first layer of a box-RPB MLP on the log-scaled deltas of one axis:
// hidden[(q * grid + g)][c] = ReLU(w0[c][0] d_lo + w0[c][1] d_hi + b0[c]) with
// d = sign(8 (coord_g - edge)) log(|8 (coord_g - edge)| + 1) / ln 2 / log2 8,
// edge lo / hi = center -+ size / 2 of box q on that axis (axis 0: x, 1: y).
__global__ void __launch_bounds__(256) rpb_hidden_kernel(const float* __restrict__ ref, int nq, int grid, int axis,
                                                         const float* __restrict__ w0, const float* __restrict__ b0,
                                                         int hidden, float inv_ln2, float inv_log2_8,
                                                         float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= int64_t(nq) * grid * hidden) return;
    const int c = static_cast<int>(idx % hidden);
    const int64_t s = idx / hidden;
    const int g = static_cast<int>(s % grid), q = static_cast<int>(s / grid);
    const float center = ref[q * 4 + axis], size = ref[q * 4 + 2 + axis];
    const float half = __fmul_rn(size, 0.5f);
    const float coord = __fdiv_rn(static_cast<float>(g), static_cast<float>(grid));
    float d[2] = {__fsub_rn(coord, __fsub_rn(center, half)), __fsub_rn(coord, __fadd_rn(center, half))};
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const float d8 = __fmul_rn(d[e], 8.0f);
        const float sg = d8 > 0.0f ? 1.0f : (d8 < 0.0f ? -1.0f : 0.0f);
        const float lv = __fmul_rn(logf(__fadd_rn(fabsf(d8), 1.0f)), inv_ln2);
        d[e] = __fmul_rn(sg, __fmul_rn(lv, inv_log2_8));
    }
    const float v = __fadd_rn(__fadd_rn(__fmul_rn(w0[c * 2], d[0]), __fmul_rn(w0[c * 2 + 1], d[1])), b0[c]);
    out[idx] = fmaxf(v, 0.0f);
}

// bias[h][q][ky * grid + kx] = q == 0 ? 0 : ry[(q-1) * grid + ky][h] + rx[(q-1) * grid + kx][h]
// (ry / rx rows of `heads` values).
__global__ void __launch_bounds__(256) rpb_assemble_kernel(const float* __restrict__ rx, const float* __restrict__ ry,
                                                           int nq, int grid, int heads, int64_t ldr,
                                                           float* __restrict__ bias) {
    pdl_wait();
    pdl_trigger();
    const int64_t keys = int64_t(grid) * grid;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= int64_t(heads) * (nq + 1) * keys) return;
    const int64_t k = idx % keys;
    const int64_t rest = idx / keys;
    const int q = static_cast<int>(rest % (nq + 1)), h = static_cast<int>(rest / (nq + 1));
    float v = 0.0f;
    if (q > 0) {
        const int ky = static_cast<int>(k / grid), kx = static_cast<int>(k % grid);
        v = __fadd_rn(ry[(int64_t(q - 1) * grid + ky) * ldr + h], rx[(int64_t(q - 1) * grid + kx) * ldr + h]);
    }
    bias[idx] = v;
}

__device__ __forceinline__ float sigmoid_f(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }

// ref = sigmoid(inverse_sigmoid(ref) + delta) (detector.hpp:42-48, 686-688).
__global__ void __launch_bounds__(256) box_refine_kernel(float* __restrict__ ref, const float* __restrict__ delta,
                                                         int64_t ldd, int nq) {
    pdl_wait();
    pdl_trigger();
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= nq * 4) return;
    const float x = fminf(fmaxf(ref[idx], 0.0f), 1.0f);
    const float a = logf(fminf(fmaxf(x, 1e-3f), 1.0f));
    const float b = logf(fminf(fmaxf(__fsub_rn(1.0f, x), 1e-3f), 1.0f));
    ref[idx] = sigmoid_f(__fadd_rn(__fsub_rn(a, b), delta[int64_t(idx / 4) * ldd + idx % 4]));
}

__global__ void __launch_bounds__(256) sigmoid_kernel(const float* __restrict__ x, float* __restrict__ y, int n) {
    pdl_wait();
    pdl_trigger();
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx < n) y[idx] = sigmoid_f(x[idx]);
}

// pooled[c] = (sum_t valid[t] x[t][c]) / T (ggml_pool_1d AVG over the masked rows).
__global__ void __launch_bounds__(256) masked_mean_kernel(const float* __restrict__ x, const float* __restrict__ valid,
                                                          int tokens, int width, float* __restrict__ pooled) {
    pdl_wait();
    pdl_trigger();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= width) return;
    float s = 0.0f;
    for (int t = 0; t < tokens; ++t) s += __fmul_rn(x[int64_t(t) * width + c], valid ? valid[t] : 1.0f);
    pooled[c] = __fdiv_rn(s, static_cast<float>(tokens));
}

// scores[q] = clamp((hs[q] . pooled) * scale, -12, 12), one warp per query.
__global__ void __launch_bounds__(256) dot_score_kernel(const float* __restrict__ hs, const float* __restrict__ p,
                                                        int nq, int width, float scale, float* __restrict__ scores) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int q = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (q >= nq) return;
    float s = 0.0f;
    for (int c = lane; c < width; c += 32) s = fmaf(hs[int64_t(q) * width + c], p[c], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) scores[q] = fminf(fmaxf(__fmul_rn(s, scale), -12.0f), 12.0f);
}

}  // namespace

// Key-split partials of the decoder's attentions (self over nq + 1 queries,
// image cross-attention over enc_tokens keys), one buffer reused by both.
size_t decoder_attention_partials(const samq_decoder_v1& dec, int64_t enc_tokens, int sms) {
    const int64_t D = linear_in(dec.layer[0].sa_in_proj);
    const int heads = dec.heads, hd = static_cast<int>(D / heads), nq1 = dec.queries + 1;
    return std::max(attention_partial_floats(nq1, nq1, heads, hd, 0, sms),
                    attention_partial_floats(nq1, static_cast<int>(enc_tokens), heads, hd, 0, sms));
}

size_t decoder_scratch_bytes(const samq_decoder_v1& dec, int64_t enc_tokens, int64_t prompt_tokens, int grid,
                             int sms) {
    const int64_t D = linear_in(dec.layer[0].sa_in_proj), nq = dec.queries, F = linear_out(dec.layer[0].linear1);
    const int64_t hidden = 256, heads = dec.heads;
    size_t linear = 0;
    auto grow = [&](const samq_linear_ref_v1& l, int64_t m) { linear = std::max(linear, linear_scratch_bytes(l, m, sms)); };
    for (int i = 0; i < dec.layers; ++i) {
        const samq_decoder_layer_v1& ly = dec.layer[i];
        for (const samq_linear_ref_v1* l : {&ly.sa_in_proj, &ly.sa_out_proj, &ly.ca_text_in_proj, &ly.ca_text_out_proj,
                                            &ly.ca_in_proj, &ly.ca_out_proj, &ly.linear1, &ly.linear2})
            grow(*l, nq + 1);
        grow(ly.ca_text_in_proj, prompt_tokens);
        grow(ly.ca_in_proj, enc_tokens);
    }
    grow(dec.rpb_x1, nq * grid);
    grow(dec.rpb_y1, nq * grid);
    grow(dec.ref_point_head[0], nq);
    grow(dec.prompt_mlp[0], prompt_tokens);
    grow(dec.prompt_mlp[1], prompt_tokens);
    const int64_t Fp = linear_out(dec.prompt_mlp[0]);
    const size_t floats = static_cast<size_t>(nq + 1) * D * 8 + (nq + 1) * F + nq * 512 + nq * 4 * 2 +
                          static_cast<size_t>(enc_tokens) * D * 3 + prompt_tokens * (2 * D + Fp) +
                          static_cast<size_t>(nq) * grid * (hidden + 16) * 2 +
                          static_cast<size_t>(heads) * (nq + 1) * grid * grid + D * 4 + nq * 2 +
                          decoder_attention_partials(dec, enc_tokens, sms);
    return floats * sizeof(float) + linear + 40 * 256;
}

void launch_decoder(const samq_decoder_v1& dec, const float* enc, const float* enc_pos, int64_t enc_tokens, int grid,
                    const float* prompt, const float* prompt_bias, const float* prompt_valid, int64_t prompt_tokens,
                    float* queries_out, float* boxes, float* scores, float* presence, void* scratch,
                    DeviceState& state, cudaStream_t stream) {
    const int64_t D = linear_in(dec.layer[0].sa_in_proj), nq = dec.queries, F = linear_out(dec.layer[0].linear1);
    const int heads = dec.heads, hd = static_cast<int>(D / heads), hidden = 256;
    const int nq1 = static_cast<int>(nq + 1);
    const float scale = 1.0f / sqrtf(static_cast<float>(hd));
    auto align = [](uintptr_t p) { return (p + 255) & ~uintptr_t(255); };
    uintptr_t cursor = align(reinterpret_cast<uintptr_t>(scratch));
    auto take = [&](int64_t floats) {
        float* p = reinterpret_cast<float*>(cursor);
        cursor = align(cursor + static_cast<size_t>(floats) * sizeof(float));
        return p;
    };
    float* q = take(nq1 * D);
    float* qpos = take(nq1 * D);
    float* qin = take(nq1 * D);
    float* qk = take(nq1 * 2 * D);
    float* v = take(nq1 * D);
    float* att = take(nq1 * D);
    float* y = take(nq1 * D);
    float* ffn = take(nq1 * F);
    float* sine = take(nq * 512);
    float* ref = take(nq * 4);
    float* delta = take(nq * 4);
    float* kin = take(enc_tokens * D);
    float* kimg = take(enc_tokens * D);
    float* vimg = take(enc_tokens * D);
    const int64_t Fp = linear_out(dec.prompt_mlp[0]);
    float* tkv = take(prompt_tokens * 2 * D);
    float* tm = take(prompt_tokens * Fp);
    float* hid = take(nq * grid * hidden);
    float* rx = take(nq * grid * 16);
    float* ry = take(nq * grid * 16);
    float* bias = take(int64_t(heads) * nq1 * grid * grid);
    float* pooled = take(D * 4);
    float* hsp = take(nq * D);
    const size_t part_floats = decoder_attention_partials(dec, enc_tokens, state.sm_count);
    float* part = take(static_cast<int64_t>(part_floats));
    void* lin = reinterpret_cast<void*>(cursor);
    auto linear = [&](const samq_linear_ref_v1& l, int64_t row0, int64_t rows, const float* x, int64_t ldx, int64_t m,
                      float* out, int64_t ldo) {
        apply_linear(l, row0, rows, x, ldx, m, SAMQ_EPILOGUE_NONE, out, ldo, lin, state, stream);
    };

    DimT dim_t;
    for (int i = 0; i < 64; ++i)
        dim_t.v[i] = 2.0f * 3.14159265358979323846f / std::pow(10000.0f, 2.0f * static_cast<float>(i) / 128.0f);
    const float inv_ln2 = 1.0f / logf(2.0f), inv_log2_8 = 1.0f / log2f(8.0f);

    // queries = [presence token; query_embed], ref = sigmoid(reference_points).
    check_cuda(cudaMemcpyAsync(q, dec.presence_token, D * sizeof(float), cudaMemcpyDeviceToDevice, stream),
               "cudaMemcpyAsync(presence token)");
    check_cuda(cudaMemcpyAsync(q + D, dec.query_embed, nq * D * sizeof(float), cudaMemcpyDeviceToDevice, stream),
               "cudaMemcpyAsync(query embed)");
    launch_pdl(sigmoid_kernel, dim3(blocks_of(nq * 4)), dim3(256), 0, stream, "sigmoid_kernel launch",
               dec.reference_points, ref, static_cast<int>(nq * 4));
    check_cuda(cudaMemsetAsync(qpos, 0, D * sizeof(float), stream), "cudaMemsetAsync(presence position)");
    // Image keys' input (enc + pos) is the same for every layer.
    launch_add2(enc, enc_pos, kin, enc_tokens, static_cast<int>(D), stream);

    for (int i = 0; i < dec.layers; ++i) {
        const samq_decoder_layer_v1& ly = dec.layer[i];
        // Query positions: ref_point_head(sine(ref)), row 0 (presence) zero.
        launch_pdl(sine_embed_kernel, dim3(blocks_of(nq * 256)), dim3(256), 0, stream, "sine_embed_kernel launch",
                   static_cast<const float*>(ref), static_cast<int>(nq), dim_t, sine);
        linear(dec.ref_point_head[0], 0, D, sine, 512, nq, y, D);
        launch_relu(y, nq * D, stream);
        linear(dec.ref_point_head[1], 0, D, y, D, nq, qpos + D, D);
        // Box relative position bias [heads][nq + 1][grid^2].
        for (int axis = 0; axis < 2; ++axis) {
            launch_pdl(rpb_hidden_kernel, dim3(blocks_of(nq * grid * hidden)), dim3(256), 0, stream,
                       "rpb_hidden_kernel launch", static_cast<const float*>(ref), static_cast<int>(nq), grid, axis,
                       axis == 0 ? dec.rpb_x0_w : dec.rpb_y0_w, axis == 0 ? dec.rpb_x0_b : dec.rpb_y0_b, hidden,
                       inv_ln2, inv_log2_8, hid);
            linear(axis == 0 ? dec.rpb_x1 : dec.rpb_y1, 0, heads, hid, hidden, nq * grid, axis == 0 ? rx : ry, 16);
        }
        launch_pdl(rpb_assemble_kernel, dim3(blocks_of(int64_t(heads) * nq1 * grid * grid)), dim3(256), 0, stream,
                   "rpb_assemble_kernel launch", static_cast<const float*>(rx), static_cast<const float*>(ry),
                   static_cast<int>(nq), grid, heads, int64_t(16), bias);
        // 1. self-attention (Q = K from queries + pos, V from queries), norm2.
        launch_add2(q, qpos, qin, nq1, static_cast<int>(D), stream);
        linear(ly.sa_in_proj, 0, 2 * D, qin, D, nq1, qk, 2 * D);
        linear(ly.sa_in_proj, 2 * D, D, q, D, nq1, v, D);
        launch_attention_gen(qk, 2 * D, qk + D, 2 * D, v, D, nq1, nq1, heads, hd, scale, 0, nullptr, 0, 0, att, D,
                             state, stream, part, part_floats);
        linear(ly.sa_out_proj, 0, D, att, D, nq1, y, D);
        launch_add_rows(q, D, y, D, nq1, static_cast<int>(D), stream);
        launch_layer_norm_f32(q, nq1, static_cast<int>(D), D, ly.norm2_w, ly.norm2_b, q, D, 1e-5f, stream);
        // 2. text cross-attention, norm_ca_text.
        launch_add2(q, qpos, qin, nq1, static_cast<int>(D), stream);
        linear(ly.ca_text_in_proj, 0, D, qin, D, nq1, qk, D);
        linear(ly.ca_text_in_proj, D, 2 * D, prompt, D, prompt_tokens, tkv, 2 * D);
        launch_attention_gen(qk, D, tkv, 2 * D, tkv + D, 2 * D, nq1, static_cast<int>(prompt_tokens), heads, hd, scale,
                             0, prompt_bias, 0, 0, att, D, state, stream);
        linear(ly.ca_text_out_proj, 0, D, att, D, nq1, y, D);
        launch_add_rows(q, D, y, D, nq1, static_cast<int>(D), stream);
        launch_layer_norm_f32(q, nq1, static_cast<int>(D), D, ly.norm_ca_text_w, ly.norm_ca_text_b, q, D, 1e-5f,
                              stream);
        // 3. image cross-attention with the box bias, norm1.
        launch_add2(q, qpos, qin, nq1, static_cast<int>(D), stream);
        linear(ly.ca_in_proj, 0, D, qin, D, nq1, qk, D);
        linear(ly.ca_in_proj, D, D, kin, D, enc_tokens, kimg, D);
        linear(ly.ca_in_proj, 2 * D, D, enc, D, enc_tokens, vimg, D);
        launch_attention_gen(qk, D, kimg, D, vimg, D, nq1, static_cast<int>(enc_tokens), heads, hd, scale, 0, bias,
                             int64_t(nq1) * grid * grid, int64_t(grid) * grid, att, D, state, stream, part, part_floats);
        linear(ly.ca_out_proj, 0, D, att, D, nq1, y, D);
        launch_add_rows(q, D, y, D, nq1, static_cast<int>(D), stream);
        launch_layer_norm_f32(q, nq1, static_cast<int>(D), D, ly.norm1_w, ly.norm1_b, q, D, 1e-5f, stream);
        // 4. ReLU FFN, norm3.
        linear(ly.linear1, 0, F, q, D, nq1, ffn, F);
        launch_relu(ffn, nq1 * F, stream);
        linear(ly.linear2, 0, D, ffn, F, nq1, y, D);
        launch_add_rows(q, D, y, D, nq1, static_cast<int>(D), stream);
        launch_layer_norm_f32(q, nq1, static_cast<int>(D), D, ly.norm3_w, ly.norm3_b, q, D, 1e-5f, stream);
        // Box refinement on LN(object queries).
        launch_layer_norm_f32(q + D, nq, static_cast<int>(D), D, dec.norm_w, dec.norm_b, y, D, 1e-5f, stream);
        linear(dec.bbox_embed[0], 0, D, y, D, nq, att, D);
        launch_relu(att, nq * D, stream);
        linear(dec.bbox_embed[1], 0, D, att, D, nq, y, D);
        launch_relu(y, nq * D, stream);
        linear(dec.bbox_embed[2], 0, 4, y, D, nq, delta, 4);
        launch_pdl(box_refine_kernel, dim3(blocks_of(nq * 4)), dim3(256), 0, stream, "box_refine_kernel launch", ref,
                   static_cast<const float*>(delta), int64_t(4), static_cast<int>(nq));
    }
    // Outputs: [presence; LN(object queries)], boxes, scores, presence logit.
    check_cuda(cudaMemcpyAsync(queries_out, q, D * sizeof(float), cudaMemcpyDeviceToDevice, stream),
               "cudaMemcpyAsync(presence query)");
    launch_layer_norm_f32(q + D, nq, static_cast<int>(D), D, dec.norm_w, dec.norm_b, queries_out + D, D, 1e-5f, stream);
    check_cuda(cudaMemcpyAsync(boxes, ref, nq * 4 * sizeof(float), cudaMemcpyDeviceToDevice, stream),
               "cudaMemcpyAsync(boxes)");
    // Scoring: prompt MLP (residual, LN), masked mean, projections, scaled dot.
    linear(dec.prompt_mlp[0], 0, Fp, prompt, D, prompt_tokens, tm, Fp);
    launch_relu(tm, prompt_tokens * Fp, stream);
    linear(dec.prompt_mlp[1], 0, D, tm, Fp, prompt_tokens, tkv, D);
    launch_add_rows(tkv, D, prompt, D, prompt_tokens, static_cast<int>(D), stream);
    launch_layer_norm_f32(tkv, prompt_tokens, static_cast<int>(D), D, dec.prompt_mlp_norm_w, dec.prompt_mlp_norm_b,
                          tkv, D, 1e-5f, stream);
    launch_pdl(masked_mean_kernel, dim3(blocks_of(D)), dim3(256), 0, stream, "masked_mean_kernel launch",
               static_cast<const float*>(tkv), prompt_valid, static_cast<int>(prompt_tokens), static_cast<int>(D),
               pooled);
    linear(dec.prompt_proj, 0, D, pooled, D, 1, pooled + D, D);
    linear(dec.hs_proj, 0, D, queries_out + D, D, nq, hsp, D);
    launch_pdl(dot_score_kernel, dim3(blocks_of(nq * 32)), dim3(256), 0, stream, "dot_score_kernel launch",
               static_cast<const float*>(hsp), static_cast<const float*>(pooled + D), static_cast<int>(nq),
               static_cast<int>(D), 1.0f / sqrtf(static_cast<float>(D)), scores);
    // Presence head: LN + MLP 256 -> 256 -> 256 -> 1 on the last presence query.
    launch_layer_norm_f32(q, 1, static_cast<int>(D), D, dec.presence_norm_w, dec.presence_norm_b, pooled + 2 * D, D,
                          1e-5f, stream);
    linear(dec.presence_head[0], 0, D, pooled + 2 * D, D, 1, y, D);
    launch_relu(y, D, stream);
    linear(dec.presence_head[1], 0, D, y, D, 1, att, D);
    launch_relu(att, D, stream);
    linear(dec.presence_head[2], 0, 1, att, D, 1, y, 4);
    check_cuda(cudaMemcpyAsync(presence, y, sizeof(float), cudaMemcpyDeviceToDevice, stream),
               "cudaMemcpyAsync(presence)");
}

}  // namespace samq
