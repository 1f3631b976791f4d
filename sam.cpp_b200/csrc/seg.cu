// seg.cu -- the SAM 3 segmentation head and the geometry encoder on the device.
//
// Segmentation head (src/models/sam3/mask_decoder.hpp:57-202):
//   enc' = enc + out_proj(attn(Q = Wq LN(enc), K/V = Wk/Wv prompt; prompt key bias))
//   p1 = ReLU(GN(conv3x3(fpn1 + up2(enc'))))        at 2 grid x 2 grid
//   p0 = ReLU(GN(conv3x3(fpn0 + up2(p1))))          at 4 grid x 4 grid
//   pixel_embed = conv1x1(p0)
//   logits[q][pixel] = mask_embed_mlp(queries)[q] . pixel_embed[pixel]
// NHWC throughout.  The convolutions and the final einsum are F32-semantics
// products on the tensor cores (the three-term TF32 split of dense.cu); every
// operand they read is written as its hi / lo split by its producer: the
// upsample-add kernel, the GroupNorm apply kernel, the 1x1 head's epilogue and
// a split of the mask embeddings.  GroupNorm(8) statistics are two passes
// (mean, then centred variance) of per-block partial sums, each finished in
// f64 by the kernel that consumes it.
//
// Geometry encoder (src/models/sam3/prompt_encoder.hpp:44-160), the
// text-only-prompt form: the learned CLS token through final_proj and a
// LayerNorm, three pre-norm layers (self-attention over the one token,
// cross-attention to the image with keys image + pos, ReLU FFN), encode_norm.
#include <algorithm>
#include <cmath>

#include "samq_internal.hpp"

namespace samq {
namespace {

constexpr int kGroups = 8;             // GroupNorm(8, C)
constexpr int kStatThreads = 256;

// hi / lo split of fpn + up2(prev): out pixel (y, x) of the (2h) x (2w) map
// adds prev[y / 2][x / 2] (ggml_upscale NEAREST then ggml_add).
__global__ void __launch_bounds__(256) upsample_add_split_kernel(const float* __restrict__ prev, int w, int h,
                                                                 const float* __restrict__ fpn, int64_t c4n,
                                                                 float* __restrict__ hi, float* __restrict__ lo) {
    pdl_wait();
    pdl_trigger();
    const int ow = 2 * w;
    const int64_t total = static_cast<int64_t>(ow) * (2 * h) * c4n;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t pix = i / c4n, c4 = i - pix * c4n;
        const int oy = static_cast<int>(pix / ow), ox = static_cast<int>(pix - static_cast<int64_t>(oy) * ow);
        const float4 a = __ldg(reinterpret_cast<const float4*>(fpn) + i);
        const float4 b =
            __ldg(reinterpret_cast<const float4*>(prev) + (static_cast<int64_t>(oy / 2) * w + ox / 2) * c4n + c4);
        float4 hv, lv;
        split_tf32(a.x + b.x, hv.x, lv.x);
        split_tf32(a.y + b.y, hv.y, lv.y);
        split_tf32(a.z + b.z, hv.z, lv.z);
        split_tf32(a.w + b.w, hv.w, lv.w);
        reinterpret_cast<float4*>(hi)[i] = hv;
        reinterpret_cast<float4*>(lo)[i] = lv;
    }
}

// f64 total over the blocks' partials of group g (partials [blocks][kGroups]),
// by the whole block; result in smem_total[g] for every g.
__device__ void reduce_partials(const float* __restrict__ partials, int blocks, double* smem, double* totals) {
    double acc[kGroups];
#pragma unroll
    for (int g = 0; g < kGroups; ++g) acc[g] = 0.0;
    for (int b = threadIdx.x; b < blocks; b += blockDim.x)
#pragma unroll
        for (int g = 0; g < kGroups; ++g) acc[g] += partials[b * kGroups + g];
#pragma unroll
    for (int g = 0; g < kGroups; ++g) smem[threadIdx.x * kGroups + g] = acc[g];
    __syncthreads();
    if (threadIdx.x < kGroups) {
        double t = 0.0;
        for (int j = 0; j < static_cast<int>(blockDim.x); ++j) t += smem[j * kGroups + threadIdx.x];
        totals[threadIdx.x] = t;
    }
    __syncthreads();
}

// One statistics pass over an NHWC map of `pixels` x C: pass 0 sums x, pass 1
// sums (x - mean_g)^2 with mean_g from pass 0's partials.  The grid-stride
// step (gridDim.x * 256 threads) is a multiple of C / 4, so each thread keeps
// one float4 column and so one group.  partials [gridDim.x][kGroups].
template <int PASS>
__global__ void __launch_bounds__(kStatThreads) group_stats_kernel(const float* __restrict__ x, int64_t pixels,
                                                                   int channels, const float* __restrict__ mean_partials,
                                                                   int mean_blocks, float* __restrict__ partials) {
    pdl_wait();
    pdl_trigger();
    __shared__ double smem[kStatThreads * kGroups];
    __shared__ double totals[kGroups];
    __shared__ float group_sum[kStatThreads / 32][kGroups];
    const int c4n = channels / 4, per_group = channels / kGroups;
    if (PASS == 1) reduce_partials(mean_partials, mean_blocks, smem, totals);
    const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    const int c4 = static_cast<int>(tid % c4n);
    const int g = c4 * 4 / per_group;
    const float m = PASS == 1 ? static_cast<float>(totals[g] / (static_cast<double>(pixels) * per_group)) : 0.0f;
    float acc = 0.0f;
    const int64_t total = pixels * c4n;
    for (int64_t i = tid; i < total; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
        if (PASS == 0) {
            acc += (v.x + v.y) + (v.z + v.w);
        } else {
            const float a = v.x - m, b = v.y - m, c = v.z - m, d = v.w - m;
            acc += (a * a + b * b) + (c * c + d * d);
        }
    }
    // Lanes of one warp cover 32 consecutive float4 columns: groups of
    // per_group / 4 lanes share a group.
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lanes_per_group = per_group / 4;
    for (int o = 1; o < lanes_per_group && o < 32; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (threadIdx.x < (kStatThreads / 32) * kGroups) (&group_sum[0][0])[threadIdx.x] = 0.0f;
    __syncthreads();
    if (lane % lanes_per_group == 0) atomicAdd(&group_sum[warp][g], acc);
    __syncthreads();
    if (threadIdx.x < kGroups) {
        float s = 0.0f;
        for (int w = 0; w < kStatThreads / 32; ++w) s += group_sum[w][threadIdx.x];
        partials[blockIdx.x * kGroups + threadIdx.x] = s;
    }
}

// y = ReLU(((x - mean_g) * rstd_g) * w[c] + b[c]) (ggml_group_norm, ggml_mul,
// ggml_add, ggml_relu), written as f32 (lo == nullptr) or the hi / lo split.
__global__ void __launch_bounds__(kStatThreads) group_apply_kernel(
    const float* __restrict__ x, int64_t pixels, int channels, const float* __restrict__ mean_partials,
    const float* __restrict__ var_partials, int blocks, const float* __restrict__ w, const float* __restrict__ b,
    float eps, float* __restrict__ y, float* __restrict__ lo) {
    pdl_wait();
    pdl_trigger();
    __shared__ double smem[kStatThreads * kGroups];
    __shared__ double totals[kGroups];
    __shared__ float stats[2 * kGroups];
    const int per_group = channels / kGroups;
    const double count = static_cast<double>(pixels) * per_group;
    reduce_partials(mean_partials, blocks, smem, totals);
    if (threadIdx.x < kGroups) stats[threadIdx.x] = static_cast<float>(totals[threadIdx.x] / count);
    __syncthreads();
    reduce_partials(var_partials, blocks, smem, totals);
    if (threadIdx.x < kGroups) {
        const float var = static_cast<float>(totals[threadIdx.x] / count);
        stats[kGroups + threadIdx.x] = 1.0f / sqrtf(var + eps);
    }
    __syncthreads();
    const int c4n = channels / 4;
    const int64_t total = pixels * c4n;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % c4n) * 4;
        const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
        const float in[4] = {v.x, v.y, v.z, v.w};
        float out[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int g = (c + e) / per_group;
            const float nrm = __fmul_rn(__fsub_rn(in[e], stats[g]), stats[kGroups + g]);
            out[e] = fmaxf(__fadd_rn(__fmul_rn(nrm, w[c + e]), b[c + e]), 0.0f);
        }
        if (lo == nullptr) {
            reinterpret_cast<float4*>(y)[i] = make_float4(out[0], out[1], out[2], out[3]);
        } else {
            float4 hv, lv;
            split_tf32(out[0], hv.x, lv.x);
            split_tf32(out[1], hv.y, lv.y);
            split_tf32(out[2], hv.z, lv.z);
            split_tf32(out[3], hv.w, lv.w);
            reinterpret_cast<float4*>(y)[i] = hv;
            reinterpret_cast<float4*>(lo)[i] = lv;
        }
    }
}

int stat_blocks(int channels, const DeviceState& state) {
    // gridDim.x * 256 must be a multiple of C / 4 (C / 4 divides 256 for C <= 1024).
    (void)channels;
    return state.sm_count * 4;
}

void launch_group_norm_relu(const float* x, int64_t pixels, int channels, const float* w, const float* b, float* y,
                            float* lo, float* partials, DeviceState& state, cudaStream_t stream) {
    const int nb = stat_blocks(channels, state);
    float* mean_p = partials;
    float* var_p = partials + nb * kGroups;
    launch_pdl(group_stats_kernel<0>, dim3(nb), dim3(kStatThreads), 0, stream, "group_stats_kernel<0> launch", x,
               pixels, channels, static_cast<const float*>(nullptr), 0, mean_p);
    launch_pdl(group_stats_kernel<1>, dim3(nb), dim3(kStatThreads), 0, stream, "group_stats_kernel<1> launch", x,
               pixels, channels, static_cast<const float*>(mean_p), nb, var_p);
    launch_pdl(group_apply_kernel, dim3(nb), dim3(kStatThreads), 0, stream, "group_apply_kernel launch", x, pixels,
               channels, static_cast<const float*>(mean_p), static_cast<const float*>(var_p), nb, w, b, 1e-5f, y, lo);
}

void launch_upsample_add_split(const float* prev, int w, int h, const float* fpn, int channels, float* hi, float* lo,
                               DeviceState& state, cudaStream_t stream) {
    const int64_t work = static_cast<int64_t>(4) * w * h * (channels / 4);
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((work + 255) / 256, int64_t(state.sm_count) * 8));
    launch_pdl(upsample_add_split_kernel, dim3(grid), dim3(256), 0, stream, "upsample_add_split_kernel launch", prev,
               w, h, fpn, static_cast<int64_t>(channels / 4), hi, lo);
}

}  // namespace

size_t seg_head_scratch_bytes(const samq_seg_head_v1& sh, int grid, int64_t queries, int64_t prompt_tokens, int sms) {
    const int64_t D = linear_in(sh.ca_in_proj), T = int64_t(grid) * grid, big = 16 * T;
    size_t linear = 0;
    for (const samq_linear_ref_v1* l : {&sh.ca_in_proj, &sh.ca_out_proj})
        linear = std::max(linear, linear_scratch_bytes(*l, T, sms));
    linear = std::max(linear, linear_scratch_bytes(sh.ca_in_proj, prompt_tokens, sms));
    for (const samq_linear_ref_v1& l : sh.mask_embed) linear = std::max(linear, linear_scratch_bytes(l, queries, sms));
    // h, q, att, y, enc' [T][D]; prompt k|v [P][2D]; p1 [4T][D]; mh, ml, c, pe_lo [16T][D];
    // mask embeddings x 3 + split x 2 [Q][D]; statistics partials
    const size_t floats = static_cast<size_t>(T) * D * 5 + prompt_tokens * 2 * D + 4 * T * D + 4 * big * D +
                          queries * D * 5 + 2 * static_cast<size_t>(sms) * 4 * kGroups;
    return floats * sizeof(float) + linear + 24 * 256;
}

void launch_seg_head(const samq_seg_head_v1& sh, const float* enc, int grid, const float* fpn0, const float* fpn1,
                     const float* queries, int64_t nq, const float* prompt, const float* prompt_bias,
                     int64_t prompt_tokens, float* logits, void* scratch, DeviceState& state, cudaStream_t stream) {
    const int64_t D = linear_in(sh.ca_in_proj), T = int64_t(grid) * grid;
    const int heads = sh.heads, hd = static_cast<int>(D / heads), g2 = 2 * grid, g4 = 4 * grid;
    const int64_t T2 = int64_t(g2) * g2, T4 = int64_t(g4) * g4;
    auto align = [](uintptr_t p) { return (p + 255) & ~uintptr_t(255); };
    uintptr_t cursor = align(reinterpret_cast<uintptr_t>(scratch));
    auto take = [&](int64_t floats) {
        float* p = reinterpret_cast<float*>(cursor);
        cursor = align(cursor + static_cast<size_t>(floats) * sizeof(float));
        return p;
    };
    float* h = take(T * D);
    float* q = take(T * D);
    float* att = take(T * D);
    float* y = take(T * D);
    float* e1 = take(T * D);
    float* pkv = take(prompt_tokens * 2 * D);
    float* p1 = take(T2 * D);
    float* mh = take(T4 * D);
    float* ml = take(T4 * D);
    float* c = take(T4 * D);
    float* pe_lo = take(T4 * D);
    float* me0 = take(nq * D);
    float* me1 = take(nq * D);
    float* me2 = take(nq * D);
    float* meh = take(nq * D);
    float* mel = take(nq * D);
    float* partials = take(2 * int64_t(state.sm_count) * 4 * kGroups);
    void* lin = reinterpret_cast<void*>(cursor);
    auto linear = [&](const samq_linear_ref_v1& l, int64_t row0, int64_t rows, const float* x, int64_t ldx, int64_t m,
                      float* out, int64_t ldo) {
        apply_linear(l, row0, rows, x, ldx, m, SAMQ_EPILOGUE_NONE, out, ldo, lin, state, stream);
    };
    const float scale = 1.0f / sqrtf(static_cast<float>(hd));

    // 1. Prompt cross-attention on the fusion output (residual, no positions).
    launch_layer_norm_f32(enc, T, static_cast<int>(D), D, sh.cross_attn_norm_w, sh.cross_attn_norm_b, h, D, 1e-5f,
                          stream);
    linear(sh.ca_in_proj, 0, D, h, D, T, q, D);
    linear(sh.ca_in_proj, D, 2 * D, prompt, D, prompt_tokens, pkv, 2 * D);
    launch_attention_gen(q, D, pkv, 2 * D, pkv + D, 2 * D, static_cast<int>(T), static_cast<int>(prompt_tokens),
                         heads, hd, scale, 0, prompt_bias, 0, 0, att, D, state, stream);
    linear(sh.ca_out_proj, 0, D, att, D, T, y, D);
    launch_add2(enc, y, e1, T, static_cast<int>(D), stream);
    // 2. Pixel decoder stage 0: fpn1 + up2(enc') -> conv3x3 -> GN -> ReLU (f32).
    launch_upsample_add_split(e1, grid, grid, fpn1, static_cast<int>(D), mh, ml, state, stream);
    launch_dense_gemm(mh, ml, *sh.conv[0], T2, g2, g2, sh.conv_b[0], 0, c, nullptr, D, state, stream);
    launch_group_norm_relu(c, T2, static_cast<int>(D), sh.norm_w[0], sh.norm_b[0], p1, nullptr, partials, state,
                           stream);
    // 3. Stage 1: fpn0 + up2(p1) -> conv3x3 -> GN -> ReLU (split for the 1x1 head).
    launch_upsample_add_split(p1, g2, g2, fpn0, static_cast<int>(D), mh, ml, state, stream);
    launch_dense_gemm(mh, ml, *sh.conv[1], T4, g4, g4, sh.conv_b[1], 0, c, nullptr, D, state, stream);
    launch_group_norm_relu(c, T4, static_cast<int>(D), sh.norm_w[1], sh.norm_b[1], mh, ml, partials, state, stream);
    // 4. Instance head (1x1), written as the split B operand of the einsum: hi in c.
    launch_dense_gemm(mh, ml, *sh.instance, T4, 0, 0, sh.instance_b, 0, c, pe_lo, D, state, stream);
    // 5. Mask embeddings: 3-layer MLP (ReLU between), split.
    linear(sh.mask_embed[0], 0, D, queries, D, nq, me0, D);
    launch_relu(me0, nq * D, stream);
    linear(sh.mask_embed[1], 0, D, me0, D, nq, me1, D);
    launch_relu(me1, nq * D, stream);
    linear(sh.mask_embed[2], 0, D, me1, D, nq, me2, D);
    launch_split_rows(me2, nq, D, D, meh, mel, state, stream);
    // 6. logits[q][pixel] = me[q] . pe[pixel]: the pixel embeddings are the
    //    "weights" [T4][D] of an F32-semantics product.
    samq_dense view;
    view.device = sh.instance->device;
    view.type = SAMQ_TYPE_F32;
    view.kind = SAMQ_DENSE_LINEAR;
    view.ks = 1;
    view.cin = D;
    view.cout = T4;
    view.n = T4;
    view.k = D;
    view.hi = c;
    view.lo = pe_lo;
    launch_dense_gemm(meh, mel, view, nq, 0, 0, nullptr, 0, logits, nullptr, T4, state, stream);
    view.hi = view.lo = nullptr;  // a view, not owned
}

size_t geometry_scratch_bytes(const samq_geometry_encoder_v1& ge, int64_t tokens, int sms) {
    const int64_t D = linear_in(ge.final_proj), F = linear_out(ge.layer[0].linear1);
    size_t linear = linear_scratch_bytes(ge.final_proj, 1, sms);
    for (int i = 0; i < ge.layers; ++i) {
        const samq_geometry_layer_v1& ly = ge.layer[i];
        for (const samq_linear_ref_v1* l : {&ly.sa_in_proj, &ly.sa_out_proj, &ly.ca_out_proj, &ly.linear1, &ly.linear2})
            linear = std::max(linear, linear_scratch_bytes(*l, 1, sms));
        linear = std::max(linear, linear_scratch_bytes(ly.ca_in_proj, tokens, sms));
    }
    // x, xn, qkv(3D), att, y, ffn(F) for the token; kin, k, v [T][D]; key-split partials
    const size_t floats = static_cast<size_t>(D) * 7 + F + static_cast<size_t>(tokens) * D * 3 +
                          attention_partial_floats(1, static_cast<int>(tokens), ge.heads,
                                                   static_cast<int>(D / ge.heads), 0, sms);
    return floats * sizeof(float) + linear + 16 * 256;
}

void launch_geometry_encoder(const samq_geometry_encoder_v1& ge, const float* image, const float* pos, int64_t tokens,
                             float* out, void* scratch, DeviceState& state, cudaStream_t stream) {
    const int64_t D = linear_in(ge.final_proj), F = linear_out(ge.layer[0].linear1);
    const int heads = ge.heads, hd = static_cast<int>(D / heads);
    const float scale = 1.0f / sqrtf(static_cast<float>(hd));
    auto align = [](uintptr_t p) { return (p + 255) & ~uintptr_t(255); };
    uintptr_t cursor = align(reinterpret_cast<uintptr_t>(scratch));
    auto take = [&](int64_t floats) {
        float* p = reinterpret_cast<float*>(cursor);
        cursor = align(cursor + static_cast<size_t>(floats) * sizeof(float));
        return p;
    };
    float* x = take(D);
    float* xn = take(D);
    float* qkv = take(3 * D);
    float* att = take(D);
    float* y = take(D);
    float* ffn = take(F);
    float* kin = take(tokens * D);
    float* k = take(tokens * D);
    float* v = take(tokens * D);
    const size_t part_floats = attention_partial_floats(1, static_cast<int>(tokens), heads, hd, 0, state.sm_count);
    float* part = take(static_cast<int64_t>(part_floats));
    void* lin = reinterpret_cast<void*>(cursor);
    auto linear = [&](const samq_linear_ref_v1& l, int64_t row0, int64_t rows, const float* in, int64_t m,
                      float* o) { apply_linear(l, row0, rows, in, D, m, SAMQ_EPILOGUE_NONE, o, rows, lin, state, stream); };

    linear(ge.final_proj, 0, D, ge.cls_token, 1, y);
    launch_layer_norm_f32(y, 1, static_cast<int>(D), D, ge.norm_w, ge.norm_b, x, D, 1e-5f, stream);
    launch_add2(image, pos, kin, tokens, static_cast<int>(D), stream);
    for (int i = 0; i < ge.layers; ++i) {
        const samq_geometry_layer_v1& ly = ge.layer[i];
        // Self-attention over the single token (Q = K = V inputs = LN1(x)).
        launch_layer_norm_f32(x, 1, static_cast<int>(D), D, ly.norm1_w, ly.norm1_b, xn, D, 1e-5f, stream);
        linear(ly.sa_in_proj, 0, 3 * D, xn, 1, qkv);
        launch_attention_gen(qkv, 3 * D, qkv + D, 3 * D, qkv + 2 * D, 3 * D, 1, 1, heads, hd, scale, 0, nullptr, 0, 0,
                             att, D, state, stream);
        linear(ly.sa_out_proj, 0, D, att, 1, y);
        launch_add_rows(x, D, y, D, 1, static_cast<int>(D), stream);
        // Cross-attention to the image: K from image + pos, V from image.
        launch_layer_norm_f32(x, 1, static_cast<int>(D), D, ly.norm2_w, ly.norm2_b, xn, D, 1e-5f, stream);
        linear(ly.ca_in_proj, 0, D, xn, 1, qkv);
        linear(ly.ca_in_proj, D, D, kin, tokens, k);
        linear(ly.ca_in_proj, 2 * D, D, image, tokens, v);
        launch_attention_gen(qkv, D, k, D, v, D, 1, static_cast<int>(tokens), heads, hd, scale, 0, nullptr, 0, 0, att,
                             D, state, stream, part, part_floats);
        linear(ly.ca_out_proj, 0, D, att, 1, y);
        launch_add_rows(x, D, y, D, 1, static_cast<int>(D), stream);
        // ReLU FFN.
        launch_layer_norm_f32(x, 1, static_cast<int>(D), D, ly.norm3_w, ly.norm3_b, xn, D, 1e-5f, stream);
        apply_linear(ly.linear1, 0, F, xn, D, 1, SAMQ_EPILOGUE_NONE, ffn, F, lin, state, stream);
        launch_relu(ffn, F, stream);
        apply_linear(ly.linear2, 0, D, ffn, F, 1, SAMQ_EPILOGUE_NONE, y, D, lin, state, stream);
        launch_add_rows(x, D, y, D, 1, static_cast<int>(D), stream);
    }
    launch_layer_norm_f32(x, 1, static_cast<int>(D), D, ge.encode_norm_w, ge.encode_norm_b, out, D, 1e-5f, stream);
}

}  // namespace samq
