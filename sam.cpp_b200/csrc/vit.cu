// vit.cu -- the SAM 3 ViT block and backbone prefix around K2 / K3.
//
// Reference: src/models/sam3/vision.hpp:152-243 (sam3_vit_block_forward) and
// :252-282 (sam3_build_vit_prefix_graph); LayerNorm is ggml_norm(eps 1e-5)
// then * w + b (src/models/sam3/ops.hpp:56-66).
//
// One block is seven launches, every activation hand-off in the layout its
// consumer reads and every quantized linear fed the Q8_1 operand GGML's CUDA
// path would stage (vision.hpp linears via ops.hpp:40-45):
//   1 ln_stage_kernel   x -> LN1 -> Q8_1 operand, rows gathered window-major
//                       (ggml_win_part, vision.hpp:170-173)
//   2 gemm (qkv)        + bias -> RoPE'd Q (x 1/8), K, V^T in f16
//   3 attention_kernel  -> Q8_1 operand of proj, raster order (win_unpart)
//   4 gemm (proj)       x = x + (acc + bias)
//   5 ln_stage_kernel   x -> LN2 -> Q8_1 operand
//   6 gemm (fc1)        + bias -> erf-GELU -> Q8_1 operand of fc2
//   7 gemm (fc2)        x = x + (acc + bias)
// The prefix is im2col of the 14x14 patches (f16), the patch-embedding GEMM
// and one kernel for + tiled pos_embed and ln_pre.  All launches use
// programmatic dependent launch; each kernel waits for its predecessor before
// touching memory.
#include <algorithm>

#include "samq_internal.hpp"

namespace samq {
namespace {

constexpr float kLnEps = 1e-5f;

// Source raster token of window-major row r (identity for global blocks).
__device__ __forceinline__ int64_t window_row_token(int64_t r, int grid_w, int window) {
    if (window == 0) return r;
    const int64_t group_n = static_cast<int64_t>(window) * window;
    const int64_t g = r / group_n, n = r - g * group_n;
    const int per_row = grid_w / window;
    const int64_t wy = g / per_row, wx = g - wy * per_row;
    const int64_t ly = n / window, lx = n - ly * window;
    return (wy * window + ly) * grid_w + wx * window + lx;
}

// LayerNorm of one row held by a warp: lane l owns elements 128 i + 4 l .. +3
// (i < NV).  f32 arithmetic: mean, centred values, biased variance, 1/sqrt.
template <int NV>
__device__ __forceinline__ void layer_norm_row(float (&v)[NV][4], const float* __restrict__ w,
                                               const float* __restrict__ b, int lane) {
    constexpr float inv_e = 1.0f / (128.0f * NV);
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) sum += (v[i][0] + v[i][1]) + (v[i][2] + v[i][3]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum * inv_e;
    float sq = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[i][j] -= mean;
            sq = fmaf(v[i][j], v[i][j], sq);
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float rstd = 1.0f / sqrtf(sq * inv_e + kLnEps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + i * 32 + lane);
        const float4 bv = __ldg(reinterpret_cast<const float4*>(b) + i * 32 + lane);
        v[i][0] = fmaf(v[i][0] * rstd, wv.x, bv.x);
        v[i][1] = fmaf(v[i][1] * rstd, wv.y, bv.y);
        v[i][2] = fmaf(v[i][2] * rstd, wv.z, bv.z);
        v[i][3] = fmaf(v[i][3] * rstd, wv.w, bv.w);
    }
}

// One warp per output row r (window-major when window > 0): LayerNorm of the
// raster row it gathers, then the Q8_1 operand (8 lanes per 32-value block).
template <int NV>
__global__ void __launch_bounds__(256) ln_stage_kernel(const float* __restrict__ x, int64_t rows, int grid_w,
                                                       int window, const float* __restrict__ w,
                                                       const float* __restrict__ b, __half* __restrict__ a,
                                                       DeviceStatus* status) {
    pdl_wait();
    pdl_trigger();
    constexpr int E = 128 * NV;
    const int lane = threadIdx.x & 31;
    const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (r >= rows) return;  // whole warps only: rows are warp-uniform
    const float4* src = reinterpret_cast<const float4*>(x + window_row_token(r, grid_w, window) * E);
    float v[NV][4];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const float4 t = src[i * 32 + lane];
        v[i][0] = t.x; v[i][1] = t.y; v[i][2] = t.z; v[i][3] = t.w;
    }
    layer_norm_row<NV>(v, w, b, lane);
    // Q8_1 operand (the stage_q8_1 rule).  Block q = 4i + lane/8 of the row is
    // spread over 8 lanes; its two IEEE divisions are done once, by lane q,
    // and the scale / inverse go back by shuffles (2 divisions per lane per
    // row instead of 16, the larger part of this kernel's instructions).
    float amax[NV];
    bool bad = false;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        float a4 = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            a4 = fmaxf(a4, fabsf(v[i][j]));
            bad |= !(fabsf(v[i][j]) <= kOperandLimit);
        }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) a4 = fmaxf(a4, __shfl_xor_sync(0xffffffffu, a4, o));
        amax[i] = a4;
    }
    float my_amax = 0.0f;  // block q = lane: i = q / 4, held by lanes 8 * (q % 4) ..
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const float t = __shfl_sync(0xffffffffu, amax[i], (lane & 3) * 8);
        if ((lane >> 2) == i) my_amax = t;
    }
    const float my_dq = __half2float(__float2half_rn(__fdiv_rn(my_amax, 127.0f)));
    const float my_inv = my_amax == 0.0f ? 0.0f : __fdiv_rn(127.0f, my_amax);
    uint2* dst = reinterpret_cast<uint2*>(a + r * E);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int q = 4 * i + (lane >> 3);
        const float dq = __shfl_sync(0xffffffffu, my_dq, q);
        const float inv = __shfl_sync(0xffffffffu, my_inv, q);
        const float q0 = round_half_away(__fmul_rn(v[i][0], inv)), q1 = round_half_away(__fmul_rn(v[i][1], inv));
        const float q2 = round_half_away(__fmul_rn(v[i][2], inv)), q3 = round_half_away(__fmul_rn(v[i][3], inv));
        const __half2 h0 = __floats2half2_rn(__fmul_rn(dq, q0), __fmul_rn(dq, q1));
        const __half2 h1 = __floats2half2_rn(__fmul_rn(dq, q2), __fmul_rn(dq, q3));
        dst[i * 32 + lane] = make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
    }
    record_range(bad, status);
}

// x[t] = LayerNorm(x[t] + pos[(py % pg) * pg + px % pg]) in place, f32
// (ggml_repeat of the 24x24 pos_embed, vision.hpp:264-272, then ln_pre).
template <int NV>
__global__ void __launch_bounds__(256) embed_ln_kernel(float* __restrict__ x, int64_t rows, int grid_w,
                                                       const float* __restrict__ pos, int pos_grid,
                                                       const float* __restrict__ w, const float* __restrict__ b) {
    pdl_wait();
    pdl_trigger();
    constexpr int E = 128 * NV;
    const int lane = threadIdx.x & 31;
    const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (r >= rows) return;
    const int py = static_cast<int>(r / grid_w), px = static_cast<int>(r % grid_w);
    const float4* p = reinterpret_cast<const float4*>(pos + static_cast<int64_t>((py % pos_grid) * pos_grid + px % pos_grid) * E);
    float4* row = reinterpret_cast<float4*>(x + r * E);
    float v[NV][4];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const float4 t = row[i * 32 + lane];
        const float4 q = __ldg(p + i * 32 + lane);
        v[i][0] = t.x + q.x; v[i][1] = t.y + q.y; v[i][2] = t.z + q.z; v[i][3] = t.w + q.w;
    }
    layer_norm_row<NV>(v, w, b, lane);
#pragma unroll
    for (int i = 0; i < NV; ++i) row[i * 32 + lane] = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
}

// F32 patch columns, a[t][c * P*P + ky * P + kx] = image[c][py*P + ky][px*P + kx]
// (kp columns per row, kp % 4 == 0), four columns per thread.
__global__ void __launch_bounds__(256) im2col_f32_kernel(const float* __restrict__ image, int width, int height,
                                                         int patch, int grid_w, int64_t tokens, int kp,
                                                         float* __restrict__ a) {
    pdl_wait();
    pdl_trigger();
    const int groups = kp / 4;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= tokens * groups) return;
    const int64_t t = idx / groups;
    const int col0 = static_cast<int>(idx - t * groups) * 4;
    const int py = static_cast<int>(t / grid_w), px = static_cast<int>(t % grid_w);
    const int pp = patch * patch;
    float out[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int col = col0 + j;
        const int c = col / pp, rem = col - c * pp, ky = rem / patch, kx = rem - ky * patch;
        out[j] = __ldg(image + (static_cast<int64_t>(c) * height + py * patch + ky) * width + px * patch + kx);
    }
    *reinterpret_cast<float4*>(a + t * kp + col0) = make_float4(out[0], out[1], out[2], out[3]);
}

// Patch columns: a[t][c * P*P + ky * P + kx] = f16(image[c][py*P + ky][px*P + kx])
// for token t = py * grid_w + px (ggml_im2col of the stride-P, unpadded patch
// convolution, ops.hpp sam3_conv_2d), zero in the padding columns kp..ld-1.
__global__ void __launch_bounds__(256) im2col_kernel(const float* __restrict__ image, int width, int height,
                                                     int patch, int grid_w, int64_t tokens, int kp, int ld,
                                                     __half* __restrict__ a) {
    pdl_wait();
    pdl_trigger();
    // One thread per 8 consecutive columns of a row: a 16-byte store (ld is a
    // multiple of 64, the row starts 16-byte aligned).
    const int groups = ld / 8;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= tokens * groups) return;
    const int64_t t = idx / groups;
    const int col0 = static_cast<int>(idx - t * groups) * 8;
    const int py = static_cast<int>(t / grid_w), px = static_cast<int>(t % grid_w);
    const int pp = patch * patch;
    __align__(16) __half out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int col = col0 + j;
        float v = 0.0f;
        if (col < kp) {
            const int c = col / pp, rem = col - c * pp, ky = rem / patch, kx = rem - ky * patch;
            v = __ldg(image + (static_cast<int64_t>(c) * height + py * patch + ky) * width + px * patch + kx);
        }
        out[j] = __float2half_rn(v);
    }
    *reinterpret_cast<uint4*>(a + t * ld + col0) = *reinterpret_cast<const uint4*>(out);
}

// f32 [n][k] -> f16 [n][ld], zero padded (the patch-embedding B operand).
__global__ void __launch_bounds__(256) pad_f16_kernel(const float* __restrict__ src, int64_t n, int k, int ld,
                                                      __half* __restrict__ dst) {
    pdl_wait();
    pdl_trigger();
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= n * ld) return;
    const int64_t row = idx / ld;
    const int col = static_cast<int>(idx - row * ld);
    dst[idx] = __float2half_rn(col < k ? __ldg(src + row * k + col) : 0.0f);
}

unsigned blocks_for(int64_t threads) { return static_cast<unsigned>((threads + 255) / 256); }

template <class Fn>
void by_width(int embed, Fn&& fn) {
    switch (embed) {
        case 256: fn(std::integral_constant<int, 2>{}); break;
        case 512: fn(std::integral_constant<int, 4>{}); break;
        case 1024: fn(std::integral_constant<int, 8>{}); break;
        default: fail(SAMQ_ERR_INVALID_ARGUMENT, "embedding width must be 256, 512 or 1024");
    }
}

}  // namespace

size_t vit_block_scratch_bytes(int64_t tokens, int64_t embed, int64_t mlp, int compute) {
    // A1 [T][E] + packed Q, K, V^T 3 [T][E] + fc2 operand [T][MLP], all f16;
    // in F32 mode the middle region holds the f32 qkv rows [T][3E] instead.
    // F32 mode also holds the TF32 hi / lo planes of K and V^T (4 x [T][E] f32)
    // for the tensor-core attention's TMA loads.
    const int64_t middle = compute == SAMQ_COMPUTE_F32 ? (3 + 4) * embed * 2 : 3 * embed;
    return static_cast<size_t>(tokens) * (embed + middle + mlp) * sizeof(__half) + 4 * 256;
}

void launch_ln_stage(const float* x, int64_t rows, int64_t embed, int grid_w, int window, const float* w,
                     const float* b, __half* a, DeviceState& state, cudaStream_t stream) {
    by_width(static_cast<int>(embed), [&](auto nv) {
        launch_pdl(ln_stage_kernel<decltype(nv)::value>, dim3(blocks_for(rows * 32)), dim3(256), 0, stream,
                   "ln_stage_kernel launch", x, rows, grid_w, window, w, b, a, state.status);
    });
}

void launch_vit_block(const VitBlockArgs& blk, float* x, int batch, int grid_w, int grid_h, void* scratch,
                      DeviceState& state, cudaStream_t stream) {
    const int64_t embed = blk.qkv->k, mlp = blk.fc1->n;
    const int heads = static_cast<int>(embed / 64);
    // A batch is one grid of batch * grid_h rows (images stacked): the LN1
    // window gather and the windowed attention see one tall grid, a global
    // block one attention group per image.
    const int64_t tokens = static_cast<int64_t>(batch) * grid_w * grid_h;
    const int group_n = blk.window > 0 ? blk.window * blk.window : grid_w * grid_h;
    const bool f32 = blk.compute == SAMQ_COMPUTE_F32;
    auto align = [](uintptr_t p) { return (p + 255) & ~uintptr_t(255); };
    uintptr_t cursor = align(reinterpret_cast<uintptr_t>(scratch));
    __half* a1 = reinterpret_cast<__half*>(cursor);
    cursor = align(cursor + tokens * embed * sizeof(__half));
    __half* packed = reinterpret_cast<__half*>(cursor);  // F16: Q, K, V^T; F32: the f32 qkv rows
    cursor = align(cursor + (f32 ? 3 * tokens * embed * sizeof(float) : 3 * tokens * embed * sizeof(__half)));
    float* planes = f32 ? reinterpret_cast<float*>(cursor) : nullptr;  // F32: K / V^T TF32 hi / lo planes
    if (f32) cursor = align(cursor + 4 * tokens * embed * sizeof(float));
    __half* a3 = reinterpret_cast<__half*>(cursor);
    __half* q = packed;
    __half* k = packed + tokens * embed;
    __half* vt = packed + 2 * tokens * embed;

    launch_ln_stage(x, tokens, embed, grid_w, blk.window, blk.norm1_w, blk.norm1_b, a1, state, stream);
    Epilogue ep;
    if (f32) {
        // F32 mode: the qkv linear's f32 output (rows window-major, as LN1
        // gathered them), then F32-precise RoPE + attention writing the proj
        // operand.
        float* qkv32 = reinterpret_cast<float*>(packed);
        ep.mode = kOutF32;
        ep.bias = blk.qkv_b;
        ep.y = qkv32;
        ep.ldy = 3 * embed;
        launch_gemm(a1, embed, blk.qkv->operand, tokens, 3 * embed, embed, ep, state, stream);
        if (mlp * 2 >= embed * 4) {
            // On the tensor cores (three-term TF32, attention_tc.cu): RoPE in
            // place on the f32 Q / K rows, one attention per window (or image),
            // f32 output rows in raster order in the fc2-operand region (free
            // until fc1), then the proj operand staged from them (K1).
            launch_rope_rows(qkv32, 3 * embed, embed, tokens, group_n, blk.freqs, stream);
            float* att32 = reinterpret_cast<float*>(a3);
            launch_attention_tc_groups(qkv32, 3 * embed, embed, static_cast<int>(tokens / group_n), group_n, heads, 64,
                                       0.125f, att32, embed, blk.window, grid_w, planes, state, stream);
            launch_act_f16(att32, tokens, embed, embed, a1, nullptr, state.status, stream);
        } else {
            launch_attention_f32(qkv32, 3 * embed, blk.window > 0, grid_w, grid_h, heads, blk.window, batch,
                                 blk.freqs, nullptr, a1, embed, state, stream);
        }
    } else {
        ep.mode = kOutQkvPack;
        ep.bias = blk.qkv_b;
        ep.q = q;
        ep.k = k;
        ep.vt = vt;
        ep.freqs = blk.freqs;
        ep.heads = heads;
        ep.group_n = group_n;
        launch_gemm(a1, embed, blk.qkv->operand, tokens, 3 * embed, embed, ep, state, stream);
        launch_attention_packed(q, k, vt, grid_w, grid_h, heads, blk.window, batch, nullptr, a1, embed, state,
                                stream);
    }
    ep = Epilogue{};
    ep.mode = kOutF32Residual;
    ep.bias = blk.proj_b;
    ep.y = x;
    ep.ldy = embed;
    ep.residual = x;
    ep.ldr = embed;
    launch_gemm(a1, embed, blk.proj->operand, tokens, embed, embed, ep, state, stream);
    launch_ln_stage(x, tokens, embed, grid_w, 0, blk.norm2_w, blk.norm2_b, a1, state, stream);
    ep = Epilogue{};
    ep.mode = kOutF16Staged;
    ep.gelu = 1;
    ep.bias = blk.fc1_b;
    ep.h = a3;
    ep.ldh = mlp;
    launch_gemm(a1, embed, blk.fc1->operand, tokens, mlp, embed, ep, state, stream);
    ep = Epilogue{};
    ep.mode = kOutF32Residual;
    ep.bias = blk.fc2_b;
    ep.y = x;
    ep.ldy = embed;
    ep.residual = x;
    ep.ldr = embed;
    launch_gemm(a3, mlp, blk.fc2->operand, tokens, embed, mlp, ep, state, stream);
}

size_t vit_prefix_scratch_bytes(int64_t tokens, int64_t embed, int patch, int compute) {
    if (compute == SAMQ_COMPUTE_F32) {
        // f32 columns [T][kp], their hi / lo split, and the weight's hi / lo.
        const int64_t kp = 3 * patch * patch;
        return static_cast<size_t>(3 * tokens + 2 * embed) * kp * sizeof(float) + 6 * 256;
    }
    const int64_t ld = (3 * patch * patch + 63) / 64 * 64;
    return static_cast<size_t>(tokens + embed) * ld * sizeof(__half) + 2 * 256;
}

void launch_vit_prefix(const float* image, int width, int height, int patch, const float* patch_w, int64_t embed,
                       const float* pos, int pos_grid, const float* ln_w, const float* ln_b, float* x, int compute,
                       void* scratch, DeviceState& state, cudaStream_t stream) {
    const int grid_w = width / patch, grid_h = height / patch;
    const int64_t tokens = static_cast<int64_t>(grid_w) * grid_h;
    const int kp = 3 * patch * patch;
    const int ld = (kp + 63) / 64 * 64;
    auto align = [](uintptr_t p) { return (p + 255) & ~uintptr_t(255); };
    uintptr_t cursor = align(reinterpret_cast<uintptr_t>(scratch));
    if (compute == SAMQ_COMPUTE_F32) {
        // F32 columns (sam3_conv_2d_sk_p0 with F32 im2col, ops.hpp:67-89), the
        // product with F32 semantics on the dense path (three-term TF32 split).
        auto take = [&](int64_t floats) {
            float* p = reinterpret_cast<float*>(cursor);
            cursor = align(cursor + floats * sizeof(float));
            return p;
        };
        float* cols = take(tokens * kp);
        float* ch = take(tokens * kp);
        float* cl = take(tokens * kp);
        float* wh = take(embed * kp);
        float* wl = take(embed * kp);
        launch_pdl(im2col_f32_kernel, dim3(blocks_for(tokens * (kp / 4))), dim3(256), 0, stream,
                   "im2col_f32_kernel launch", image, width, height, patch, grid_w, tokens, kp, cols);
        launch_split_rows(cols, tokens, kp, kp, ch, cl, state, stream);
        launch_split_rows(patch_w, embed, kp, kp, wh, wl, state, stream);
        samq_dense w;  // a view of the split weight in scratch (not owned)
        w.device = state.device;
        w.type = SAMQ_TYPE_F32;
        w.kind = SAMQ_DENSE_LINEAR;
        w.cin = kp;
        w.cout = embed;
        w.n = embed;
        w.k = kp;
        w.hi = wh;
        w.lo = wl;
        launch_dense_gemm(ch, cl, w, tokens, 0, 0, nullptr, 0, x, nullptr, embed, state, stream);
        by_width(static_cast<int>(embed), [&](auto nv) {
            launch_pdl(embed_ln_kernel<decltype(nv)::value>, dim3(blocks_for(tokens * 32)), dim3(256), 0, stream,
                       "embed_ln_kernel launch", x, tokens, grid_w, pos, pos_grid, ln_w, ln_b);
        });
        return;
    }
    __half* cols = reinterpret_cast<__half*>(cursor);
    cursor = align(cursor + tokens * ld * sizeof(__half));
    __half* wp = reinterpret_cast<__half*>(cursor);
    launch_pdl(im2col_kernel, dim3(blocks_for(tokens * (ld / 8))), dim3(256), 0, stream, "im2col_kernel launch", image,
               width, height, patch, grid_w, tokens, kp, ld, cols);
    launch_pdl(pad_f16_kernel, dim3(blocks_for(embed * ld)), dim3(256), 0, stream, "pad_f16_kernel launch", patch_w,
               embed, kp, ld, wp);
    Epilogue ep;
    ep.mode = kOutF32;
    ep.y = x;
    ep.ldy = embed;
    launch_gemm(cols, ld, wp, tokens, embed, ld, ep, state, stream);
    by_width(static_cast<int>(embed), [&](auto nv) {
        launch_pdl(embed_ln_kernel<decltype(nv)::value>, dim3(blocks_for(tokens * 32)), dim3(256), 0, stream,
                   "embed_ln_kernel launch", x, tokens, grid_w, pos, pos_grid, ln_w, ln_b);
    });
}

}  // namespace samq
