// attention_f32.cu -- F32-precise RoPE + windowed / global attention of a SAM 3
// ViT block (the reference's default CudaComputeMode::F32).
//
// The reference's CUDA backend runs ViT attention at GGML_PREC_F32 unless the
// F16 compute mode is selected (src/runtime/ggml/backends/cuda.hpp:82-92,
// 156-189): F32 Q, K and V, F32 products (cuBLAS SGEMM in the SAM patch,
// cmake/patches/ggml-precise-cuda.patch:448-606) and an F32 softmax, checked by
// a closed-form probe at 1e-5 (tests/runtime/ggml/test_precision.cpp:68-126).
// Here every operand stays f32 and the products run on the FP32 pipe:
//   rope_f32_kernel       sam3_apply_rope (src/models/sam3/vision.hpp:100-148)
//                         with GGML's op sequence and rounding: re*cos and
//                         im*sin are separate f32 products, then one f32
//                         subtraction (ggml_mul, ggml_mul, ggml_sub), and
//                         likewise re*sin + im*cos.
//   attention_f32_kernel  one CTA per (64 queries, head, group): Q (RoPE'd,
//                         x 1/8, exact as 1/8 is a power of two) held in
//                         shared memory, K (RoPE'd) and V staged 64 keys at a
//                         time, S = Q K^T and O += P V as 4 x 4 register
//                         tiles per thread over float4 shared-memory loads,
//                         online softmax with expf, O / l at the end.  The
//                         output is f32 in raster token order or, in the ViT
//                         block, the proj linear's Q8_1-staged f16 operand.
// Window partition / unpartition (ggml_win_part / win_unpart,
// vision.hpp:170-173,225-227) are the same address maps as in attention.cu.
// No waits on other CTAs, so nothing here can hang.
#include <algorithm>

#include "samq_internal.hpp"

namespace samq {
namespace {

constexpr int kHd = 64;
constexpr int kTile = 64;       // queries per CTA and keys per step
constexpr int kPitch = 68;      // shared-memory row pitch (floats): conflict-free float4 columns
constexpr int kF32Threads = 256;
constexpr int kF32Smem = 4 * kTile * kPitch * 4;  // Q, K, V^T, P

struct GeometryF32 {
    int grid_w, grid_h, heads, window;
    int groups, group_n;
    int qkv_window_major;  // qkv rows stored window-major (g * group_n + n) instead of raster
};

__device__ __forceinline__ int raster_token(const GeometryF32& geo, int g, int n) {
    if (geo.window == 0) return g * geo.group_n + n;
    const int per_row = geo.grid_w / geo.window;
    const int wy = g / per_row, wx = g % per_row;
    const int ly = n / geo.window, lx = n % geo.window;
    return (wy * geo.window + ly) * geo.grid_w + wx * geo.window + lx;
}

__device__ __forceinline__ int qkv_row(const GeometryF32& geo, int g, int n) {
    return geo.qkv_window_major ? g * geo.group_n + n : raster_token(geo, g, n);
}

// GGML's RoPE arithmetic for the pairs (x0, x1) and (x2, x3) of a float4.
__device__ __forceinline__ float4 rope4(float4 x, float4 f) {
    float4 r;
    r.x = __fsub_rn(__fmul_rn(x.x, f.x), __fmul_rn(x.y, f.y));
    r.y = __fadd_rn(__fmul_rn(x.x, f.y), __fmul_rn(x.y, f.x));
    r.z = __fsub_rn(__fmul_rn(x.z, f.z), __fmul_rn(x.w, f.w));
    r.w = __fadd_rn(__fmul_rn(x.z, f.w), __fmul_rn(x.w, f.z));
    return r;
}

__global__ void __launch_bounds__(256) rope_f32_kernel(const float* __restrict__ x, const float* __restrict__ freqs,
                                                       int64_t tokens, int64_t head_batches, float* __restrict__ out) {
    const int64_t units = head_batches * tokens * (kHd / 4);
    for (int64_t u = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; u < units; u += int64_t(gridDim.x) * blockDim.x) {
        const int64_t c4 = u % (kHd / 4);
        const int64_t token = (u / (kHd / 4)) % tokens;
        const float4 v = __ldg(reinterpret_cast<const float4*>(x) + u);
        const float4 f = __ldg(reinterpret_cast<const float4*>(freqs + (token * (kHd / 2) + c4 * 2) * 2));
        reinterpret_cast<float4*>(out)[u] = rope4(v, f);
    }
}

// In place on f32 qkv rows [rows][ldq] (Q at columns 0.., K at embed..): the
// RoPE of sam3_apply_rope for token position r % group_n of every row r.
__global__ void __launch_bounds__(256) rope_rows_kernel(float* __restrict__ qkv, int64_t ldq, int64_t embed,
                                                        int64_t rows, int group_n, const float* __restrict__ freqs) {
    const int64_t per_row = 2 * embed / 4;  // float4 units of Q and K
    const int64_t units = rows * per_row;
    for (int64_t u = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; u < units; u += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = u / per_row, c4 = u - r * per_row;
        const int64_t pos = r % group_n;
        const int64_t col = c4 * 4;  // Q: col, K: col (>= embed)
        const int64_t in_head = (col % embed) % kHd;
        float4* p = reinterpret_cast<float4*>(qkv + r * ldq + col);
        const float4 f = __ldg(reinterpret_cast<const float4*>(freqs + (pos * (kHd / 2) + in_head / 2) * 2));
        *p = rope4(*p, f);
    }
}

__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
    acc = fmaf(a.z, b.z, acc);
    return fmaf(a.w, b.w, acc);
}

template <bool STAGED>
__global__ void __launch_bounds__(kF32Threads, 2)
attention_f32_kernel(const float* __restrict__ qkv, int64_t ldq, const float* __restrict__ freqs, GeometryF32 geo,
                     float* __restrict__ out, __half* __restrict__ out_h, int64_t ldo, DeviceStatus* status) {
    extern __shared__ float4 smem_f4[];
    float* qs = reinterpret_cast<float*>(smem_f4);   // [64 queries][kPitch]
    float* ks = qs + kTile * kPitch;                 // [64 keys][kPitch]
    float* vt = ks + kTile * kPitch;                 // [64 dims][kPitch]  (V transposed)
    float* ps = vt + kTile * kPitch;                 // [64 queries][kPitch]
    const int t = threadIdx.x;
    const int rq = t >> 4, u = t & 15;               // rows 4rq..4rq+3; keys / dims u + 16j
    const int q0 = blockIdx.x * kTile, h = blockIdx.y, g = blockIdx.z;
    const int E = geo.heads * kHd;
    pdl_wait();

    // Q: RoPE by the query's position in its group, x 1/8 (exact).
    for (int idx = t; idx < kTile * 16; idx += kF32Threads) {
        const int r = idx >> 4, c4 = idx & 15, n = q0 + r;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (n < geo.group_n) {
            const float4 x = __ldg(reinterpret_cast<const float4*>(qkv + int64_t(qkv_row(geo, g, n)) * ldq + h * kHd) + c4);
            const float4 f = __ldg(reinterpret_cast<const float4*>(freqs + (int64_t(n) * (kHd / 2) + c4 * 2) * 2));
            v = rope4(x, f);
            v.x *= 0.125f;
            v.y *= 0.125f;
            v.z *= 0.125f;
            v.w *= 0.125f;
        }
        *reinterpret_cast<float4*>(qs + r * kPitch + c4 * 4) = v;
    }

    float o[4][4], m[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) o[i][j] = 0.0f;
    }
    const int kblocks = (geo.group_n + kTile - 1) / kTile;
    for (int kb = 0; kb < kblocks; ++kb) {
        __syncthreads();  // previous step's K, V^T and P reads are done (and Q is written)
        for (int idx = t; idx < kTile * 16; idx += kF32Threads) {
            const int r = idx >> 4, c4 = idx & 15, n = kb * kTile + r;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (n < geo.group_n) {
                const float4 x =
                    __ldg(reinterpret_cast<const float4*>(qkv + int64_t(qkv_row(geo, g, n)) * ldq + E + h * kHd) + c4);
                const float4 f = __ldg(reinterpret_cast<const float4*>(freqs + (int64_t(n) * (kHd / 2) + c4 * 2) * 2));
                v = rope4(x, f);
            }
            *reinterpret_cast<float4*>(ks + r * kPitch + c4 * 4) = v;
        }
        for (int idx = t; idx < kTile * 16; idx += kF32Threads) {
            const int r = idx & 63, d4 = idx >> 6, n = kb * kTile + r;  // consecutive lanes: consecutive keys
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (n < geo.group_n)
                v = __ldg(reinterpret_cast<const float4*>(qkv + int64_t(qkv_row(geo, g, n)) * ldq + 2 * E + h * kHd) + d4);
            vt[(4 * d4 + 0) * kPitch + r] = v.x;
            vt[(4 * d4 + 1) * kPitch + r] = v.y;
            vt[(4 * d4 + 2) * kPitch + r] = v.z;
            vt[(4 * d4 + 3) * kPitch + r] = v.w;
        }
        __syncthreads();

        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll 4
        for (int d4 = 0; d4 < 16; ++d4) {
            float4 a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4*>(qs + (4 * rq + i) * kPitch + 4 * d4);
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(ks + (u + 16 * j) * kPitch + 4 * d4);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) s[i][j] = dot4(a[i], b[j], s[i][j]);
        }
        // Online softmax of the 4 rows; a row's 64 scores sit on 16 neighbouring lanes.
        float alpha[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (kb * kTile + u + 16 * j >= geo.group_n) s[i][j] = -INFINITY;
                mx = fmaxf(mx, s[i][j]);
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m[i], mx);
            alpha[i] = expf(m[i] - m_new);
            float sum = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float p = expf(s[i][j] - m_new);
                ps[(4 * rq + i) * kPitch + u + 16 * j] = p;
                sum += p;
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            l[i] = fmaf(l[i], alpha[i], sum);
            m[i] = m_new;
        }
        __syncthreads();
        // This tile's P V in fresh accumulators, added to the running O once:
        // a long sequential sum over thousands of keys would let f32 rounding
        // grow with the key count (the reference's closed-form probe at 5184
        // keys needs the blocked sum to stay within 1e-5).
        float ot[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) ot[i][j] = 0.0f;
#pragma unroll 4
        for (int k4 = 0; k4 < 16; ++k4) {
            float4 a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4*>(ps + (4 * rq + i) * kPitch + 4 * k4);
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(vt + (u + 16 * j) * kPitch + 4 * k4);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) ot[i][j] = dot4(a[i], b[j], ot[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) o[i][j] = fmaf(o[i][j], alpha[i], ot[i][j]);
    }
    pdl_trigger();

    if constexpr (!STAGED) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int n = q0 + 4 * rq + i;
            if (n >= geo.group_n) continue;
            float* row = out + int64_t(raster_token(geo, g, n)) * ldo + h * kHd;
#pragma unroll
            for (int j = 0; j < 4; ++j) row[u + 16 * j] = __fdiv_rn(o[i][j], l[i]);
        }
    } else {
        // O / l through shared memory, then each warp stages whole rows: lane
        // holds channels 2 lane, 2 lane + 1, so one Q8_1 block is 16 lanes.
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) ps[(4 * rq + i) * kPitch + u + 16 * j] = __fdiv_rn(o[i][j], l[i]);
        __syncthreads();
        const int warp = t >> 5, lane = t & 31;
        for (int r = warp; r < kTile; r += kF32Threads / 32) {
            const int n = q0 + r;
            if (n >= geo.group_n) break;  // warp-uniform
            const float2 v2 = *reinterpret_cast<const float2*>(ps + r * kPitch + 2 * lane);
            const float v[2] = {v2.x, v2.y};
            uint32_t packed[1];
            const bool bad = stage_q8_1<16, 2>(v, packed);
            record_range(bad, status);
            *reinterpret_cast<uint32_t*>(out_h + int64_t(raster_token(geo, g, n)) * ldo + h * kHd + 2 * lane) = packed[0];
        }
    }
}

// ---- general attention (text encoder, fusion / decoder attention) ----------
//
// softmax(scale * Q K^T + bias) V per head with F32 operands, GGML
// flash_attn_ext semantics at GGML_PREC_F32: Q [lq][ldq], K [lk][ldk],
// V [lk][ldv] with head h at columns h*HD .. h*HD + HD - 1; out [lq][ldo] the
// same.  The mask is additive: bias[h * bias_h + q * bias_q + k] (a per-key
// padding mask has bias_h = bias_q = 0; box relative-position biases vary with
// both), and `causal` masks keys k > q (the text encoder's triangular mask).
// A row whose keys are all masked yields 0.  One CTA per (64 queries, head);
// the 4 x 4 register tiles and the per-tile blocked P V sums of the ViT kernel.
struct AttnGenArgs {
    const float* q;
    const float* k;
    const float* v;
    const float* bias;
    float* out;
    int64_t ldq, ldk, ldv, ldo, bias_h, bias_q;
    int lq, lk, causal;
    float scale;
    // Key split (few queries, many keys): CTA z covers keys [z kps, (z + 1) kps)
    // and writes its unnormalized output and (max, sum) to part
    // [splits][heads][lq][HD + 2]; attention_combine_kernel merges them.
    float* part;
    int kps;
};

template <int HD>
__global__ void __launch_bounds__(kF32Threads, 2) attention_gen_kernel(AttnGenArgs a) {
    constexpr int kP = HD + 4;    // Q / K row pitch (floats)
    constexpr int kJ = HD / 16;   // output channels per thread
    extern __shared__ float4 smem_f4[];
    float* qs = reinterpret_cast<float*>(smem_f4);  // [64][kP]
    float* ks = qs + kTile * kP;                    // [64][kP]
    float* vt = ks + kTile * kP;                    // [HD][kPitch]
    float* ps = vt + HD * kPitch;                   // [64][kPitch]
    const int t = threadIdx.x;
    const int rq = t >> 4, u = t & 15;
    const int q0 = blockIdx.x * kTile, h = blockIdx.y;
    pdl_wait();
    for (int idx = t; idx < kTile * (HD / 4); idx += kF32Threads) {
        const int r = idx / (HD / 4), c4 = idx % (HD / 4), n = q0 + r;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (n < a.lq) v = __ldg(reinterpret_cast<const float4*>(a.q + int64_t(n) * a.ldq + h * HD) + c4);
        *reinterpret_cast<float4*>(qs + r * kP + c4 * 4) = v;
    }
    float o[4][kJ], m[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int j = 0; j < kJ; ++j) o[i][j] = 0.0f;
    }
    int kend = a.lk;
    if (a.causal) kend = min(kend, q0 + kTile);
    int kb_begin = 0;
    if (a.part != nullptr) {
        kb_begin = static_cast<int>(blockIdx.z) * (a.kps / kTile);
        kend = min(kend, static_cast<int>(blockIdx.z + 1) * a.kps);
    }
    const int kblocks = (kend + kTile - 1) / kTile;
    for (int kb = kb_begin; kb < kblocks; ++kb) {
        __syncthreads();
        for (int idx = t; idx < kTile * (HD / 4); idx += kF32Threads) {
            const int r = idx / (HD / 4), c4 = idx % (HD / 4), n = kb * kTile + r;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (n < a.lk) v = __ldg(reinterpret_cast<const float4*>(a.k + int64_t(n) * a.ldk + h * HD) + c4);
            *reinterpret_cast<float4*>(ks + r * kP + c4 * 4) = v;
        }
        for (int idx = t; idx < kTile * (HD / 4); idx += kF32Threads) {
            const int r = idx & 63, d4 = idx >> 6, n = kb * kTile + r;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (n < a.lk) v = __ldg(reinterpret_cast<const float4*>(a.v + int64_t(n) * a.ldv + h * HD) + d4);
            vt[(4 * d4 + 0) * kPitch + r] = v.x;
            vt[(4 * d4 + 1) * kPitch + r] = v.y;
            vt[(4 * d4 + 2) * kPitch + r] = v.z;
            vt[(4 * d4 + 3) * kPitch + r] = v.w;
        }
        __syncthreads();
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll
        for (int d4 = 0; d4 < HD / 4; ++d4) {
            float4 qa[4], kb4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) qa[i] = *reinterpret_cast<const float4*>(qs + (4 * rq + i) * kP + 4 * d4);
#pragma unroll
            for (int j = 0; j < 4; ++j) kb4[j] = *reinterpret_cast<const float4*>(ks + (u + 16 * j) * kP + 4 * d4);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) s[i][j] = dot4(qa[i], kb4[j], s[i][j]);
        }
        float alpha[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int qn = q0 + 4 * rq + i;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int kn = kb * kTile + u + 16 * j;
                float sv = s[i][j] * a.scale;
                if (kn >= a.lk || (a.causal && kn > qn)) sv = -INFINITY;
                else if (a.bias && qn < a.lq) sv += __ldg(a.bias + h * a.bias_h + int64_t(qn) * a.bias_q + kn);
                s[i][j] = sv;
                mx = fmaxf(mx, sv);
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m[i], mx);
            // All keys so far masked: keep the row empty (no NaN from -inf - -inf).
            const float m_use = m_new == -INFINITY ? 0.0f : m_new;
            alpha[i] = expf(m[i] - m_use);
            float sum = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float p = expf(s[i][j] - m_use);
                ps[(4 * rq + i) * kPitch + u + 16 * j] = p;
                sum += p;
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            l[i] = fmaf(l[i], alpha[i], sum);
            m[i] = m_new;
        }
        __syncthreads();
        float ot[4][kJ];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < kJ; ++j) ot[i][j] = 0.0f;
#pragma unroll 4
        for (int k4 = 0; k4 < 16; ++k4) {
            float4 pa[4], vb[kJ];
#pragma unroll
            for (int i = 0; i < 4; ++i) pa[i] = *reinterpret_cast<const float4*>(ps + (4 * rq + i) * kPitch + 4 * k4);
#pragma unroll
            for (int j = 0; j < kJ; ++j) vb[j] = *reinterpret_cast<const float4*>(vt + (u + 16 * j) * kPitch + 4 * k4);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < kJ; ++j) ot[i][j] = dot4(pa[i], vb[j], ot[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < kJ; ++j) o[i][j] = fmaf(o[i][j], alpha[i], ot[i][j]);
    }
    pdl_trigger();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int n = q0 + 4 * rq + i;
        if (n >= a.lq) continue;
        if (a.part != nullptr) {
            float* row = a.part + ((int64_t(blockIdx.z) * gridDim.y + h) * a.lq + n) * (HD + 2);
#pragma unroll
            for (int j = 0; j < kJ; ++j) row[u + 16 * j] = o[i][j];
            if (u == 0) {
                row[HD] = m[i];
                row[HD + 1] = l[i];
            }
            continue;
        }
        float* row = a.out + int64_t(n) * a.ldo + h * HD;
#pragma unroll
        for (int j = 0; j < kJ; ++j) row[u + 16 * j] = l[i] > 0.0f ? __fdiv_rn(o[i][j], l[i]) : 0.0f;
    }
}

// Merges the key splits of attention_gen_kernel: one warp per (head, query),
// M = max_s m_s, L = sum_s l_s e^(m_s - M), out = sum_s o_s e^(m_s - M) / L
// (0 for a row whose keys are all masked), the online softmax's own rescale.
template <int HD>
__global__ void __launch_bounds__(256) attention_combine_kernel(const float* __restrict__ part, int splits, int heads,
                                                                int lq, float* __restrict__ out, int64_t ldo) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (row >= int64_t(heads) * lq) return;
    const int h = static_cast<int>(row / lq), n = static_cast<int>(row % lq);
    const int64_t split_stride = int64_t(heads) * lq * (HD + 2);
    const float* base = part + row * (HD + 2);
    float mx = -INFINITY;
    for (int s = 0; s < splits; ++s) mx = fmaxf(mx, base[s * split_stride + HD]);
    const float m_use = mx == -INFINITY ? 0.0f : mx;
    constexpr int kC = HD / 32;
    float acc[kC], sum = 0.0f;
#pragma unroll
    for (int c = 0; c < kC; ++c) acc[c] = 0.0f;
    for (int s = 0; s < splits; ++s) {
        const float* p = base + s * split_stride;
        const float w = expf(p[HD] - m_use);
        sum = fmaf(p[HD + 1], w, sum);
#pragma unroll
        for (int c = 0; c < kC; ++c) acc[c] = fmaf(p[lane + 32 * c], w, acc[c]);
    }
    float* dst = out + int64_t(n) * ldo + h * HD;
#pragma unroll
    for (int c = 0; c < kC; ++c) dst[lane + 32 * c] = sum > 0.0f ? __fdiv_rn(acc[c], sum) : 0.0f;
}

// Key splits for lq queries x lk keys over `heads`: enough CTAs for two per SM
// when the query tiles alone do not fill the GPU, at least 2 key tiles each.
int key_splits(int lq, int lk, int heads, int causal, int sms) {
    if (causal) return 1;
    const int ctas = (lq + kTile - 1) / kTile * heads;
    const int tiles = (lk + kTile - 1) / kTile;
    if (ctas >= sms || tiles < 4) return 1;
    int splits = std::min({(2 * sms + ctas - 1) / ctas, tiles / 2, 64});
    if (splits < 2) return 1;
    const int per = (tiles + splits - 1) / splits;
    return (tiles + per - 1) / per;
}

GeometryF32 make_geometry_f32(int grid_w, int grid_h, int heads, int window, int batch, bool window_major) {
    GeometryF32 geo{grid_w, grid_h * batch, heads, window, batch, grid_w * grid_h, window_major ? 1 : 0};
    if (window > 0) {
        geo.groups = (grid_w / window) * (grid_h * batch / window);
        geo.group_n = window * window;
    }
    return geo;
}

}  // namespace

void launch_attention_f32(const float* qkv, int64_t ldq, bool qkv_window_major, int grid_w, int grid_h, int heads,
                          int window, int batch, const float* freqs, float* out, __half* out_h, int64_t ldo,
                          DeviceState& state, cudaStream_t stream) {
    const GeometryF32 geo = make_geometry_f32(grid_w, grid_h, heads, window, batch, qkv_window_major);
    const dim3 grid((geo.group_n + kTile - 1) / kTile, heads, geo.groups);
    if (out_h) {
        set_smem_limit_once(state, reinterpret_cast<const void*>(attention_f32_kernel<true>), kF32Smem,
                            "cudaFuncSetAttribute(attention_f32 smem)");
        launch_pdl(attention_f32_kernel<true>, grid, dim3(kF32Threads), kF32Smem, stream,
                   "attention_f32_kernel launch", qkv, ldq, freqs, geo, out, out_h, ldo, state.status);
    } else {
        set_smem_limit_once(state, reinterpret_cast<const void*>(attention_f32_kernel<false>), kF32Smem,
                            "cudaFuncSetAttribute(attention_f32 smem)");
        launch_pdl(attention_f32_kernel<false>, grid, dim3(kF32Threads), kF32Smem, stream,
                   "attention_f32_kernel launch", qkv, ldq, freqs, geo, out, out_h, ldo, state.status);
    }
}

size_t attention_gen_plane_bytes(int lq, int lk, int heads, int head_dim, int causal, const float* bias,
                                 const float* out, int64_t ldo) {
    return attention_tc_eligible(lq, lk, head_dim, causal, bias, out, ldo)
               ? attention_tc_scratch_bytes(lq, lk, heads, head_dim)
               : 0;
}

size_t attention_partial_floats(int lq, int lk, int heads, int head_dim, int causal, int sms) {
    const int splits = key_splits(lq, lk, heads, causal, sms);
    return splits > 1 ? static_cast<size_t>(splits) * heads * lq * (head_dim + 2) : 0;
}

void launch_attention_gen(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                          int lq, int lk, int heads, int head_dim, float scale, int causal, const float* bias,
                          int64_t bias_h, int64_t bias_q, float* out, int64_t ldo, DeviceState& state,
                          cudaStream_t stream, float* partials, size_t partial_floats, float* tc_planes) {
    if (lq == 0) return;
    if (attention_tc_eligible(lq, lk, head_dim, causal, bias, out, ldo)) {
        launch_attention_tc(q, ldq, k, ldk, v, ldv, lq, lk, heads, head_dim, scale, out, ldo, tc_planes, state, stream);
        return;
    }
    AttnGenArgs a{q, k, v, bias, out, ldq, ldk, ldv, ldo, bias_h, bias_q, lq, lk, causal, scale, nullptr, 0};
    int splits = key_splits(lq, lk, heads, causal, state.sm_count);
    if (partials == nullptr || partial_floats < attention_partial_floats(lq, lk, heads, head_dim, causal, state.sm_count))
        splits = 1;
    if (splits > 1) {
        const int tiles = (lk + kTile - 1) / kTile;
        a.kps = (tiles + splits - 1) / splits * kTile;
        a.part = partials;
    }
    const dim3 grid((lq + kTile - 1) / kTile, heads, splits);
    const unsigned combine_blocks = static_cast<unsigned>((int64_t(heads) * lq * 32 + 255) / 256);
    if (head_dim == 64) {
        constexpr int smem = (2 * kTile * 68 + 64 * kPitch + kTile * kPitch) * 4;
        set_smem_limit_once(state, reinterpret_cast<const void*>(attention_gen_kernel<64>), smem,
                            "cudaFuncSetAttribute(attention_gen smem)");
        launch_pdl(attention_gen_kernel<64>, grid, dim3(kF32Threads), smem, stream, "attention_gen_kernel launch", a);
        if (splits > 1)
            launch_pdl(attention_combine_kernel<64>, dim3(combine_blocks), dim3(256), 0, stream,
                       "attention_combine_kernel launch", static_cast<const float*>(partials), splits, heads, lq, out,
                       ldo);
    } else {
        constexpr int smem = (2 * kTile * 36 + 32 * kPitch + kTile * kPitch) * 4;
        set_smem_limit_once(state, reinterpret_cast<const void*>(attention_gen_kernel<32>), smem,
                            "cudaFuncSetAttribute(attention_gen smem)");
        launch_pdl(attention_gen_kernel<32>, grid, dim3(kF32Threads), smem, stream, "attention_gen_kernel launch", a);
        if (splits > 1)
            launch_pdl(attention_combine_kernel<32>, dim3(combine_blocks), dim3(256), 0, stream,
                       "attention_combine_kernel launch", static_cast<const float*>(partials), splits, heads, lq, out,
                       ldo);
    }
}

void launch_attention_combine(const float* part, int splits, int heads, int lq, int head_dim, float* out,
                              int64_t ldo, cudaStream_t stream) {
    const unsigned blocks = static_cast<unsigned>((int64_t(heads) * lq * 32 + 255) / 256);
    if (head_dim == 64)
        launch_pdl(attention_combine_kernel<64>, dim3(blocks), dim3(256), 0, stream, "attention_combine_kernel launch",
                   part, splits, heads, lq, out, ldo);
    else
        launch_pdl(attention_combine_kernel<32>, dim3(blocks), dim3(256), 0, stream, "attention_combine_kernel launch",
                   part, splits, heads, lq, out, ldo);
}

void launch_rope_rows(float* qkv, int64_t ldq, int64_t embed, int64_t rows, int group_n, const float* freqs,
                      cudaStream_t stream) {
    const int64_t units = rows * (2 * embed / 4);
    if (units == 0) return;
    const int64_t blocks = std::min<int64_t>((units + 255) / 256, int64_t(148) * 16);
    rope_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(qkv, ldq, embed, rows, group_n, freqs);
    check_cuda(cudaGetLastError(), "rope_rows_kernel launch");
}

void launch_rope_f32(const float* x, const float* freqs, int64_t tokens, int64_t head_batches, float* out,
                     cudaStream_t stream) {
    const int64_t units = head_batches * tokens * (kHd / 4);
    if (units == 0) return;
    const int64_t blocks = std::min<int64_t>((units + 255) / 256, int64_t(148) * 16);
    rope_f32_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x, freqs, tokens, head_batches, out);
    check_cuda(cudaGetLastError(), "rope_f32_kernel launch");
}

}  // namespace samq
