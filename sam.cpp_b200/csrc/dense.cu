// dense.cu -- F32-semantics dense linears and convolutions (the modules SAM.cpp
// keeps unquantized: the SimpleFPN neck, fusion / decoder linears) on the
// sm_100a tensor cores.
//
// Semantics: ggml_mul_mat on F32 (or F16) weights x F32 activations at
// GGML_PREC_F32, which the reference routes to cuBLAS with
// CUBLAS_COMPUTE_32F_PEDANTIC (cmake/patches/ggml-precise-cuda.patch:288-356),
// and sam3_conv_2d / sam3_deconv_2x2 over F32 im2col columns
// (src/models/sam3/ops.hpp:67-117).  The neck composition is
// sam3_build_neck_graph (src/models/sam3/vision.hpp:307-366).
//
// F32 accuracy from the TF32 tensor cores: every operand x is split once into
// hi = rna_tf32(x) and lo = rna_tf32(x - hi) (x - hi is exact in f32), and a
// tile accumulates hi*hi + hi*lo + lo*hi with tcgen05.mma kind::tf32 in f32
// TMEM.  The dropped lo*lo term and the rounding of lo are ~2^-22 of each
// product, the order of an f32 product's own rounding.  Weights are split at
// load time, activations by the producer of each operand (a split kernel, the
// max-pool kernel, or the epilogue of the previous layer, which writes hi/lo
// directly), so the GEMM reads four operand tiles per k-block and converts
// nothing.
//
// dense_gemm_kernel: persistent, warp-specialised, one CTA per SM, 192 threads:
//   warp 0     TMA producer: A hi/lo (128 rows x 32 f32, 128-byte swizzle) and
//              B hi/lo (128 rows x 32 f32) per stage, 3 stages.  In the
//              convolution mode the A tile of output pixels (8 rows x 16
//              columns of the image) and tap (ky, kx) is a 3-D box of the
//              NHWC input at (c0, x0 + kx - pad, y0 + ky - pad): TMA zero-fills
//              the padding, so the implicit im2col costs no extra pass.
//   warp 1     TMEM owner and MMA issuer: 3 x 4 tcgen05.mma (M=128, N=128,
//              K=8) per k-block: hi*hi into a segment accumulator that is
//              handed to the epilogue every kSegBlocks k-blocks, hi*lo +
//              lo*hi into a per-tile correction accumulator.
//   warps 2-9  epilogue, two per TMEM lane quarter (64 columns each): the
//              running f32 sum of the segments (round-to-nearest), then the
//              corrections, bias, erf-GELU (erff, as GGML's F32 gelu_erf), and
//              the store: f32 rows, or the hi/lo
//              split of the next layer's operand; rows are remapped for the
//              2x2 deconvolution's pixel shuffle and the convolution's pixel
//              tiles.
// No TMA load uses cluster multicast; every mbarrier wait is bounded.
#include <algorithm>

#include "samq_internal.hpp"

namespace samq {
namespace {

constexpr int DM = 128;                    // tile rows (MMA M)
constexpr int DN = 128;                    // tile columns (MMA N)
constexpr int DK = 32;                     // f32 per k-block: one 128-byte swizzle row
constexpr int kStages = 3;
constexpr int kEpiWarps = 8;               // two per TMEM lane quarter, 64 columns each
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer, MMA, epilogue
constexpr int kPart = DM * 128;            // one operand tile: 128 rows x 128 B
constexpr int kStageBytes = 4 * kPart;     // A hi, A lo, B hi, B lo
constexpr int kBarOff = kStages * kStageBytes;
constexpr int kSmemTotal = kBarOff + 256 + 1024;  // + barriers + alignment slack
// The tensor cores' f32 accumulation rounds toward zero once per MMA, an
// error that grows with K.  So the hi*hi products accumulate in TMEM only over
// segments of kSegBlocks k-blocks (two ping-pong segment buffers, columns
// 0..2DN-1); the epilogue warps add the segments in registers with f32
// round-to-nearest.  The hi*lo + lo*hi corrections (2^-11 of the products)
// accumulate over the whole K in their own double-buffered accumulator
// (columns 2DN..4DN-1).
// Four k-blocks (16 MMAs) per segment: an error within ~1.2x of an f32 SGEMM's
// (two: ~0.8x, 7% slower; eight: ~2x).
constexpr int kSegBlocks = 4;
constexpr uint32_t kCorrCol = 2 * DN;
constexpr uint32_t kTmemCols = 4 * DN;

// Conv pixel tile: 8 image rows x 16 columns = 128 GEMM rows.
constexpr int kTileH = 8, kTileW = 16;

// Instruction descriptor: kind::tf32, A/B tf32, D f32, both K-major.
constexpr uint32_t idesc_tf32(int m, int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// ggml_gelu_erf in f32: 0.5 x (1 + erf(x / sqrt 2)).
__device__ __forceinline__ float gelu_erf_f32(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

struct DenseGeom {
    int m, n, k;          // GEMM rows, columns, depth (conv: taps * cin)
    int conv;             // A: 0 rows of a [m][k] matrix, 1 pixel tiles of an NHWC image
    int width, height;    // conv: image size
    int ksize, pad, cin;  // conv
    int tiles_x;          // conv: 16-column blocks per image row
    int m_tiles, n_tiles;
};

enum : int { kMapRows = 0, kMapDeconv = 1, kMapConv = 2 };

struct DenseOut {
    float* y;             // f32 output, or hi of the split output
    float* y_lo;          // lo of the split output (nullptr: f32 output)
    int64_t ldy;
    const float* bias;    // [n] (deconv: [cout])
    int gelu;
    int map;
    int cout;             // deconv: output channels per tap
    int width;            // deconv: input width; conv: image width
    int height;           // conv: image height
};

__device__ __forceinline__ void store_chunk(float* dst, float* dst_lo, const float (&v)[32], int valid_cols) {
    if (valid_cols >= 32) {
        if (dst_lo == nullptr) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
                reinterpret_cast<float4*>(dst)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float h[4], l[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) split_tf32(v[4 * j + e], h[e], l[e]);
                reinterpret_cast<float4*>(dst)[j] = make_float4(h[0], h[1], h[2], h[3]);
                reinterpret_cast<float4*>(dst_lo)[j] = make_float4(l[0], l[1], l[2], l[3]);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if (i < valid_cols) {
                if (dst_lo == nullptr) {
                    dst[i] = v[i];
                } else {
                    float h, l;
                    split_tf32(v[i], h, l);
                    dst[i] = h;
                    dst_lo[i] = l;
                }
            }
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1)
dense_gemm_kernel(const __grid_constant__ CUtensorMap tm_ah, const __grid_constant__ CUtensorMap tm_al,
                  const __grid_constant__ CUtensorMap tm_bh, const __grid_constant__ CUtensorMap tm_bl,
                  const DenseGeom geo, const DenseOut out, DeviceStatus* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff);
    uint64_t* empty = full + kStages;
    uint64_t* seg_full = empty + kStages;  // [2]
    uint64_t* seg_empty = seg_full + 2;    // [2]
    uint64_t* corr_full = seg_empty + 2;   // [2]
    uint64_t* corr_empty = corr_full + 2;  // [2]
    uint64_t* drain = corr_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles = geo.m_tiles * geo.n_tiles;
    const int kblocks = (geo.k + DK - 1) / DK;
    const int cblocks = geo.cin / DK;  // conv: k-blocks per tap
    const int segments = (kblocks + kSegBlocks - 1) / kSegBlocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&seg_full[b], 1);
            mbar_init(&seg_empty[b], kEpiWarps);
            mbar_init(&corr_full[b], 1);
            mbar_init(&corr_empty[b], kEpiWarps);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tm_ah);
        tma_prefetch_desc(&tm_al);
        tma_prefetch_desc(&tm_bh);
        tma_prefetch_desc(&tm_bl);
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0, issued = 0, issued_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                const int mt = tile / geo.n_tiles, nt = tile % geo.n_tiles;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1u, status, 41)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + s * kStageBytes;
                    mbar_arrive_expect_tx(&full[s], kStageBytes);
                    if (geo.conv) {
                        const int tap = kb / cblocks, cb = kb - tap * cblocks;
                        const int ky = tap / geo.ksize, kx = tap - ky * geo.ksize;
                        const int ty = mt / geo.tiles_x, tx = mt - ty * geo.tiles_x;
                        const int x0 = tx * kTileW + kx - geo.pad, y0 = ty * kTileH + ky - geo.pad;
                        tma_load_3d(st, &tm_ah, &full[s], cb * DK, x0, y0);
                        tma_load_3d(st + kPart, &tm_al, &full[s], cb * DK, x0, y0);
                    } else {
                        tma_load_2d(st, &tm_ah, &full[s], kb * DK, mt * DM);
                        tma_load_2d(st + kPart, &tm_al, &full[s], kb * DK, mt * DM);
                    }
                    tma_load_2d(st + 2 * kPart, &tm_bh, &full[s], kb * DK, nt * DN);
                    tma_load_2d(st + 3 * kPart, &tm_bl, &full[s], kb * DK, nt * DN);
                    issued |= 1u << s;
                    issued_phase = (issued_phase & ~(1u << s)) | (ph << s);
                    if (++s == kStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            pdl_trigger();
            if (!ok) {
                for (int i = 0; i < kStages; ++i)
                    if (issued & (1u << i)) mbar_wait(&full[i], (issued_phase >> i) & 1u, status, 45);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32(DM, DN);
            int s = 0, sb = 0, cb = 0;
            uint32_t ph = 0, s_ph = 0, c_ph = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                if (!mbar_wait(&corr_empty[cb], c_ph ^ 1u, status, 42)) break;
                const uint32_t dc = tmem_base + kCorrCol + static_cast<uint32_t>(cb * DN);
                int kb = 0;
                for (int seg = 0; seg < segments && ok; ++seg) {
                    if (!mbar_wait(&seg_empty[sb], s_ph ^ 1u, status, 47)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem_base + static_cast<uint32_t>(sb * DN);
                    const int kb_begin = kb, kb_end = min(kb + kSegBlocks, kblocks);
                    for (; kb < kb_end; ++kb) {
                        if (!mbar_wait(&full[s], ph, status, 43)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t ah = smem_u32(smem + s * kStageBytes);
                        const uint32_t al = ah + kPart, bh = ah + 2 * kPart, bl = ah + 3 * kPart;
#pragma unroll
                        for (int kk = 0; kk < DK / 8; ++kk) {
                            const uint32_t off = static_cast<uint32_t>(kk) * 32;
                            tc_mma_tf32(dc, smem_desc_sw128(ah + off), smem_desc_sw128(bl + off), idesc,
                                        (kb | kk) != 0 ? 1u : 0u);
                            tc_mma_tf32(dc, smem_desc_sw128(al + off), smem_desc_sw128(bh + off), idesc, 1u);
                            tc_mma_tf32(d, smem_desc_sw128(ah + off), smem_desc_sw128(bh + off), idesc,
                                        (kb != kb_begin || kk != 0) ? 1u : 0u);
                        }
                        tc_commit(&empty[s]);
                        if (++s == kStages) {
                            s = 0;
                            ph ^= 1u;
                        }
                    }
                    if (!ok) break;
                    tc_commit(&seg_full[sb]);
                    sb ^= 1;
                    if (sb == 0) s_ph ^= 1u;
                }
                if (!ok) break;
                tc_commit(&corr_full[cb]);
                cb ^= 1;
                if (cb == 0) c_ph ^= 1u;
            }
            tc_commit(drain);
            mbar_wait(drain, 0, status, 46);
        }
    } else {
        // Epilogue warps 2..9: TMEM lane quarter warp % 4, column half
        // (warp - 2) / 4 of the tile (64 columns).
        const int quarter = warp & 3, half = (warp - 2) >> 2;
        const int r = quarter * 32 + lane;  // row of the tile
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        int sb = 0, cb = 0;
        uint32_t s_ph = 0, c_ph = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
            const int mt = tile / geo.n_tiles, nt = tile % geo.n_tiles;
            // The hi*hi segments, summed here in f32 with round-to-nearest.
            float sum[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) sum[i] = 0.0f;
            for (int seg = 0; seg < segments; ++seg) {
                // Warp-uniform: tcgen05.ld is warp-collective.
                if (!__all_sync(0xffffffffu, mbar_wait(&seg_full[sb], s_ph, status, 48))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t a0[32], a1[32];
                const uint32_t taddr = tmem_base + lane_off + static_cast<uint32_t>(sb * DN + half * 64);
                tc_ld_32x32b_x32(taddr, a0);
                tc_ld_32x32b_x32(taddr + 32, a1);
                tc_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&seg_empty[sb]);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    sum[i] = __fadd_rn(sum[i], __uint_as_float(a0[i]));
                    sum[32 + i] = __fadd_rn(sum[32 + i], __uint_as_float(a1[i]));
                }
                sb ^= 1;
                if (sb == 0) s_ph ^= 1u;
            }
            if (!ok || !__all_sync(0xffffffffu, mbar_wait(&corr_full[cb], c_ph, status, 44))) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t c0[32], c1[32];
            const uint32_t caddr = tmem_base + lane_off + kCorrCol + static_cast<uint32_t>(cb * DN + half * 64);
            tc_ld_32x32b_x32(caddr, c0);
            tc_ld_32x32b_x32(caddr + 32, c1);
            tc_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&corr_empty[cb]);
            cb ^= 1;
            if (cb == 0) c_ph ^= 1u;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                sum[i] = __fadd_rn(sum[i], __uint_as_float(c0[i]));
                sum[32 + i] = __fadd_rn(sum[32 + i], __uint_as_float(c1[i]));
            }
            // Destination pixel / row of this lane.
            int64_t row = -1;  // -1: no output row
            int in_y = 0, in_x = 0;
            if (out.map == kMapConv) {
                const int ty = mt / geo.tiles_x, tx = mt - ty * geo.tiles_x;
                const int py = ty * kTileH + (r >> 4), px = tx * kTileW + (r & 15);
                if (py < out.height && px < out.width) row = static_cast<int64_t>(py) * out.width + px;
            } else {
                const int m_row = mt * DM + r;
                if (m_row < geo.m) {
                    row = m_row;
                    if (out.map == kMapDeconv) {
                        in_y = m_row / out.width;
                        in_x = m_row - in_y * out.width;
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int col0 = nt * DN + half * 64 + c * 32;
                if (col0 >= geo.n) break;
                int bcol = col0, tap = 0;
                if (out.map == kMapDeconv) {
                    tap = col0 / out.cout;
                    bcol = col0 - tap * out.cout;
                }
                const float b_lane =
                    (out.bias != nullptr && col0 + lane < geo.n) ? __ldg(out.bias + bcol + lane) : 0.0f;
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    float x = __fadd_rn(sum[c * 32 + i], __shfl_sync(0xffffffffu, b_lane, i));
                    if (out.gelu) x = gelu_erf_f32(x);
                    v[i] = x;
                }
                if (row < 0) continue;
                int64_t dst_row = row;
                if (out.map == kMapDeconv)
                    dst_row = static_cast<int64_t>(2 * in_y + (tap >> 1)) * (2 * out.width) + 2 * in_x + (tap & 1);
                const int64_t off = dst_row * out.ldy + bcol;
                store_chunk(out.y + off, out.y_lo ? out.y_lo + off : nullptr, v, geo.n - col0);
            }
        }
    }
    tc_fence_before();
    // Reconverge each warp before the aligned CTA barrier (lane-0 role loops).
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ---------------------------------------------------------------- operand prep

// x [rows][ld] f32 -> hi, lo [rows][k] (k % 4 == 0).
__global__ void __launch_bounds__(256) split_rows_kernel(const float* __restrict__ x, int64_t rows, int64_t k,
                                                         int64_t ld, float* __restrict__ hi, float* __restrict__ lo) {
    pdl_wait();
    pdl_trigger();
    const int64_t per_row = k / 4;
    const int64_t total = rows * per_row;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t rr = i / per_row, c4 = i - rr * per_row;
        const float4 v = __ldg(reinterpret_cast<const float4*>(x + rr * ld) + c4);
        float4 h, l;
        split_tf32(v.x, h.x, l.x);
        split_tf32(v.y, h.y, l.y);
        split_tf32(v.z, h.z, l.z);
        split_tf32(v.w, h.w, l.w);
        reinterpret_cast<float4*>(hi + rr * k)[c4] = h;
        reinterpret_cast<float4*>(lo + rr * k)[c4] = l;
    }
}

// 2x2 / stride 2 max pooling of an NHWC image; with lo != nullptr the output
// is written as the hi / lo split of the next convolution's operand.
__global__ void __launch_bounds__(256) maxpool2x2_kernel(const float* __restrict__ x, int width, int height,
                                                         int64_t channels, float* __restrict__ y,
                                                         float* __restrict__ lo) {
    pdl_wait();
    pdl_trigger();
    const int ow = width / 2, oh = height / 2;
    const int64_t c4n = channels / 4;
    const int64_t total = static_cast<int64_t>(ow) * oh * c4n;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t pix = i / c4n, c4 = i - pix * c4n;
        const int oy = static_cast<int>(pix / ow), ox = static_cast<int>(pix - static_cast<int64_t>(oy) * ow);
        const float4* base = reinterpret_cast<const float4*>(x);
        const int64_t p00 = (static_cast<int64_t>(2 * oy) * width + 2 * ox) * c4n + c4;
        const float4 a = __ldg(base + p00), b = __ldg(base + p00 + c4n);
        const float4 c = __ldg(base + p00 + static_cast<int64_t>(width) * c4n),
                     d = __ldg(base + p00 + static_cast<int64_t>(width) * c4n + c4n);
        float4 m;
        m.x = fmaxf(fmaxf(a.x, b.x), fmaxf(c.x, d.x));
        m.y = fmaxf(fmaxf(a.y, b.y), fmaxf(c.y, d.y));
        m.z = fmaxf(fmaxf(a.z, b.z), fmaxf(c.z, d.z));
        m.w = fmaxf(fmaxf(a.w, b.w), fmaxf(c.w, d.w));
        if (lo == nullptr) {
            reinterpret_cast<float4*>(y)[i] = m;
        } else {
            float4 h, l;
            split_tf32(m.x, h.x, l.x);
            split_tf32(m.y, h.y, l.y);
            split_tf32(m.z, h.z, l.z);
            split_tf32(m.w, h.w, l.w);
            reinterpret_cast<float4*>(y)[i] = h;
            reinterpret_cast<float4*>(lo)[i] = l;
        }
    }
}

// Weights in their GGML layout (f32 or f16) -> hi / lo [n][k] GEMM operand:
//   LINEAR    [k, n]: B[n][k] = W[n][k]
//   CONV      [ks, ks, cin, cout]: B[co][(ky ks + kx) cin + ci] = W[co][ci][ky][kx]
//   DECONV2X2 [2, 2, cout, cin]:   B[(2 ky + kx) cout + co][ci] = W[ci][co][ky][kx]
__global__ void __launch_bounds__(256) dense_prep_kernel(const void* __restrict__ src, int type, int kind, int ks,
                                                         int64_t cin, int64_t cout, int64_t n, int64_t k,
                                                         float* __restrict__ hi, float* __restrict__ lo) {
    const int64_t total = n * k;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t nn = i / k, kk = i - nn * k;
        int64_t s = i;
        if (kind == SAMQ_DENSE_CONV) {
            const int64_t tap = kk / cin, ci = kk - tap * cin;
            const int64_t ky = tap / ks, kx = tap - ky * ks;
            s = ((nn * cin + ci) * ks + ky) * ks + kx;
        } else if (kind == SAMQ_DENSE_DECONV2X2) {
            const int64_t tap = nn / cout, co = nn - tap * cout;
            s = ((kk * cout + co) * 2 + (tap >> 1)) * 2 + (tap & 1);
        }
        const float v = type == SAMQ_TYPE_F16 ? __half2float(static_cast<const __half*>(src)[s])
                                              : static_cast<const float*>(src)[s];
        float h, l;
        split_tf32(v, h, l);
        hi[i] = h;
        lo[i] = l;
    }
}

int grid_for(int64_t work, const DeviceState& state) {
    const int64_t blocks = (work + 255) / 256;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, int64_t(state.sm_count) * 8)));
}

}  // namespace

void launch_dense_prep(const void* src, int type, int kind, int ks, int64_t cin, int64_t cout, int64_t n, int64_t k,
                       float* hi, float* lo, DeviceState& state, cudaStream_t stream) {
    dense_prep_kernel<<<grid_for(n * k, state), 256, 0, stream>>>(src, type, kind, ks, cin, cout, n, k, hi, lo);
    check_cuda(cudaGetLastError(), "dense_prep_kernel launch");
}

void launch_split_rows(const float* x, int64_t rows, int64_t k, int64_t ld, float* hi, float* lo, DeviceState& state,
                       cudaStream_t stream) {
    if (rows == 0) return;
    launch_pdl(split_rows_kernel, dim3(grid_for(rows * (k / 4), state)), dim3(256), 0, stream,
               "split_rows_kernel launch", x, rows, k, ld, hi, lo);
}

void launch_maxpool2x2(const float* x, int width, int height, int64_t channels, float* y, float* lo,
                       DeviceState& state, cudaStream_t stream) {
    const int64_t work = static_cast<int64_t>(width / 2) * (height / 2) * (channels / 4);
    if (work == 0) return;
    launch_pdl(maxpool2x2_kernel, dim3(grid_for(work, state)), dim3(256), 0, stream, "maxpool2x2_kernel launch", x,
               width, height, channels, y, lo);
}

// A operand: hi / lo [m][k] rows (lda = k), or NHWC images [height][width][cin]
// (conv); B operand: hi / lo [n][k].
void launch_dense_gemm(const float* a_hi, const float* a_lo, const samq_dense& w, int64_t m, int conv_width,
                       int conv_height, const float* bias, int gelu, float* y, float* y_lo, int64_t ldy,
                       DeviceState& state, cudaStream_t stream) {
    DenseGeom geo{};
    geo.n = static_cast<int>(w.n);
    geo.k = static_cast<int>(w.k);
    geo.cin = static_cast<int>(w.cin);
    DenseOut out{};
    out.y = y;
    out.y_lo = y_lo;
    out.ldy = ldy;
    out.bias = bias;
    out.gelu = gelu;
    out.cout = static_cast<int>(w.cout);
    CUtensorMap tah, tal, tbh, tbl;
    if (w.kind == SAMQ_DENSE_CONV && w.ks > 1) {
        geo.conv = 1;
        geo.width = conv_width;
        geo.height = conv_height;
        geo.ksize = w.ks;
        geo.pad = w.ks / 2;
        geo.m = conv_width * conv_height;
        geo.tiles_x = (conv_width + kTileW - 1) / kTileW;
        geo.m_tiles = geo.tiles_x * ((conv_height + kTileH - 1) / kTileH);
        out.map = kMapConv;
        out.width = conv_width;
        out.height = conv_height;
        for (int part = 0; part < 2; ++part)
            encode_tensor_map_3d_box(part == 0 ? &tah : &tal, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, part == 0 ? a_hi : a_lo,
                                     w.cin, conv_width, conv_height, w.cin * 4, w.cin * 4 * conv_width, DK, kTileW,
                                     kTileH, CU_TENSOR_MAP_SWIZZLE_128B);
    } else {
        // Rows: linears, 1x1 convolutions (m = pixels) and the 2x2
        // deconvolution (m = input pixels, conv_width = input width).
        if (m <= 0) return;
        geo.m = static_cast<int>(m);
        geo.m_tiles = static_cast<int>((m + DM - 1) / DM);
        out.map = w.kind == SAMQ_DENSE_DECONV2X2 ? kMapDeconv : kMapRows;
        out.width = conv_width;  // deconv: input width
        encode_tensor_map_2d(&tah, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a_hi, w.k, m, w.k * 4, DK, DM,
                             CU_TENSOR_MAP_SWIZZLE_128B);
        encode_tensor_map_2d(&tal, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a_lo, w.k, m, w.k * 4, DK, DM,
                             CU_TENSOR_MAP_SWIZZLE_128B);
    }
    encode_tensor_map_2d(&tbh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.hi, w.k, w.n, w.k * 4, DK, DN,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    encode_tensor_map_2d(&tbl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.lo, w.k, w.n, w.k * 4, DK, DN,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    geo.n_tiles = static_cast<int>((w.n + DN - 1) / DN);
    const int64_t tiles = static_cast<int64_t>(geo.m_tiles) * geo.n_tiles;
    if (tiles == 0) return;
    set_smem_limit_once(state, reinterpret_cast<const void*>(dense_gemm_kernel), kSmemTotal,
                        "cudaFuncSetAttribute(dense smem)");
    const int grid = static_cast<int>(std::min<int64_t>(tiles, state.sm_count));
    launch_pdl(dense_gemm_kernel, dim3(grid), dim3(kThreads), kSmemTotal, stream, "dense_gemm_kernel launch", tah,
               tal, tbh, tbl, geo, out, state.status);
}

// ---------------------------------------------------------------- neck

namespace {

struct NeckDims {
    int64_t embed, mid, d;
};

NeckDims neck_dims(const samq_neck_v1& nk) {
    const samq_dense* all[12] = {nk.s0_deconv1, nk.s0_deconv2, nk.s0_conv1x1, nk.s0_conv3x3,
                                 nk.s1_deconv1, nk.s1_conv1x1, nk.s1_conv3x3, nk.s2_conv1x1,
                                 nk.s2_conv3x3, nk.s3_conv1x1, nk.s3_conv3x3, nullptr};
    for (int i = 0; i < 11; ++i)
        if (all[i] == nullptr) fail(SAMQ_ERR_INVALID_ARGUMENT, "neck weight missing");
    auto is = [](const samq_dense* w, int kind, int ks) { return w->kind == kind && (kind != SAMQ_DENSE_CONV || w->ks == ks); };
    const int64_t E = nk.s0_deconv1->cin, D = nk.s0_conv3x3->cout;
    bool ok = is(nk.s0_deconv1, SAMQ_DENSE_DECONV2X2, 0) && is(nk.s0_deconv2, SAMQ_DENSE_DECONV2X2, 0) &&
              is(nk.s0_conv1x1, SAMQ_DENSE_CONV, 1) && is(nk.s0_conv3x3, SAMQ_DENSE_CONV, 3) &&
              is(nk.s1_deconv1, SAMQ_DENSE_DECONV2X2, 0) && is(nk.s1_conv1x1, SAMQ_DENSE_CONV, 1) &&
              is(nk.s1_conv3x3, SAMQ_DENSE_CONV, 3) && is(nk.s2_conv1x1, SAMQ_DENSE_CONV, 1) &&
              is(nk.s2_conv3x3, SAMQ_DENSE_CONV, 3) && is(nk.s3_conv1x1, SAMQ_DENSE_CONV, 1) &&
              is(nk.s3_conv3x3, SAMQ_DENSE_CONV, 3);
    if (!ok) fail(SAMQ_ERR_INVALID_ARGUMENT, "neck weight of the wrong kind");
    ok = nk.s0_deconv2->cin == nk.s0_deconv1->cout && nk.s0_deconv2->cout == D && nk.s0_conv1x1->cin == D &&
         nk.s0_conv1x1->cout == D && nk.s0_conv3x3->cin == D && nk.s1_deconv1->cin == E &&
         nk.s1_conv1x1->cin == nk.s1_deconv1->cout && nk.s1_conv1x1->cout == D && nk.s1_conv3x3->cin == D &&
         nk.s1_conv3x3->cout == D && nk.s2_conv1x1->cin == E && nk.s2_conv1x1->cout == D &&
         nk.s2_conv3x3->cin == D && nk.s2_conv3x3->cout == D && nk.s3_conv1x1->cin == E &&
         nk.s3_conv1x1->cout == D && nk.s3_conv3x3->cin == D && nk.s3_conv3x3->cout == D;
    if (!ok) fail(SAMQ_ERR_INVALID_ARGUMENT, "neck channel counts do not chain");
    return {E, std::max(nk.s0_deconv1->cout, nk.s1_deconv1->cout), D};
}

// Floats of one intermediate buffer (hi and lo halves).
int64_t neck_buffer_floats(const NeckDims& dm, int64_t tokens) {
    return std::max({4 * tokens * dm.mid, 16 * tokens * dm.d, (tokens / 4 + 1) * dm.embed});
}

}  // namespace

size_t neck_scratch_bytes(const samq_neck_v1& neck, int grid_w, int grid_h) {
    const NeckDims dm = neck_dims(neck);
    const int64_t tokens = static_cast<int64_t>(grid_w) * grid_h;
    return static_cast<size_t>(2 * tokens * dm.embed + 4 * neck_buffer_floats(dm, tokens)) * sizeof(float) + 1024;
}

// sam3_build_neck_graph (src/models/sam3/vision.hpp:307-366), NHWC throughout:
// every intermediate is written by its producer's epilogue as the hi / lo
// split its consumer reads.  Two buffers alternate between the layers.
void launch_neck(const samq_neck_v1& nk, const float* x, int gw, int gh, float* const out[4], void* scratch,
                 DeviceState& state, cudaStream_t stream) {
    const NeckDims dm = neck_dims(nk);
    const int64_t T = static_cast<int64_t>(gw) * gh;
    const int64_t bf = neck_buffer_floats(dm, T);
    float* base = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(scratch) + 255) & ~uintptr_t(255));
    float* xh = base;
    float* xl = xh + T * dm.embed;
    float* b1h = xl + T * dm.embed;
    float* b1l = b1h + bf;
    float* b2h = b1l + bf;
    float* b2l = b2h + bf;
    launch_split_rows(x, T, dm.embed, dm.embed, xh, xl, state, stream);
    auto gemm_rows = [&](const float* ah, const float* al, const samq_dense* w, int64_t m, int in_w, const float* b,
                         int gelu, float* yh, float* yl) {
        launch_dense_gemm(ah, al, *w, m, in_w, 0, b, gelu, yh, yl, w->cout, state, stream);
    };
    auto conv3 = [&](const float* ah, const float* al, const samq_dense* w, int wd, int ht, const float* b, float* y) {
        launch_dense_gemm(ah, al, *w, static_cast<int64_t>(wd) * ht, wd, ht, b, 0, y, nullptr, w->cout, state, stream);
    };
    // Scale 0 (4x): deconv, GELU, deconv, conv1x1, conv3x3.
    gemm_rows(xh, xl, nk.s0_deconv1, T, gw, nk.s0_deconv1_b, 1, b1h, b1l);
    gemm_rows(b1h, b1l, nk.s0_deconv2, 4 * T, 2 * gw, nk.s0_deconv2_b, 0, b2h, b2l);
    gemm_rows(b2h, b2l, nk.s0_conv1x1, 16 * T, 0, nk.s0_conv1x1_b, 0, b1h, b1l);
    conv3(b1h, b1l, nk.s0_conv3x3, 4 * gw, 4 * gh, nk.s0_conv3x3_b, out[0]);
    // Scale 1 (2x): deconv, conv1x1, conv3x3.
    gemm_rows(xh, xl, nk.s1_deconv1, T, gw, nk.s1_deconv1_b, 0, b1h, b1l);
    gemm_rows(b1h, b1l, nk.s1_conv1x1, 4 * T, 0, nk.s1_conv1x1_b, 0, b2h, b2l);
    conv3(b2h, b2l, nk.s1_conv3x3, 2 * gw, 2 * gh, nk.s1_conv3x3_b, out[1]);
    // Scale 2 (1x): conv1x1, conv3x3.
    gemm_rows(xh, xl, nk.s2_conv1x1, T, 0, nk.s2_conv1x1_b, 0, b1h, b1l);
    conv3(b1h, b1l, nk.s2_conv3x3, gw, gh, nk.s2_conv3x3_b, out[2]);
    // Scale 3 (0.5x): 2x2 max pool of the ViT output, conv1x1, conv3x3.
    const int pw = gw / 2, ph = gh / 2;
    launch_maxpool2x2(x, gw, gh, dm.embed, b1h, b1l, state, stream);
    gemm_rows(b1h, b1l, nk.s3_conv1x1, static_cast<int64_t>(pw) * ph, 0, nk.s3_conv1x1_b, 0, b2h, b2l);
    conv3(b2h, b2l, nk.s3_conv3x3, pw, ph, nk.s3_conv3x3_b, out[3]);
}

}  // namespace samq
