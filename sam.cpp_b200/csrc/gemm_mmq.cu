// gemm_mmq.cu -- the quantized linear with GGML MMQ's own arithmetic on the
// sm_100a tensor cores: Y[m][n] = sum over 32-value blocks b of
// d_w[n][b] * d_x[m][b] * (sum_k q_w[n][k] q_x[m][k]) + bias, the integer
// block dot exact and the per-block rescale in f32 (GGML CUDA mul_mat_q over
// Q8_0 weights and MMQ-D4 staged activations, contract
// tools/validation/verify_q8_mmq_dots.py:54-105 and the D4 staging of
// verify_q8_mmq_rhs_staging.py:24-67).
//
// K2 (gemm.cu) folds the scales into f16 operands, which rounds every decoded
// value to 11 bits.  Here the operands are the integer codes themselves and
// the tensor core computes each 32-value block's dot exactly into its own
// TMEM accumulator slot; the epilogue warps rescale every block and add it
// to f32 registers, so the result carries only f32 rounding.  Two variants
// share the kernel:
//   CODES_F16  the codes as f16 (exact for |q| <= 127): tcgen05.mma
//              kind::f16, K = 16, two MMAs per block, f32 accumulator (the
//              block dot, |sum| <= 32 * 127 * 127 < 2^24, is exact in f32);
//   CODES_I8   the codes as int8: tcgen05.mma kind::i8, K = 32, one MMA per
//              block, s32 accumulator, converted by the epilogue.
// Every block's accumulator has to be drained and rescaled: 2 f32 operations
// per output value per block, 256 FMA-pipe cycles per 128 x 128 block on an
// SM against 128 tensor cycles for the f16 MMAs (64 for int8), so the
// epilogue, not the tensor core, sets the pace.  Measured on B200 at the
// ViT-block shapes: ~0.2 of K2's speed for both variants alike (instruction
// issue bound, tensor pipe ~4% active): the int8 rate cannot be used behind
// a per-block drain, which is why K2 folds the scales into f16 operands.
// This path is the exact-arithmetic option (and has no activation range limit).
//
// Persistent, warp-specialised, one CTA per SM, 320 threads:
//   warp 0   TMA producer: 128-row A code tiles and 128-row B code tiles,
//            128-byte swizzle, one swizzle row (128 bytes) of K per stage;
//   warp 1   TMEM owner (4 slots x 128 columns) and MMA issuer: block b of
//            the stream goes to slot b % 4 once the epilogue released it;
//   warps 2-9 epilogue, two per TMEM lane quarter (64 columns each): wait for
//            a slot, load it (tcgen05.ld), release it, rescale into the f32
//            accumulators; after a tile's last block: bias (+ erf-GELU),
//            swizzled staging in shared memory, TMA store.
// No TMA load uses cluster multicast; every mbarrier wait is bounded.
#include <algorithm>

#include "samq_internal.hpp"

namespace samq {
namespace {

constexpr int QM = 128, QN = 128;
constexpr int kSlots = 4;
constexpr int kQEpiWarps = 8;                  // two per TMEM lane quarter
constexpr int kQCols = QN / (kQEpiWarps / 4);  // columns of a tile per epilogue warp
constexpr int kQThreads = 64 + 32 * kQEpiWarps;
constexpr int kQOutChunk = 32 * 32 * 4;
// Per epilogue warp, a ring of kScaleDepth blocks' scales (64 weight scales of
// its columns, 32 activation scales of its rows) filled by cp.async
// kScaleDepth - 1 blocks ahead of use, so no global load latency sits on a
// block's path.
constexpr int kScaleDepth = 4;
constexpr int kScaleEntry = kQCols + 32;       // weight scales of its columns, activation scales of its rows
constexpr int kScaleRing = kScaleDepth * kScaleEntry * 4;
constexpr uint32_t kQTmemCols = kSlots * QN;

template <int VARIANT>
struct MmqShape {
    static constexpr int elem = VARIANT == SAMQ_MMQ_CODES_I8 ? 1 : 2;
    static constexpr int bk = 128 / elem;                 // K per stage: one 128-byte swizzle row
    static constexpr int blocks = bk / 32;                // quant blocks per stage
    static constexpr int k_mma = 32 / elem;               // K of one MMA instruction
    static constexpr int mma_per_block = 32 / k_mma;
    static constexpr int tile_bytes = QM * 128;           // A or B tile of one stage
    static constexpr int stages = 5;
    static constexpr int a_off = 0;
    static constexpr int b_off = stages * tile_bytes;
    static constexpr int out_off = b_off + stages * tile_bytes;
    static constexpr int scale_off = out_off + kQEpiWarps * kQOutChunk;
    static constexpr int bar_off = scale_off + kQEpiWarps * kScaleRing;
    static constexpr int bar_bytes = (2 * stages + 2 * kSlots + 1) * 8 + 8;
    static constexpr int total = bar_off + bar_bytes + 1024;
};

// Instruction descriptors (K-major A and B, dense): D f32 from f16 inputs, or
// D s32 from signed 8-bit inputs.
__host__ __device__ constexpr uint32_t idesc_codes(int variant, int m, int n) {
    return variant == SAMQ_MMQ_CODES_I8
               ? (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
                     (static_cast<uint32_t>(m >> 4) << 24)
               : (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void cp_async_8(void* smem_dst, const void* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(smem_dst)), "l"(src),
                 "r"(valid ? 8 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_4(void* smem_dst, const void* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(smem_dst)), "l"(src),
                 "r"(valid ? 4 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void tc_mma_codes(int variant, uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
    if (variant == SAMQ_MMQ_CODES_I8) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        tc_mma_f16(tmem_d, adesc, bdesc, idesc, accumulate);
    }
}

struct MmqArgs {
    const float* dx;   // [k / 32][m] activation block scales
    const float* dw;   // [k / 32][n] weight block scales
    const float* bias;
    int gelu;
    int m, n, k;
    DeviceStatus* status;
};

template <int VARIANT>
__global__ void __launch_bounds__(kQThreads, 1)
gemm_mmq_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                const __grid_constant__ CUtensorMap tma_y, const MmqArgs args) {
    using S = MmqShape<VARIANT>;
    static_assert(S::total <= 232448, "shared memory budget");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sa = smem + S::a_off;
    uint8_t* sb = smem + S::b_off;
    uint8_t* sout = smem + S::out_off;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::bar_off);
    uint64_t* empty = full + S::stages;
    uint64_t* slot_full = empty + S::stages;
    uint64_t* slot_empty = slot_full + kSlots;
    uint64_t* drain = slot_empty + kSlots;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    DeviceStatus* status = args.status;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m = args.m, n = args.n;
    const int m_tiles = (m + QM - 1) / QM, n_tiles = (n + QN - 1) / QN;
    const int tiles = m_tiles * n_tiles;
    const int kstages = args.k / S::bk;
    const int nblocks = args.k / 32;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S::stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&slot_full[s], 1);
            mbar_init(&slot_empty[s], kQEpiWarps);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tma_a);
        tma_prefetch_desc(&tma_b);
        tma_prefetch_desc(&tma_y);
    }
    if (warp == 1) tmem_alloc(tmem_slot, kQTmemCols);
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
                const int mt = tile / n_tiles, nt = tile % n_tiles;
                for (int ks = 0; ks < kstages; ++ks) {
                    if (!mbar_wait(&empty[s], ph ^ 1u, status, 61)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], 2 * S::tile_bytes);
                    tma_load_2d(sa + s * S::tile_bytes, &tma_a, &full[s], ks * S::bk, mt * QM);
                    tma_load_2d(sb + s * S::tile_bytes, &tma_b, &full[s], ks * S::bk, nt * QN);
                    issued |= 1u << s;
                    issued_phase = (issued_phase & ~(1u << s)) | (ph << s);
                    if (++s == S::stages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            pdl_trigger();
            if (!ok)
                for (int i = 0; i < S::stages; ++i)
                    if (issued & (1u << i)) mbar_wait(&full[i], (issued_phase >> i) & 1u, status, 62);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_codes(VARIANT, QM, QN);
            int s = 0;
            uint32_t ph = 0;
            uint32_t g = 0;  // block counter over the whole stream: slot g % kSlots
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                for (int ks = 0; ks < kstages && ok; ++ks) {
                    if (!mbar_wait(&full[s], ph, status, 63)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sa + s * S::tile_bytes);
                    const uint32_t b_addr = smem_u32(sb + s * S::tile_bytes);
                    for (int blk = 0; blk < S::blocks; ++blk, ++g) {
                        const int slot = static_cast<int>(g % kSlots);
                        if (!mbar_wait(&slot_empty[slot], ((g / kSlots) & 1u) ^ 1u, status, 64)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t d = tmem_base + static_cast<uint32_t>(slot * QN);
#pragma unroll
                        for (int j = 0; j < S::mma_per_block; ++j) {
                            const uint32_t off = static_cast<uint32_t>((blk * S::mma_per_block + j) * 32);
                            tc_mma_codes(VARIANT, d, smem_desc_sw128(a_addr + off), smem_desc_sw128(b_addr + off),
                                         idesc, j != 0 ? 1u : 0u);
                        }
                        tc_commit(&slot_full[slot]);
                    }
                    tc_commit(&empty[s]);
                    if (++s == S::stages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            tc_commit(drain);
            mbar_wait(drain, 0, status, 65);
        }
    } else {
        const int quarter = warp & 3;
        const int part = (warp - 2) >> 2;  // columns kQCols * part .. of the tile
        uint8_t* stage_buf = sout + (warp - 2) * kQOutChunk;
        float* ring = reinterpret_cast<float*>(smem + S::scale_off + (warp - 2) * kScaleRing);
        // Block g of this warp's stream (its tiles' blocks in order) -> ring
        // entry g % kScaleDepth: 64 weight scales, then 32 activation scales.
        const int my_tiles = blockIdx.x < tiles ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
        const uint32_t total_blocks = static_cast<uint32_t>(my_tiles) * nblocks;
        auto prefetch = [&](uint32_t gb) {
            if (gb < total_blocks) {
                const int t = blockIdx.x + static_cast<int>(gb / nblocks) * gridDim.x;
                const int b = static_cast<int>(gb % nblocks);
                const int tm = t / n_tiles, tn = t % n_tiles;
                const int r = tm * QM + quarter * 32 + lane;
                float* e = ring + (gb % kScaleDepth) * kScaleEntry;
                if (kQCols == 64) {
                    const int c = tn * QN + part * 64 + 2 * lane;
                    cp_async_8(e + 2 * lane, args.dw + static_cast<int64_t>(b) * n + (c + 1 < n ? c : 0), c + 1 < n);
                } else {
                    const int c = tn * QN + part * kQCols + lane;
                    cp_async_4(e + lane, args.dw + static_cast<int64_t>(b) * n + (c < n ? c : 0), c < n);
                }
                cp_async_4(e + kQCols + lane, args.dx + static_cast<int64_t>(b) * m + (r < m ? r : 0), r < m);
            }
            cp_async_commit();  // an empty group keeps the wait count uniform
        };
        // n is even for Q8_0 rows of whole blocks (n % 2 == 0 is checked by the host).
        for (uint32_t gb = 0; gb < kScaleDepth - 1; ++gb) prefetch(gb);
        uint32_t g = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
            const int mt = tile / n_tiles, nt = tile % n_tiles;
            const int row0 = mt * QM + quarter * 32;
            const int col_base = nt * QN + part * kQCols;
            float acc[kQCols];
#pragma unroll
            for (int i = 0; i < kQCols; ++i) acc[i] = 0.0f;
            for (int b = 0; b < nblocks; ++b, ++g) {
                const int slot = static_cast<int>(g % kSlots);
                prefetch(g + kScaleDepth - 1);
                cp_async_wait<kScaleDepth - 1>();
                __syncwarp();
                const float* e = ring + (g % kScaleDepth) * kScaleEntry;
                const float dx = e[kQCols + lane];
                // Warp-uniform wait: tcgen05.ld is warp-collective.
                if (!__all_sync(0xffffffffu, mbar_wait(&slot_full[slot], (g / kSlots) & 1u, status, 66))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t t[kQCols];
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                       static_cast<uint32_t>(slot * QN + part * kQCols);
#pragma unroll
                for (int h = 0; h < kQCols / 32; ++h)
                    tc_ld_32x32b_x32(taddr + 32 * h, *reinterpret_cast<uint32_t(*)[32]>(t + 32 * h));
                tc_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&slot_empty[slot]);
#pragma unroll
                for (int c4 = 0; c4 < kQCols / 4; ++c4) {
                    const int c = c4 * 4;
                    const float4 w = *reinterpret_cast<const float4*>(e + c);
                    const uint32_t* src = t + c;
                    const float ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float v = VARIANT == SAMQ_MMQ_CODES_I8 ? static_cast<float>(static_cast<int32_t>(src[j]))
                                                                     : __uint_as_float(src[j]);
                        acc[c + j] = fmaf(v, ws[j] * dx, acc[c + j]);
                    }
                }
                __syncwarp();  // the ring entry is rewritten kScaleDepth - 1 blocks later
            }
            if (!ok) break;
            // Tile done: bias (+ erf-GELU), 32 x 32 chunks through shared memory, TMA store.
#pragma unroll
            for (int chunk = 0; chunk < kQCols / 32; ++chunk) {
                const int col0 = col_base + chunk * 32;
                if (col0 >= n) break;
                const float bias_lane = (args.bias != nullptr && col0 + lane < n) ? __ldg(args.bias + col0 + lane) : 0.0f;
                if (lane == 0) bulk_wait_group_read<0>();
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    float o[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        float x = acc[chunk * 32 + 4 * j + e] + __shfl_sync(0xffffffffu, bias_lane, 4 * j + e);
                        if (args.gelu) x = gelu_erf(x);
                        o[e] = x;
                    }
                    *reinterpret_cast<float4*>(stage_buf + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                        make_float4(o[0], o[1], o[2], o[3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0 && row0 < m) {
                    tma_store_2d(&tma_y, stage_buf, col0, row0);
                    bulk_commit_group();
                }
            }
        }
        cp_async_wait<0>();
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
    }
    tc_fence_before();
    // Reconverge each warp before the aligned CTA barrier (lane-0 role loops).
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kQTmemCols);
    }
}

// Activation staging for the exact path: MMQ-D4 rule (d = amax / 127 and
// q = round(x * 127 / amax), IEEE divisions, f32 scale), codes [rows][k] as
// f16 or int8, scales [k / 32][rows].  8 lanes per 32-value block, 4 values
// per lane.  Non-finite inputs are flagged (kStatusRange); there is no range
// limit otherwise.
template <int VARIANT>
__global__ void __launch_bounds__(256) mmq_stage_kernel(const float* __restrict__ x, int64_t rows, int64_t k,
                                                        int64_t ld, void* __restrict__ codes,
                                                        float* __restrict__ scales, DeviceStatus* status) {
    pdl_wait();
    pdl_trigger();
    const int64_t per_row = k / 4;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const bool active = idx < rows * per_row;  // k % 32 == 0: a block's 8 lanes share `active`
    const int64_t row = active ? idx / per_row : 0;
    const int64_t c4 = active ? idx - row * per_row : 0;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (active) v = __ldg(reinterpret_cast<const float4*>(x + row * ld) + c4);
    const bool bad = active && !(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w));
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float inv = amax == 0.0f ? 0.0f : __fdiv_rn(127.0f, amax);
    record_range(bad, status);
    if (!active) return;
    const float q0 = roundf(__fmul_rn(v.x, inv)), q1 = roundf(__fmul_rn(v.y, inv));
    const float q2 = roundf(__fmul_rn(v.z, inv)), q3 = roundf(__fmul_rn(v.w, inv));
    if (VARIANT == SAMQ_MMQ_CODES_I8) {
        const uint32_t word = (static_cast<uint32_t>(static_cast<int>(q0)) & 0xffu) |
                              ((static_cast<uint32_t>(static_cast<int>(q1)) & 0xffu) << 8) |
                              ((static_cast<uint32_t>(static_cast<int>(q2)) & 0xffu) << 16) |
                              ((static_cast<uint32_t>(static_cast<int>(q3)) & 0xffu) << 24);
        reinterpret_cast<uint32_t*>(codes)[row * per_row + c4] = word;
    } else {
        const __half2 h0 = __floats2half2_rn(q0, q1), h1 = __floats2half2_rn(q2, q3);
        reinterpret_cast<uint2*>(codes)[row * per_row + c4] =
            make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
    }
    if ((c4 & 7) == 0) scales[(c4 / 8) * rows + row] = d;
}

// Q8_0 GGUF rows -> weight codes [n][k] (f16 or int8) and scales [k / 32][n].
template <int VARIANT>
__global__ void __launch_bounds__(256) mmq_weights_kernel(const uint8_t* __restrict__ rows, int64_t n, int64_t k,
                                                          void* __restrict__ codes, float* __restrict__ scales) {
    const int64_t blocks = k / 32;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n * blocks;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / blocks, b = i - r * blocks;
        const uint8_t* blk = rows + (r * blocks + b) * 34;
        __half_raw hr;
        hr.x = static_cast<uint16_t>(blk[0] | (blk[1] << 8));
        scales[b * n + r] = __half2float(__half(hr));
        for (int j = 0; j < 32; ++j) {
            const int8_t q = static_cast<int8_t>(blk[2 + j]);
            if (VARIANT == SAMQ_MMQ_CODES_I8)
                static_cast<int8_t*>(codes)[r * k + b * 32 + j] = q;
            else
                static_cast<__half*>(codes)[r * k + b * 32 + j] = __int2half_rn(q);
        }
    }
}

}  // namespace

size_t mmq_code_bytes(int variant) { return variant == SAMQ_MMQ_CODES_I8 ? 1 : 2; }

void launch_mmq_weights(int variant, const uint8_t* rows, int64_t n, int64_t k, void* codes, float* scales,
                        cudaStream_t stream) {
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n * (k / 32) + 255) / 256, 148 * 16));
    if (variant == SAMQ_MMQ_CODES_I8)
        mmq_weights_kernel<SAMQ_MMQ_CODES_I8><<<grid, 256, 0, stream>>>(rows, n, k, codes, scales);
    else
        mmq_weights_kernel<SAMQ_MMQ_CODES_F16><<<grid, 256, 0, stream>>>(rows, n, k, codes, scales);
    check_cuda(cudaGetLastError(), "mmq_weights_kernel launch");
}

void launch_mmq_stage(int variant, const float* x, int64_t rows, int64_t k, int64_t ld, void* codes, float* scales,
                      DeviceStatus* status, cudaStream_t stream) {
    if (rows == 0) return;
    const dim3 grid(static_cast<unsigned>((rows * (k / 4) + 255) / 256));
    if (variant == SAMQ_MMQ_CODES_I8)
        launch_pdl(mmq_stage_kernel<SAMQ_MMQ_CODES_I8>, grid, dim3(256), 0, stream, "mmq_stage_kernel launch", x,
                   rows, k, ld, codes, scales, status);
    else
        launch_pdl(mmq_stage_kernel<SAMQ_MMQ_CODES_F16>, grid, dim3(256), 0, stream, "mmq_stage_kernel launch", x,
                   rows, k, ld, codes, scales, status);
}

void launch_mmq_gemm(int variant, const void* a_codes, const float* dx, const void* b_codes, const float* dw,
                     int64_t m, int64_t n, int64_t k, const float* bias, int gelu, float* y, int64_t ldy,
                     DeviceState& state, cudaStream_t stream) {
    if (m == 0) return;
    const CUtensorMapDataType dt =
        variant == SAMQ_MMQ_CODES_I8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int elem = variant == SAMQ_MMQ_CODES_I8 ? 1 : 2;
    CUtensorMap ta, tb, ty;
    encode_tensor_map_2d(&ta, dt, a_codes, k, m, k * elem, 128 / elem, QM, CU_TENSOR_MAP_SWIZZLE_128B);
    encode_tensor_map_2d(&tb, dt, b_codes, k, n, k * elem, 128 / elem, QN, CU_TENSOR_MAP_SWIZZLE_128B);
    encode_tensor_map_2d(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, y, n, m, ldy * 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
    MmqArgs args{dx, dw, bias, gelu, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), state.status};
    const int64_t tiles = ((m + QM - 1) / QM) * ((n + QN - 1) / QN);
    const int grid = static_cast<int>(tiles < state.sm_count ? tiles : state.sm_count);
    if (variant == SAMQ_MMQ_CODES_I8) {
        using S = MmqShape<SAMQ_MMQ_CODES_I8>;
        set_smem_limit_once(state, reinterpret_cast<const void*>(gemm_mmq_kernel<SAMQ_MMQ_CODES_I8>), S::total,
                            "cudaFuncSetAttribute(gemm_mmq smem)");
        launch_pdl(gemm_mmq_kernel<SAMQ_MMQ_CODES_I8>, dim3(grid), dim3(kQThreads), S::total, stream,
                   "gemm_mmq_kernel launch", ta, tb, ty, args);
    } else {
        using S = MmqShape<SAMQ_MMQ_CODES_F16>;
        set_smem_limit_once(state, reinterpret_cast<const void*>(gemm_mmq_kernel<SAMQ_MMQ_CODES_F16>), S::total,
                            "cudaFuncSetAttribute(gemm_mmq smem)");
        launch_pdl(gemm_mmq_kernel<SAMQ_MMQ_CODES_F16>, dim3(grid), dim3(kQThreads), S::total, stream,
                   "gemm_mmq_kernel launch", ta, tb, ty, args);
    }
}

}  // namespace samq
