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
// per output value per block (a packed f32x2 multiply and fused add), so the
// epilogue, not the tensor core, sets the pace.  This is the trade the f16
// path avoids; the kernel measures it.
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
constexpr int kQEpiWarps = 8;
constexpr int kQThreads = 64 + 32 * kQEpiWarps;
constexpr int kQOutChunk = 32 * 32 * 4;
constexpr uint32_t kQTmemCols = kSlots * QN;

template <int VARIANT>
struct MmqShape {
    static constexpr int elem = VARIANT == SAMQ_MMQ_CODES_I8 ? 1 : 2;
    static constexpr int bk = 128 / elem;                 // K per stage: one 128-byte swizzle row
    static constexpr int blocks = bk / 32;                // quant blocks per stage
    static constexpr int k_mma = 32 / elem;               // K of one MMA instruction
    static constexpr int mma_per_block = 32 / k_mma;
    static constexpr int tile_bytes = QM * 128;           // A or B tile of one stage
    static constexpr int stages = 6;
    static constexpr int a_off = 0;
    static constexpr int b_off = stages * tile_bytes;
    static constexpr int out_off = b_off + stages * tile_bytes;
    static constexpr int bar_off = out_off + kQEpiWarps * kQOutChunk;
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

// acc += t * s for two f32 pairs (packed f32x2 FMA on sm_100).
__device__ __forceinline__ void fma2(float& a0, float& a1, float t0, float t1, float s0, float s1) {
    uint64_t acc, t, s;
    asm("mov.b64 %0, {%1, %2};" : "=l"(acc) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(t) : "f"(t0), "f"(t1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(s) : "f"(s0), "f"(s1));
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(t), "l"(s));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(acc));
}

__device__ __forceinline__ void mul2(float& r0, float& r1, float a0, float a1, float b) {
    uint64_t r, a, bb;
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1, %1};" : "=l"(bb) : "f"(b));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(bb));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r0), "=f"(r1) : "l"(r));
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
        const int half = (warp - 2) >> 2;  // columns 64 * half .. + 63 of the tile
        uint8_t* stage_buf = sout + (warp - 2) * kQOutChunk;
        uint32_t g = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
            const int mt = tile / n_tiles, nt = tile % n_tiles;
            const int row0 = mt * QM + quarter * 32;
            const int row = row0 + lane;
            const int col_base = nt * QN + half * 64;
            float acc[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) acc[i] = 0.0f;
            for (int b = 0; b < nblocks; ++b, ++g) {
                const int slot = static_cast<int>(g % kSlots);
                // The row's activation scale and the 64 columns' weight scales
                // of this block, issued before the wait for the slot.
                const float dx = row < m ? __ldg(args.dx + static_cast<int64_t>(b) * m + row) : 0.0f;
                const float* dwp = args.dw + static_cast<int64_t>(b) * n + col_base;
                // Warp-uniform wait: tcgen05.ld is warp-collective.
                if (!__all_sync(0xffffffffu, mbar_wait(&slot_full[slot], (g / kSlots) & 1u, status, 66))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t t0[32], t1[32];
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                       static_cast<uint32_t>(slot * QN + half * 64);
                tc_ld_32x32b_x32(taddr, t0);
                tc_ld_32x32b_x32(taddr + 32, t1);
                tc_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&slot_empty[slot]);
#pragma unroll
                for (int c4 = 0; c4 < 16; ++c4) {
                    const int c = c4 * 4;
                    float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (col_base + c + 3 < n) {
                        w = __ldg(reinterpret_cast<const float4*>(dwp + c));
                    } else {
                        if (col_base + c < n) w.x = __ldg(dwp + c);
                        if (col_base + c + 1 < n) w.y = __ldg(dwp + c + 1);
                        if (col_base + c + 2 < n) w.z = __ldg(dwp + c + 2);
                    }
                    float s0, s1, s2, s3;
                    mul2(s0, s1, w.x, w.y, dx);
                    mul2(s2, s3, w.z, w.w, dx);
                    const uint32_t* src = c < 32 ? t0 + c : t1 + (c - 32);
                    float v0, v1, v2, v3;
                    if (VARIANT == SAMQ_MMQ_CODES_I8) {
                        v0 = static_cast<float>(static_cast<int32_t>(src[0]));
                        v1 = static_cast<float>(static_cast<int32_t>(src[1]));
                        v2 = static_cast<float>(static_cast<int32_t>(src[2]));
                        v3 = static_cast<float>(static_cast<int32_t>(src[3]));
                    } else {
                        v0 = __uint_as_float(src[0]);
                        v1 = __uint_as_float(src[1]);
                        v2 = __uint_as_float(src[2]);
                        v3 = __uint_as_float(src[3]);
                    }
                    fma2(acc[c], acc[c + 1], v0, v1, s0, s1);
                    fma2(acc[c + 2], acc[c + 3], v2, v3, s2, s3);
                }
            }
            if (!ok) break;
            // Tile done: bias (+ erf-GELU), 32 x 32 chunks through shared memory, TMA store.
#pragma unroll
            for (int chunk = 0; chunk < 2; ++chunk) {
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
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
    }
    tc_fence_before();
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
