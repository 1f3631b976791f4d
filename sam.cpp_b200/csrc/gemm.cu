// gemm.cu -- K2: Y = epilogue(A . B^T + bias) on the sm_100a tensor cores.
//
// A is the f16 activation operand staged by K1 ([m][k], row-major), B the f16
// weight operand expanded from the K4 packets ([n][k], row-major).  This is
// GGML mul_mat(W, X) with W = B and X = A (src/models/sam3/ops.hpp:40-45),
// with the bias add and ggml_gelu_erf of the ViT MLP fused
// (src/models/sam3/vision.hpp:234-236).  The epilogue writes one of (OutMode):
//   f32 Y [m][ldy] (TMA store), optionally plus a residual (the ViT block's
//     shortcut adds, vision.hpp:228,240);
//   the Q8_1-staged f16 operand of the next linear (fc1 -> fc2), bit-identical
//     to K1 run on the f32 values the f32 mode stores;
//   the qkv split into RoPE'd Q (x 1/8), K and V^T in the attention kernel's
//     layout (vision.hpp:180-214).
//
// Persistent, warp-specialised kernel, one CTA per SM (64 + 32*EW threads):
//   warp 0     TMA producer: 128x64 A and BNx64 B tiles, 128-byte swizzle,
//              into a STAGES-deep shared-memory ring (full/empty mbarriers);
//   warp 1     TMEM owner and MMA issuer: one thread issues
//              tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16) into a
//              double-buffered f32 accumulator (2 x BN TMEM columns), then
//              tcgen05.commit to release the smem stage / publish the tile;
//   warps 2..  EW epilogue warps, EW/4 per TMEM lane quarter (the quarter a
//              warp may access is warp % 4), each owning 1/(EW/4) of the
//              tile's columns: tcgen05.ld 32 columns at a time, bias (one
//              coalesced load per 32 columns, broadcast by warp shuffles) and
//              erf-GELU in registers, swizzled staging in shared memory, TMA
//              store (clipped at the m / n edges).  The next tile's MMAs
//              overlap this epilogue.
// Measured on B200 (ViT shapes, M=5184, %globaltimer stamps per tile): the
// epilogue of a tile (2.5-3.5 us) hides behind the next tile's mainloop
// (6-8 us); the mainloop waits for its operand stages ~40% of the time, as
// the L2-to-shared-memory stream delivers ~100 GB/s per SM against the
// ~170 GB/s per SM full-rate MMAs would consume, the same rate whether the
// operands come from HBM or are L2-resident (a latency bound: ~180 KB in
// flight per SM).  EW=8 is used without GELU, EW=16 with erf-GELU.
// gemm_f16_pair_kernel below (cta_group::2, 256 x BN tiles) moves a third
// fewer operand bytes per FLOP and is used where a pair runs 3 or more tiles.
// No TMA load uses cluster multicast.  Every mbarrier wait is bounded and
// reports kStatusTimeout instead of hanging.
#include <algorithm>
#include <climits>

#include "samq_internal.hpp"

namespace samq {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;   // 64 f16 = 128 bytes = one swizzle row
// The two accumulator buffers start 256 TMEM columns apart whatever BN is.
constexpr int kAccStride = 256;

// Epilogue warps per CTA (EW, 8 or 16): EW/4 warps per TMEM lane quarter,
// each owning 1/(EW/4) of the tile's columns.
constexpr int threads_for(int ew) { return 64 + 32 * ew; }
constexpr int kOutChunkBytes = 32 * 32 * 4;  // 32 rows x 32 f32 columns
constexpr int kOutBuffers = 1;               // staging buffers per epilogue warp (4 stages fit beside them)

// Operand stages that fit in 227 KB beside EW staging buffers.
constexpr int stages_for(int bn, int ew) {
    return (232448 - 1024 - 256 - ew * 1 * 4096) / (128 * 64 * 2 + bn * 64 * 2) > 6
               ? 6
               : (232448 - 1024 - 256 - ew * 1 * 4096) / (128 * 64 * 2 + bn * 64 * 2);
}

template <int BN, int STAGES, int EW>
struct Layout {
    static constexpr int a_bytes = BM * BK * 2;
    static constexpr int b_bytes = BN * BK * 2;
    static constexpr int stage_tx = a_bytes + b_bytes;
    static constexpr int a_off = 0;
    static constexpr int b_off = STAGES * a_bytes;
    static constexpr int out_off = b_off + STAGES * b_bytes;
    static constexpr int bar_off = out_off + EW * kOutBuffers * kOutChunkBytes;
    static constexpr int bar_bytes = (2 * STAGES + 5) * 8 + 8;
    static constexpr int total = bar_off + bar_bytes + 1024;  // + alignment slack
    static constexpr uint32_t tmem_cols = 2 * kAccStride;       // double-buffered accumulator
};

// One epilogue warp's share of an accumulator tile: TMEM lanes 32*quarter..+31
// (output rows row0..row0+31, one row per lane) and 32-column chunks
// [part*C/PARTS, (part+1)*C/PARTS) of the C = BN/32 chunks of the tile starting
// at output column col_base.  32 columns at a time: tcgen05.ld, bias (one
// coalesced load, broadcast by shuffles), erf-GELU, then per OutMode either
// swizzled staging in shared memory and a TMA store (clipped by the tensor map
// at the m / n edges), or direct stores of f16 rows.
// What a chunk needs from global memory besides the accumulator: the bias of
// column col0 + lane and, for the residual mode, the row's 32 residual values.
// They are issued together with the chunk's TMEM load; in the residual mode a
// warp's first chunk loads them before the accumulator is even ready (under
// the tile's MMAs), as the 128-byte residual read is the longest wait there.
template <int MODE>
struct ChunkInputs {
    float bias = 0.0f;
    float4 res[MODE == kOutF32Residual ? 8 : 1];
};

template <int MODE>
__device__ __forceinline__ void load_chunk_inputs(const Epilogue& ep, int col0, int row, int m, int n, int lane,
                                                  ChunkInputs<MODE>& in) {
    in.bias = (ep.bias != nullptr && col0 + lane < n) ? __ldg(ep.bias + col0 + lane) : 0.0f;
    if constexpr (MODE == kOutF32Residual) {
        if (row < m) {
            const float4* res = reinterpret_cast<const float4*>(ep.residual + static_cast<int64_t>(row) * ep.ldr + col0);
#pragma unroll
            for (int j = 0; j < 8; ++j) in.res[j] = col0 + 4 * j < n ? res[j] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
}

template <int BN, int PARTS, int MODE, bool GELU>
__device__ __forceinline__ void drain_tile(uint32_t tmem_base, int quarter, int part, int acc, int row0,
                                           int col_base, int m, int n, const Epilogue& ep,
                                           const CUtensorMap* tma_y, const CUtensorMap* tma_k,
                                           const CUtensorMap* tma_v, uint8_t* stage_buf, int& buf, int lane,
                                           const ChunkInputs<MODE>& first, DeviceStatus* status) {
    constexpr int kChunks = BN / 32;
    const int row = row0 + lane;
    const int c_begin = part * kChunks / PARTS, c_end = (part + 1) * kChunks / PARTS;
#pragma unroll 1
    for (int chunk = c_begin; chunk < c_end; ++chunk) {
        const int col0 = col_base + chunk * 32;
        if (col0 >= n) break;
        uint32_t r[32];
        tc_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * kAccStride + chunk * 32),
                         r);
        ChunkInputs<MODE> cur;
        if (MODE == kOutF32Residual && chunk == c_begin) cur = first;
        else load_chunk_inputs<MODE>(ep, col0, row, m, n, lane, cur);
        const float bias_lane = cur.bias;
        // qkv split: the RoPE table entries of this row's 16 channel pairs,
        // fetched while the accumulator load is in flight (8-warp epilogues
        // only: the 16-warp ones have no registers to spare for them).
        constexpr bool kPrefetchRope = PARTS <= 2;
        float4 fr[8];
        int sec = 0, c0 = 0, nn = 0;
        int64_t gh = 0;
        if constexpr (MODE == kOutQkvPack) {
            const int embed = ep.heads * 64;
            const int rr = row < m ? row : 0;
            const int g = rr / ep.group_n;
            nn = rr - g * ep.group_n;
            sec = col0 / embed;
            const int rem = col0 - sec * embed;
            gh = static_cast<int64_t>(g) * ep.heads + (rem >> 6);
            c0 = rem & 63;
            if (kPrefetchRope && sec < 2) {
                const float4* src = reinterpret_cast<const float4*>(ep.freqs + (static_cast<int64_t>(nn) * 32 + c0 / 2) * 2);
#pragma unroll
                for (int p = 0; p < 8; ++p) fr[p] = __ldg(src + p);
            }
        }
        tc_wait_ld();
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            float x = __uint_as_float(r[i]) + __shfl_sync(0xffffffffu, bias_lane, i);
            if constexpr (GELU) x = gelu_erf(x);
            v[i] = x;
        }
        if constexpr (MODE == kOutF16Staged) {
            uint32_t out[16];
            const bool bad = stage_q8_1<1, 32>(v, out);
            record_range(bad && row < m, status);
            // 32 rows x 64 bytes through shared memory in the 64-byte swizzle
            // (16-byte unit u of row r at u ^ ((r >> 1) & 3)), one TMA store.
            if (lane == 0) bulk_wait_group_read<kOutBuffers - 1>();
            __syncwarp();
            uint8_t* sbuf = stage_buf + buf * kOutChunkBytes;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                *reinterpret_cast<uint4*>(sbuf + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
                    make_uint4(out[4 * j], out[4 * j + 1], out[4 * j + 2], out[4 * j + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && row0 < m) {
                tma_store_2d(tma_y, sbuf, col0, row0);
                bulk_commit_group();
            }
            buf = (buf + 1) % kOutBuffers;
            continue;
        }
        if constexpr (MODE == kOutQkvPack) {
            // Whole 32-row blocks of one group (group_n % 32 == 0, the ViT's
            // 576 and 5184): Q / K rows and the V^T tile leave through shared
            // memory (64-byte swizzle) and one TMA store each.  Otherwise
            // direct stores.
            const bool tiled = (ep.group_n & 31) == 0;
            uint32_t out[16];
            if (sec < 2) {
                // RoPE on channel pairs (2i, 2i+1), i = c0/2 .. c0/2 + 15
                // (vision.hpp:100-148); the 1/8 softmax scale folds into Q
                // exactly (a power of two).
                const float scale = sec == 0 ? 0.125f : 1.0f;
                if (!kPrefetchRope && row < m) {
                    const float4* src = reinterpret_cast<const float4*>(ep.freqs + (static_cast<int64_t>(nn) * 32 + c0 / 2) * 2);
#pragma unroll
                    for (int p = 0; p < 8; ++p) fr[p] = __ldg(src + p);
                }
#pragma unroll
                for (int p = 0; p < 8; ++p) {
                    const float4 f = fr[p];  // (cos, sin) of pairs 2p and 2p+1
                    const float x0 = v[4 * p], x1 = v[4 * p + 1], x2 = v[4 * p + 2], x3 = v[4 * p + 3];
                    const float re0 = __fsub_rn(__fmul_rn(x0, f.x), __fmul_rn(x1, f.y));
                    const float im0 = __fadd_rn(__fmul_rn(x0, f.y), __fmul_rn(x1, f.x));
                    const float re1 = __fsub_rn(__fmul_rn(x2, f.z), __fmul_rn(x3, f.w));
                    const float im1 = __fadd_rn(__fmul_rn(x2, f.w), __fmul_rn(x3, f.z));
                    const __half2 h0 = __floats2half2_rn(re0 * scale, im0 * scale);
                    const __half2 h1 = __floats2half2_rn(re1 * scale, im1 * scale);
                    out[2 * p] = *reinterpret_cast<const uint32_t*>(&h0);
                    out[2 * p + 1] = *reinterpret_cast<const uint32_t*>(&h1);
                }
            }
            if (tiled) {
                if (lane == 0) bulk_wait_group_read<kOutBuffers - 1>();
                __syncwarp();
                uint8_t* sbuf = stage_buf + buf * kOutChunkBytes;
                if (sec < 2) {
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        *reinterpret_cast<uint4*>(sbuf + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
                            make_uint4(out[4 * j], out[4 * j + 1], out[4 * j + 2], out[4 * j + 3]);
                } else {
                    // V^T tile: channel rows i, token columns lane.
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        *reinterpret_cast<__half*>(sbuf + i * 64 + (((lane >> 3) ^ ((i >> 1) & 3)) << 4) + (lane & 7) * 2) =
                            __float2half_rn(v[i]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0 && row0 < m) {
                    const int nn0 = nn - lane;  // lane 0: nn of row0
                    if (sec < 2)
                        tma_store_2d(sec == 0 ? tma_y : tma_k, sbuf, c0, static_cast<int32_t>(gh * ep.group_n + nn0));
                    else
                        tma_store_2d(tma_v, sbuf, nn0, static_cast<int32_t>(gh * 64 + c0));
                    bulk_commit_group();
                }
                buf = (buf + 1) % kOutBuffers;
            } else if (row < m) {
                if (sec < 2) {
                    __half* base = sec == 0 ? ep.q : ep.k;
                    uint4* dst = reinterpret_cast<uint4*>(base + (gh * ep.group_n + nn) * 64 + c0);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        dst[j] = make_uint4(out[4 * j], out[4 * j + 1], out[4 * j + 2], out[4 * j + 3]);
                } else {
                    __half* base = ep.vt + (gh * 64 + c0) * ep.group_n + nn;
#pragma unroll
                    for (int i = 0; i < 32; ++i) base[static_cast<int64_t>(i) * ep.group_n] = __float2half_rn(v[i]);
                }
            }
            continue;
        }
        if constexpr (MODE == kOutF32Residual) {
            // The ViT shortcut add: residual + (acc + bias), one f32 add.
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 rv = cur.res[j];
                v[4 * j] = __fadd_rn(rv.x, v[4 * j]);
                v[4 * j + 1] = __fadd_rn(rv.y, v[4 * j + 1]);
                v[4 * j + 2] = __fadd_rn(rv.z, v[4 * j + 2]);
                v[4 * j + 3] = __fadd_rn(rv.w, v[4 * j + 3]);
            }
        }
        if (lane == 0) bulk_wait_group_read<kOutBuffers - 1>();
        __syncwarp();
        uint8_t* sbuf = stage_buf + buf * kOutChunkBytes;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 val = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            *reinterpret_cast<float4*>(sbuf + lane * 128 + ((j ^ (lane & 7)) << 4)) = val;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && row0 < m) {
            tma_store_2d(tma_y, sbuf, col0, row0);
            bulk_commit_group();
        }
        buf = (buf + 1) % kOutBuffers;
    }
}

template <int BN, int STAGES, int EW, int MODE, bool GELU>
__global__ void __launch_bounds__(threads_for(EW), 1)
gemm_f16_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                const __grid_constant__ CUtensorMap tma_y, const __grid_constant__ CUtensorMap tma_k,
                const __grid_constant__ CUtensorMap tma_v, const Epilogue ep, int m, int n, int k,
                DeviceStatus* status) {
    using L = Layout<BN, STAGES, EW>;
    static_assert(L::total <= 232448, "shared memory budget");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sa = smem + L::a_off;
    uint8_t* sb = smem + L::b_off;
    uint8_t* sout = smem + L::out_off;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bar_off);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tiles = (m + BM - 1) / BM, n_tiles = (n + BN - 1) / BN;
    const int tiles = m_tiles * n_tiles;
    const int kblocks = (k + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], EW);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tma_a);
        tma_prefetch_desc(&tma_b);
        tma_prefetch_desc(&tma_y);
        tma_prefetch_desc(&tma_k);
        tma_prefetch_desc(&tma_v);
    }
    if (warp == 1) tmem_alloc(tmem_slot, L::tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Everything above overlaps the previous kernel; A (and the output buffer)
    // may be in use by it until it completes.
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            uint32_t issued = 0, issued_phase = 0;  // per stage: ever issued / parity of last issue
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                const int mt = tile / n_tiles, nt = tile % n_tiles;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1u, status, 1)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], L::stage_tx);
                    tma_load_2d(sa + s * L::a_bytes, &tma_a, &full[s], kb * BK, mt * BM);
                    tma_load_2d(sb + s * L::b_bytes, &tma_b, &full[s], kb * BK, nt * BN);
                    issued |= 1u << s;
                    issued_phase = (issued_phase & ~(1u << s)) | (ph << s);
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            pdl_trigger();  // all loads issued: the next kernel may begin its prologue
            if (!ok) {
                // Let every copy already in flight land before the CTA exits.
                for (int i = 0; i < STAGES; ++i)
                    if (issued & (1u << i)) mbar_wait(&full[i], (issued_phase >> i) & 1u, status, 5);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(BM, BN);
            int s = 0;
            uint32_t ph = 0;
            int acc = 0;
            uint32_t acc_ph = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                if (!mbar_wait(&tempty[acc], acc_ph ^ 1u, status, 2)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + static_cast<uint32_t>(acc * kAccStride);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&full[s], ph, status, 3)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sa + s * L::a_bytes);
                    const uint32_t b_addr = smem_u32(sb + s * L::b_bytes);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        tc_mma_f16(d, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32), idesc,
                                   (kb | kk) != 0 ? 1u : 0u);
                    tc_commit(&empty[s]);
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(&tfull[acc]);
                acc ^= 1;
                if (acc == 0) acc_ph ^= 1u;
            }
            // Wait for every MMA this thread issued before TMEM is released.
            tc_commit(drain);
            mbar_wait(drain, 0, status, 6);
        }
    } else {
        const int quarter = warp & 3;          // TMEM lanes 32*quarter .. +31
        const int part = (warp - 2) >> 2;      // column part of the tile (EW/4 parts)
        uint8_t* stage_buf = sout + (warp - 2) * kOutBuffers * kOutChunkBytes;
        int acc = 0;
        uint32_t acc_ph = 0;
        int buf = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            const int mt = tile / n_tiles, nt = tile % n_tiles;
            const int row0 = mt * BM + quarter * 32;
            // Residual mode: the first chunk's inputs load while the tile's MMAs run.
            ChunkInputs<MODE> first;
            if constexpr (MODE == kOutF32Residual) {
                const int first_col = nt * BN + (part * (BN / 32) / (EW / 4)) * 32;
                if (first_col < n) load_chunk_inputs<MODE>(ep, first_col, row0 + lane, m, n, lane, first);
            }
            // Warp-uniform: the tcgen05.ld in drain_tile is warp-collective.
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_ph, status, 4))) break;
            tc_fence_after();
            drain_tile<BN, EW / 4, MODE, GELU>(tmem_base, quarter, part, acc, row0, nt * BN, m, n, ep, &tma_y, &tma_k,
                                               &tma_v, stage_buf, buf, lane, first, status);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
            acc ^= 1;
            if (acc == 0) acc_ph ^= 1u;
        }
        // The CTA may exit once its TMA stores have read their shared-memory
        // sources; completion of the grid makes the global writes visible.
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
    }
    tc_fence_before();
    // Reconverge each warp before the CTA barrier: __syncthreads is an aligned
    // barrier (every thread of a warp executes it together), and lane 0 alone
    // ran the producer and MMA loops.
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, L::tmem_cols);
    }
}

// ---------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs on the two SMs of a TPC computes a
// 256 x BN tile with tcgen05.mma.cta_group::2 (M=256, N=BN, K=16).  CTA r of
// the pair loads A rows [128r, 128r+128) and B rows [r*BN/2, (r+1)*BN/2) of
// the tile into its own shared memory; the pair MMA reads both CTAs' halves,
// and each CTA's TMEM holds its 128 rows x BN columns of the accumulator.
// Per SM and 64-deep K step this moves (128 + BN/2) x 128 bytes of operands
// instead of (128 + BN) x 128 for the same tensor work, and a stage covers
// 1.5-1.8x more MMA time against the load latency.  Measured on B200, the
// single-CTA mainloop waits for its operands ~40% of each tile (it streams
// ~100 GB/s per SM from L2, the same rate as a loads-only copy of it).
//   warp 0 of each CTA: TMA producer of its halves; both signal the even
//       CTA's `full` barrier (the even CTA's expect_tx covers both halves);
//   warp 1: TMEM (both CTAs allocate together); in the even CTA one thread
//       issues the pair MMAs, whose commits release `empty` stages and
//       publish `tfull` in both CTAs;
//   warps 2.. of both CTAs: the epilogue of their own 128 rows (drain_tile,
//       every output mode); they return the accumulator through the even
//       CTA's `tempty` barrier.
// No TMA load uses multicast; remote signals go through mapa addresses.
constexpr int kPairTmemCols = 2 * kAccStride;

// Operand stages per CTA that fit in 227 KB beside EW staging buffers.
constexpr int pair_stages_for(int bn, int ew) {
    return (232448 - 1024 - 256 - ew * 4096) / (BM * BK * 2 + (bn / 2) * BK * 2) > 8
               ? 8
               : (232448 - 1024 - 256 - ew * 4096) / (BM * BK * 2 + (bn / 2) * BK * 2);
}

template <int BN, int STAGES, int EW>
struct PairLayout {
    static constexpr int a_bytes = BM * BK * 2;
    static constexpr int b_bytes = (BN / 2) * BK * 2;
    static constexpr int stage_tx = 2 * (a_bytes + b_bytes);  // both CTAs' halves
    static constexpr int a_off = 0;
    static constexpr int b_off = STAGES * a_bytes;
    static constexpr int out_off = b_off + STAGES * b_bytes;
    static constexpr int bar_off = out_off + EW * kOutBuffers * kOutChunkBytes;
    static constexpr int bar_bytes = (2 * STAGES + 5) * 8 + 8;
    static constexpr int total = bar_off + bar_bytes + 1024;  // + alignment slack
};

template <int BN, int STAGES, int EW, int MODE, bool GELU>
__global__ void __launch_bounds__(threads_for(EW), 1)
gemm_f16_pair_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ CUtensorMap tma_y, const __grid_constant__ CUtensorMap tma_k,
                     const __grid_constant__ CUtensorMap tma_v, const Epilogue ep, int m, int n, int k,
                     DeviceStatus* status) {
    using L = PairLayout<BN, STAGES, EW>;
    static_assert(L::total <= 232448, "shared memory budget");
    static_assert(BN % 32 == 0 && BN <= 256, "pair tile width");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sa = smem + L::a_off;
    uint8_t* sb = smem + L::b_off;
    uint8_t* sout = smem + L::out_off;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bar_off);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_cta_rank();
    const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
    const int m_tiles = (m + 2 * BM - 1) / (2 * BM), n_tiles = (n + BN - 1) / BN;
    const int tiles = m_tiles * n_tiles;
    const int kblocks = (k + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * EW);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tma_a);
        tma_prefetch_desc(&tma_b);
        tma_prefetch_desc(&tma_y);
        tma_prefetch_desc(&tma_k);
        tma_prefetch_desc(&tma_v);
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, kPairTmemCols);
    tc_fence_before();
    cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Everything above overlaps the previous kernel; A (and the output buffer)
    // may be in use by it until it completes.
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            bool ok = true, any = false;
            for (int tile = pair; tile < tiles && ok; tile += pairs) {
                const int mt = tile / n_tiles, nt = tile % n_tiles;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1u, status, 11)) {
                        ok = false;
                        break;
                    }
                    const uint32_t full_even = cluster_map(&full[s], 0);
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], L::stage_tx);
                    tma_load_2d_pair(sa + s * L::a_bytes, &tma_a, full_even, kb * BK,
                                     mt * 2 * BM + static_cast<int>(rank) * BM);
                    tma_load_2d_pair(sb + s * L::b_bytes, &tma_b, full_even, kb * BK,
                                     nt * BN + static_cast<int>(rank) * (BN / 2));
                    any = true;
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            pdl_trigger();  // all loads issued: the next kernel may begin its prologue
            if (!ok && any) {
                // Copies in flight signal the even CTA's barrier; give them time to land.
                const uint64_t start = global_timer_ns();
                while (global_timer_ns() - start < 2000000ull) __nanosleep(1000);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(2 * BM, BN);
            int s = 0;
            uint32_t ph = 0;
            int acc = 0;
            uint32_t acc_ph = 0;
            bool ok = true;
            for (int tile = pair; tile < tiles && ok; tile += pairs) {
                if (!mbar_wait_cluster(&tempty[acc], acc_ph ^ 1u, status, 12)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + static_cast<uint32_t>(acc * kAccStride);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&full[s], ph, status, 13)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sa + s * L::a_bytes);
                    const uint32_t b_addr = smem_u32(sb + s * L::b_bytes);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        tc_mma_f16_pair(d, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(b_addr + kk * 32),
                                        idesc, (kb | kk) != 0 ? 1u : 0u);
                    tc_commit_pair(cluster_map(&empty[s], 0));
                    tc_commit_pair(cluster_map(&empty[s], 1));
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit_pair(cluster_map(&tfull[acc], 0));
                tc_commit_pair(cluster_map(&tfull[acc], 1));
                acc ^= 1;
                if (acc == 0) acc_ph ^= 1u;
            }
            // Wait for every MMA this thread issued before TMEM is released.
            tc_commit_pair(cluster_map(drain, 0));
            mbar_wait(drain, 0, status, 16);
        }
    } else {
        const int quarter = warp & 3;          // TMEM lanes 32*quarter .. +31
        const int part = (warp - 2) >> 2;      // column part of the tile (EW/4 parts)
        uint8_t* stage_buf = sout + (warp - 2) * kOutBuffers * kOutChunkBytes;
        const uint32_t tempty_even[2] = {cluster_map(&tempty[0], 0), cluster_map(&tempty[1], 0)};
        int acc = 0;
        uint32_t acc_ph = 0;
        int buf = 0;
        for (int tile = pair; tile < tiles; tile += pairs) {
            const int mt = tile / n_tiles, nt = tile % n_tiles;
            const int row0 = mt * 2 * BM + static_cast<int>(rank) * BM + quarter * 32;
            ChunkInputs<MODE> first;
            if constexpr (MODE == kOutF32Residual) {
                const int first_col = nt * BN + (part * (BN / 32) / (EW / 4)) * 32;
                if (first_col < n) load_chunk_inputs<MODE>(ep, first_col, row0 + lane, m, n, lane, first);
            }
            // Warp-uniform: the tcgen05.ld in drain_tile is warp-collective.
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_ph, status, 14))) break;
            tc_fence_after();
            drain_tile<BN, EW / 4, MODE, GELU>(tmem_base, quarter, part, acc, row0, nt * BN, m, n, ep, &tma_y, &tma_k,
                                               &tma_v, stage_buf, buf, lane, first, status);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_even[acc]);
            acc ^= 1;
            if (acc == 0) acc_ph ^= 1u;
        }
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
    }
    tc_fence_before();
    __syncwarp();        // converged for the aligned cluster barrier
    cluster_sync_all();  // both CTAs done with TMEM and with each other's barriers
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kPairTmemCols);
    }
}

// The output tensor maps of an epilogue (maps a mode does not use cover A:
// valid, never stored to).
void encode_output_maps(const __half* a, int64_t lda, int64_t m, int64_t n, int64_t k, const Epilogue& ep,
                        CUtensorMap& ty, CUtensorMap& tk, CUtensorMap& tv) {
    if (ep.mode == kOutF32 || ep.mode == kOutF32Residual)
        encode_tensor_map_2d(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, ep.y, n, m, ep.ldy * 4, 32, 32,
                             CU_TENSOR_MAP_SWIZZLE_128B);
    else if (ep.mode == kOutF16Staged)
        encode_tensor_map_2d(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ep.h, n, m, ep.ldh * 2, 32, 32,
                             CU_TENSOR_MAP_SWIZZLE_64B);
    encode_tensor_map_2d(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a, k, m, lda * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    tv = tk;
    if (ep.mode == kOutQkvPack) {
        // Q and K [group * heads + head][group_n][64], V^T [group * heads + head][64][group_n].
        const uint64_t rows = static_cast<uint64_t>(m / ep.group_n) * ep.heads * ep.group_n;
        encode_tensor_map_2d(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ep.q, 64, rows, 128, 32, 32,
                             CU_TENSOR_MAP_SWIZZLE_64B);
        encode_tensor_map_2d(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ep.k, 64, rows, 128, 32, 32,
                             CU_TENSOR_MAP_SWIZZLE_64B);
        encode_tensor_map_2d(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ep.vt, ep.group_n,
                             static_cast<uint64_t>(m / ep.group_n) * ep.heads * 64,
                             static_cast<uint64_t>(ep.group_n) * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    } else if (ep.mode != kOutF32 && ep.mode != kOutF32Residual && ep.mode != kOutF16Staged) {
        ty = tk;
    }
}

template <int BN, int STAGES, int EW, int MODE, bool GELU>
void run(const __half* a, int64_t lda, const __half* b, int64_t m, int64_t n, int64_t k, const Epilogue& ep,
         DeviceState& state, cudaStream_t stream) {
    using L = Layout<BN, STAGES, EW>;
    CUtensorMap ta, tb, ty, tk, tv;
    encode_tensor_map_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a, k, m, lda * 2, BK, BM,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    encode_tensor_map_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, b, k, n, k * 2, BK, BN,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    encode_output_maps(a, lda, m, n, k, ep, ty, tk, tv);
    auto kernel = gemm_f16_kernel<BN, STAGES, EW, MODE, GELU>;
    set_smem_limit_once(state, reinterpret_cast<const void*>(kernel), L::total, "cudaFuncSetAttribute(gemm smem)");
    const int64_t tiles = ((m + BM - 1) / BM) * ((n + BN - 1) / BN);
    const int grid = static_cast<int>(tiles < state.sm_count ? tiles : state.sm_count);
    launch_pdl(kernel, dim3(grid), dim3(threads_for(EW)), L::total, stream, "gemm_f16_kernel launch", ta, tb, ty, tk, tv,
               ep, static_cast<int>(m), static_cast<int>(n), static_cast<int>(k), state.status);
}

template <int BN, int EW, int MODE, bool GELU>
void run_pair(const __half* a, int64_t lda, const __half* b, int64_t m, int64_t n, int64_t k, const Epilogue& ep,
              DeviceState& state, cudaStream_t stream) {
    constexpr int kStages = pair_stages_for(BN, EW);
    using L = PairLayout<BN, kStages, EW>;
    CUtensorMap ta, tb, ty, tk, tv;
    encode_tensor_map_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a, k, m, lda * 2, BK, BM,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    encode_tensor_map_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, b, k, n, k * 2, BK, BN / 2,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    encode_output_maps(a, lda, m, n, k, ep, ty, tk, tv);
    auto kernel = gemm_f16_pair_kernel<BN, kStages, EW, MODE, GELU>;
    set_smem_limit_once(state, reinterpret_cast<const void*>(kernel), L::total,
                        "cudaFuncSetAttribute(pair gemm smem)");
    const int resident = pair_clusters_resident(state, reinterpret_cast<const void*>(kernel), threads_for(EW),
                                                L::total, "cudaOccupancyMaxActiveClusters(pair gemm)");
    const int64_t tiles = ((m + 2 * BM - 1) / (2 * BM)) * ((n + BN - 1) / BN);
    const int64_t pairs = std::min<int64_t>(tiles, resident);
    launch_pdl_pairs(kernel, dim3(static_cast<unsigned>(2 * pairs)), dim3(threads_for(EW)), L::total, stream,
                     "gemm_f16_pair_kernel launch", ta, tb, ty, tk, tv, ep, static_cast<int>(m),
                     static_cast<int>(n), static_cast<int>(k), state.status);
}

}  // namespace

// Tile shape: single CTA (128 x BN) or CTA pair (256 x BN), BN a multiple of
// 32.  Each candidate is scored by its per-SM critical path, (waves of tiles
// over the SMs or pairs) x the time of one 64-deep K step of a tile, the
// larger of the tensor time (BN columns) and the operand stream time
// ((128 + B rows per SM) x 128 bytes at the ~100 GB/s per SM measured for the
// L2-to-shared-memory stream); the weights 915 : 1000 are those two rates
// per row (14 TFLOP/s per SM against 100 GB/s per SM, B200, 1.8 GHz).  Ties go
// to the pair, then to the wider tile (less operand traffic per FLOP).
// The operand stream is latency-bound rather than byte-bound (the pair moves
// a third fewer bytes per FLOP but its tiles measured only 10-25% faster), and
// a pair's start-up and last epilogue cost more, so the pair is taken only
// where it runs at least kPairMinWaves tiles per pair: measured on B200 at
// M = 5184 it wins for N = 3072 / 4736 (4 and 6 waves) and loses for N = 1024
// (2 waves).
constexpr int64_t kPairMinWaves = 3;

struct GemmShape {
    bool pair;
    int bn;
};

GemmShape choose_shape(int64_t m, int64_t n, int sms) {
    static const int kWidths[4] = {256, 224, 192, 160};
    GemmShape best{false, 256};
    int64_t best_cost = INT64_MAX;
    for (int pair = 1; pair >= 0; --pair) {
        if (pair && (m <= BM || sms < 2)) continue;
        const int64_t rows = pair ? 2 * BM : BM, units = pair ? sms / 2 : sms;
        for (int bn : kWidths) {
            const int64_t tiles = ((m + rows - 1) / rows) * ((n + bn - 1) / bn);
            const int64_t waves = (tiles + units - 1) / units;
            if (pair && waves < kPairMinWaves) continue;
            const int64_t b_rows = pair ? bn / 2 : bn;
            const int64_t step = std::max<int64_t>(int64_t(bn) * 915, (BM + b_rows) * 1000);
            const int64_t cost = waves * step;
            if (cost < best_cost) {
                best_cost = cost;
                best = GemmShape{pair != 0, bn};
            }
        }
    }
    return best;
}

template <int EW, int MODE, bool GELU>
void run_width(GemmShape shape, const __half* a, int64_t lda, const __half* b, int64_t m, int64_t n, int64_t k,
               const Epilogue& ep, DeviceState& state, cudaStream_t stream) {
    if (n <= 128) {
        run<128, 6, 8, MODE, GELU>(a, lda, b, m, n, k, ep, state, stream);
        return;
    }
    if (shape.pair) {
        switch (shape.bn) {
            case 160: run_pair<160, EW, MODE, GELU>(a, lda, b, m, n, k, ep, state, stream); break;
            case 192: run_pair<192, EW, MODE, GELU>(a, lda, b, m, n, k, ep, state, stream); break;
            case 224: run_pair<224, EW, MODE, GELU>(a, lda, b, m, n, k, ep, state, stream); break;
            default: run_pair<256, EW, MODE, GELU>(a, lda, b, m, n, k, ep, state, stream); break;
        }
        return;
    }
    switch (shape.bn) {
        case 160: run<160, stages_for(160, EW), EW, MODE, GELU>(a, lda, b, m, n, k, ep, state, stream); break;
        case 192: run<192, stages_for(192, EW), EW, MODE, GELU>(a, lda, b, m, n, k, ep, state, stream); break;
        case 224: run<224, stages_for(224, EW), EW, MODE, GELU>(a, lda, b, m, n, k, ep, state, stream); break;
        default: run<256, stages_for(256, EW), EW, MODE, GELU>(a, lda, b, m, n, k, ep, state, stream); break;
    }
}

// One kernel instantiation per output mode (and erf-GELU), so each carries
// only its own epilogue's registers.  erf-GELU makes the epilogue the longer
// pipeline: 16 epilogue warps there, 8 otherwise.
void launch_gemm(const __half* a, int64_t lda, const __half* b, int64_t m, int64_t n, int64_t k, const Epilogue& ep,
                 DeviceState& state, cudaStream_t stream) {
    if (m == 0) return;
    const GemmShape shape = choose_shape(m, n, state.sm_count);
    switch (ep.mode) {
        case kOutF32:
            if (ep.gelu) run_width<16, kOutF32, true>(shape, a, lda, b, m, n, k, ep, state, stream);
            else run_width<8, kOutF32, false>(shape, a, lda, b, m, n, k, ep, state, stream);
            break;
        case kOutF32Residual:
            if (ep.gelu) fail(SAMQ_ERR_INVALID_ARGUMENT, "residual epilogue takes no GELU");
            run_width<8, kOutF32Residual, false>(shape, a, lda, b, m, n, k, ep, state, stream);
            break;
        case kOutF16Staged:
            if (ep.gelu) run_width<16, kOutF16Staged, true>(shape, a, lda, b, m, n, k, ep, state, stream);
            else run_width<8, kOutF16Staged, false>(shape, a, lda, b, m, n, k, ep, state, stream);
            break;
        case kOutQkvPack:
            if (ep.gelu) fail(SAMQ_ERR_INVALID_ARGUMENT, "qkv split takes no GELU");
            run_width<8, kOutQkvPack, false>(shape, a, lda, b, m, n, k, ep, state, stream);
            break;
        default: fail(SAMQ_ERR_INVALID_ARGUMENT, "unknown GEMM output mode");
    }
}

void launch_gemm_f16(const __half* a, int64_t lda, const __half* b, int64_t m, int64_t n, int64_t k,
                     const float* bias, int epilogue, float* y, int64_t ldy, DeviceState& state,
                     cudaStream_t stream) {
    Epilogue ep;
    ep.mode = kOutF32;
    ep.gelu = epilogue == SAMQ_EPILOGUE_GELU_ERF ? 1 : 0;
    ep.bias = bias;
    ep.y = y;
    ep.ldy = ldy;
    launch_gemm(a, lda, b, m, n, k, ep, state, stream);
}

}  // namespace samq
