// stream.cu -- small-M quantized linears (text encoder M = 32, prompt KV M = 33,
// any M <= 64): the weights stream from their K4 packets and are decoded in the
// producer, so HBM carries the packed bytes (0.56-1.06 B per weight) instead
// of the 2-byte f16 expansion K2 reads.
//
// Y[m][n] = act(sum_k W[n][k] X[m][k] + bias[n]) with X the Q8_1-staged f16
// operand [m][k] (K1) and W the packed weights.  The product is computed
// transposed ("swap AB") on the tensor cores: D[128 weight rows][TOK tokens]
// = W_tile[128][64] . X[TOK][64]^T per 64-column chunk, tcgen05.mma M=128,
// N=TOK (32 or 64), accumulated in TMEM.
//
// One CTA per (128-row tile of W, range of 64-column chunks), 192 threads:
//   warp 0     loads: each chunk's packet (one contiguous span) by a 1-D bulk
//              copy and the chunk's X tile by TMA (rows past m zero-filled),
//              into a 4-stage ring;
//   warp 1     TMEM owner and MMA issuer;
//   warps 2-5  decode the packet into a 128-byte-swizzled f16 A tile (8 lanes
//              per row, each decoding 8 columns with the K4 decoder, so the
//              operand equals K2's f16 weights bit for bit), double buffered;
//              then the epilogue: the accumulator out of TMEM, bias and
//              erf-GELU when the CTA covers all of K, otherwise an f32 partial
//              per chunk range, summed in split order by splitk_reduce_kernel
//              (deterministic; its launch overlaps this kernel's tail through
//              programmatic dependent launch).  Summing in the last-arriving
//              warp instead (atomic tickets) left 32 warps with all the work
//              and measured 23 us against 10 + 6 us for this pair.
// All waits are bounded; no load uses multicast.
#include <algorithm>

#include "packets.cuh"
#include "samq_internal.hpp"

namespace samq {
namespace {

constexpr int kStreamStages = 4;
constexpr int kStreamThreads = 192;
constexpr int kMaxSplits = 16;  // split-K ways at most

template <int TYPE, int TOK>
struct StreamSmem {
    static constexpr int raw_bytes = 128 * (code_bytes_of(TYPE) + 8);  // one packet
    static constexpr int x_bytes = TOK * 128;                          // TOK rows x 64 f16
    static constexpr int a_bytes = 128 * 128;                          // 128 rows x 64 f16
    static constexpr int a_off = 0;
    static constexpr int x_off = a_off + 2 * a_bytes;
    static constexpr int raw_off = x_off + kStreamStages * x_bytes;
    static constexpr int bar_off = raw_off + kStreamStages * raw_bytes;
    // full[S], empty[S], a_full[2], a_empty[2], d_full, drain
    static constexpr int bar_count = 2 * kStreamStages + 4 + 2;
    static constexpr int total = bar_off + bar_count * 8 + 8 + 1024;
};

template <int TYPE, int TOK>
__global__ void __launch_bounds__(kStreamThreads, 2)
gemm_stream_kernel(const uint8_t* __restrict__ packets, const __grid_constant__ CUtensorMap tm_x, int64_t n, int m,
                   int chunks_total, int chunks_per_split, int splits, float* __restrict__ partials,
                   const float* __restrict__ bias, int gelu, float* __restrict__ y, int64_t ldy,
                   DeviceStatus* status) {
    using L = StreamSmem<TYPE, TOK>;
    constexpr int cb = code_bytes_of(TYPE);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sa = smem + L::a_off;
    uint8_t* sx = smem + L::x_off;
    uint8_t* sraw = smem + L::raw_off;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bar_off);
    uint64_t* empty = full + kStreamStages;
    uint64_t* a_full = empty + kStreamStages;
    uint64_t* a_empty = a_full + 2;
    uint64_t* d_full = a_empty + 2;
    uint64_t* drain = d_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x, split = blockIdx.y;
    const int c_begin = split * chunks_per_split;
    const int nchunks = min(chunks_total, c_begin + chunks_per_split) - c_begin;  // >= 1 (host)
    constexpr uint32_t kTmemCols = TOK < 32 ? 32 : TOK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStreamStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&a_full[b], 4);
            mbar_init(&a_empty[b], 1);
        }
        mbar_init(d_full, 1);
        mbar_init(drain, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tm_x);
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = *tmem_slot;
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            bool ok = true;
            uint32_t issued = 0, issued_phase = 0;
            const uint8_t* tile_packets =
                packets + (static_cast<int64_t>(tile) * chunks_total + c_begin) * L::raw_bytes;
            for (int i = 0; i < nchunks; ++i) {
                const int s = i % kStreamStages;
                const uint32_t par = static_cast<uint32_t>(i / kStreamStages) & 1u;
                if (!mbar_wait(&empty[s], par ^ 1u, status, 41)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&full[s], L::raw_bytes + L::x_bytes);
                bulk_load_1d(sraw + s * L::raw_bytes, tile_packets + static_cast<int64_t>(i) * L::raw_bytes,
                             L::raw_bytes, &full[s]);
                tma_load_2d(sx + s * L::x_bytes, &tm_x, &full[s], (c_begin + i) * 64, 0);
                issued |= 1u << s;
                issued_phase = (issued_phase & ~(1u << s)) | (par << s);
            }
            pdl_trigger();
            if (!ok) {  // let the copies in flight land before the CTA exits
                for (int s = 0; s < kStreamStages; ++s)
                    if (issued & (1u << s)) mbar_wait(&full[s], (issued_phase >> s) & 1u, status, 45);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(128, TOK);
            bool ok = true;
            for (int i = 0; i < nchunks && ok; ++i) {
                const int s = i % kStreamStages, ab = i & 1;
                if (!mbar_wait(&full[s], static_cast<uint32_t>(i / kStreamStages) & 1u, status, 42) ||
                    !mbar_wait(&a_full[ab], static_cast<uint32_t>(i >> 1) & 1u, status, 43)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(sa + ab * L::a_bytes);
                const uint32_t x_addr = smem_u32(sx + s * L::x_bytes);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    tc_mma_f16(tmem_d, smem_desc_sw128(a_addr + kk * 32), smem_desc_sw128(x_addr + kk * 32), idesc,
                               (i | kk) != 0 ? 1u : 0u);
                tc_commit(&empty[s]);
                tc_commit(&a_empty[ab]);
            }
            if (ok) tc_commit(d_full);
            tc_commit(drain);  // every MMA this thread issued is complete before TMEM is released
            mbar_wait(drain, 0, status, 46);
        }
    } else {
        const int tid = threadIdx.x - 64;  // 0..127
        const int j = tid & 7;             // 8-column group of the row
        const int rg = tid >> 3;           // rows rg, rg + 16, ...
        bool ok = true;
        for (int i = 0; i < nchunks; ++i) {
            const int s = i % kStreamStages, ab = i & 1;
            if (!mbar_wait(&full[s], static_cast<uint32_t>(i / kStreamStages) & 1u, status, 47) ||
                !mbar_wait(&a_empty[ab], (static_cast<uint32_t>(i >> 1) & 1u) ^ 1u, status, 44)) {
                ok = false;
                break;
            }
            const uint8_t* raw = sraw + s * L::raw_bytes;
            uint8_t* a = sa + ab * L::a_bytes;
#pragma unroll 2
            for (int it = 0; it < 8; ++it) {
                const int r = rg + 16 * it;
                float w[8];
                decode8<TYPE>(raw + r * cb, raw + 128 * cb + r * 8, j, w);
                __align__(16) __half2 h[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(w[2 * e], w[2 * e + 1]);
                *reinterpret_cast<uint4*>(a + r * 128 + ((j ^ (r & 7)) << 4)) = *reinterpret_cast<const uint4*>(h);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[ab]);
        }
        // Epilogue: TMEM lane quarter warp % 4 holds weight rows 32*quarter + lane.
        if (__all_sync(0xffffffffu, ok && mbar_wait(d_full, 0, status, 48))) {
            tc_fence_after();
            const int quarter = warp & 3;
            const int64_t row = static_cast<int64_t>(tile) * 128 + quarter * 32 + lane;
            uint32_t acc[TOK];
#pragma unroll
            for (int c = 0; c < TOK / 32; ++c)
                tc_ld_32x32b_x32(tmem_d + (static_cast<uint32_t>(quarter * 32) << 16) + c * 32,
                                 *reinterpret_cast<uint32_t(*)[32]>(acc + 32 * c));
            tc_wait_ld();
            auto finish = [&](int t, float v) {
                if (bias != nullptr) v += __ldg(bias + row);
                if (gelu) v = gelu_erf(v);
                y[t * ldy + row] = v;
            };
            if (splits == 1) {
                if (row < n) {
#pragma unroll
                    for (int t = 0; t < TOK; ++t)
                        if (t < m) finish(t, __uint_as_float(acc[t]));
                }
            } else if (row < n) {
                // Partials are [split][m][n], summed by splitk_reduce_kernel.
                float* part = partials + split * static_cast<int64_t>(m) * n;
#pragma unroll
                for (int t = 0; t < TOK; ++t)
                    if (t < m) part[t * n + row] = __uint_as_float(acc[t]);
            }
        }
        tc_fence_before();
    }
    // Reconverge each warp before the aligned CTA barrier (lane-0 role loops).
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_d, kTmemCols);
    }
}

// y[t][col] = act(sum over splits s of partials[s][t][col] + bias[col]), the
// splits summed in index order.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ partials, int splits,
                                                            int64_t split_stride, int m, int64_t n,
                                                            const float* __restrict__ bias, int gelu,
                                                            float* __restrict__ y, int64_t ldy) {
    pdl_wait();
    pdl_trigger();
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<int64_t>(m) * n) return;
    const int64_t t = idx / n, col = idx - t * n;
    float v = 0.0f;
    for (int s = 0; s < splits; ++s) v += partials[s * split_stride + idx];
    if (bias != nullptr) v += __ldg(bias + col);
    if (gelu) v = gelu_erf(v);
    y[t * ldy + col] = v;
}

struct SplitPlan {
    int chunks, n_tiles, splits, per_split;
};

SplitPlan plan_splits(int64_t n, int64_t k, int sms) {
    SplitPlan p{};
    p.chunks = static_cast<int>(k / 64);
    p.n_tiles = static_cast<int>((n + 127) / 128);
    // Two CTAs per SM in flight; at most 16 partial sums (their traffic stays
    // below the packed weights' for K >= 1024).
    int splits = std::max(1, std::min({2 * sms / std::max(p.n_tiles, 1), p.chunks, kMaxSplits}));
    p.per_split = (p.chunks + splits - 1) / splits;
    p.splits = (p.chunks + p.per_split - 1) / p.per_split;
    return p;
}

template <int TYPE, int TOK>
void run_stream(const samq_weights* w, const __half* x16, int64_t ldx, int64_t m, const float* bias, int gelu,
                float* y, int64_t ldy, float* partials, DeviceState& state, cudaStream_t stream) {
    using L = StreamSmem<TYPE, TOK>;
    const SplitPlan p = plan_splits(w->n, w->k, state.sm_count);
    CUtensorMap tx;
    encode_tensor_map_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x16, w->k, m, ldx * 2, 64, TOK,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    auto kernel = gemm_stream_kernel<TYPE, TOK>;
    set_smem_limit_once(state, reinterpret_cast<const void*>(kernel), L::total, "cudaFuncSetAttribute(stream smem)");
    const dim3 grid(p.n_tiles, p.splits);
    launch_pdl(kernel, grid, dim3(kStreamThreads), L::total, stream, "gemm_stream_kernel launch",
               static_cast<const uint8_t*>(w->packets), tx, w->n, static_cast<int>(m), p.chunks, p.per_split,
               p.splits, partials, bias, gelu, y, ldy, state.status);
    if (p.splits > 1)
        launch_pdl(splitk_reduce_kernel, dim3(static_cast<unsigned>((m * w->n + 255) / 256)), dim3(256), 0, stream,
                   "splitk_reduce_kernel launch", static_cast<const float*>(partials), p.splits, m * w->n,
                   static_cast<int>(m), w->n, bias, gelu, y, ldy);
}

template <int TOK>
void run_stream_type(const samq_weights* w, const __half* x16, int64_t ldx, int64_t m, const float* bias, int gelu,
                     float* y, int64_t ldy, float* partials, DeviceState& state, cudaStream_t stream) {
    switch (w->type) {
        case SAMQ_TYPE_Q8_0: run_stream<SAMQ_TYPE_Q8_0, TOK>(w, x16, ldx, m, bias, gelu, y, ldy, partials, state, stream); break;
        case SAMQ_TYPE_Q4_K: run_stream<SAMQ_TYPE_Q4_K, TOK>(w, x16, ldx, m, bias, gelu, y, ldy, partials, state, stream); break;
        case SAMQ_TYPE_Q5_K: run_stream<SAMQ_TYPE_Q5_K, TOK>(w, x16, ldx, m, bias, gelu, y, ldy, partials, state, stream); break;
        default: run_stream<SAMQ_TYPE_Q6_K, TOK>(w, x16, ldx, m, bias, gelu, y, ldy, partials, state, stream); break;
    }
}

}  // namespace

bool stream_eligible(const samq_weights* w, int64_t m) {
    return m >= 1 && m <= kStreamMaxRows && w->k % 64 == 0 && w->n >= 1;
}

size_t stream_partial_bytes(const samq_weights* w, int64_t m, int sms) {
    const SplitPlan p = plan_splits(w->n, w->k, sms);
    return p.splits > 1 ? static_cast<size_t>(p.splits) * m * w->n * sizeof(float) : 0;
}

void launch_linear_stream(const samq_weights* w, const __half* x16, int64_t ldx, int64_t m, const float* bias,
                          int epilogue, float* y, int64_t ldy, float* partials, DeviceState& state,
                          cudaStream_t stream) {
    const int gelu = epilogue == SAMQ_EPILOGUE_GELU_ERF ? 1 : 0;
    if (m <= 32)
        run_stream_type<32>(w, x16, ldx, m, bias, gelu, y, ldy, partials, state, stream);
    else
        run_stream_type<64>(w, x16, ldx, m, bias, gelu, y, ldy, partials, state, stream);
}

}  // namespace samq
