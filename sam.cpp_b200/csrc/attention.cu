// attention.cu -- K3: RoPE + windowed / global self-attention of a SAM 3 ViT
// block on the sm_100a tensor cores.
//
// Semantics (src/models/sam3/vision.hpp:152-227): the qkv linear's f32 output
// holds, per token, Q | K | V (each head-major, head h at channels
// 64h..64h+63).  RoPE rotates channel pairs (2i, 2i+1) of Q and K by
// (cos, sin) = freqs[pos][i] (vision.hpp:100-148), pos being the token's
// raster position inside its 24x24 window (windowed blocks) or in the whole
// grid (global blocks 7/15/23/31).  Attention is softmax(Q K^T / 8) V per head
// within each window (ggml_win_part, vision.hpp:170-173) or over the grid, and
// the output goes back to the raster token order (ggml_win_unpart, :226) as
// [token][head * 64 + d].
//
// Two kernels:
//   rope_pack_kernel  f32 qkv -> f16 Q (RoPE, x 1/8), K (RoPE), V^T, gathered
//                     into window-major order: Q,K [group*heads][n][64],
//                     V^T [group*heads][64][n].  The 1/8 softmax scale is a
//                     power of two, so folding it into Q is exact.
//   attention_kernel  one CTA per (128 queries, head, group): warp 0 TMA loads
//                     Q once and K / V^T blocks of 128 keys (double buffered);
//                     warp 1 issues tcgen05.mma S = Q K^T (M=128, N=128, K=64)
//                     into TMEM, then O += P V (M=128, N=64, K=128) into TMEM;
//                     warps 2-5 own one query row each: online softmax in the
//                     log2 domain with the MUFU exp2, P (f16) to swizzled
//                     shared memory, O rescaled in TMEM when the reference
//                     max moves by more than 8, and finally O / l to f32.
//                     K and V stages have separate barriers (K is released by
//                     the S MMA, V by the PV MMA); two CTAs fit per SM.
// Keys past the group's end are zero-filled by TMA and masked to -inf.  All
// waits are bounded (kStatusTimeout).  No TMA load uses multicast.
#include <algorithm>

#include "samq_internal.hpp"

namespace samq {
namespace {

constexpr int kHeadDim = 64;
constexpr int kQTile = 128;   // queries per CTA (MMA M)
constexpr int kKvTile = 128;  // keys per block (S MMA N, PV MMA K)
constexpr int kAttnThreads = 192;
constexpr float kLog2e = 1.4426950408889634f;

struct Geometry {
    int grid_w, grid_h, heads, window;
    int groups;   // windows (or 1)
    int group_n;  // tokens per group
};

// Raster token of position n of group g (global blocks: one group per image
// of a batch, stored image after image).
__device__ __forceinline__ int group_token(const Geometry& geo, int g, int n) {
    if (geo.window == 0) return g * geo.group_n + n;
    const int per_row = geo.grid_w / geo.window;
    const int wy = g / per_row, wx = g % per_row;
    const int ly = n / geo.window, lx = n % geo.window;
    return (wy * geo.window + ly) * geo.grid_w + wx * geo.window + lx;
}

// ---------------------------------------------------------------- pack

// One block per (64 tokens of a group, head, group): Q and K rotated and
// converted (8 channels per thread per step), V transposed through shared
// memory so that V^T rows (keys contiguous) are written coalesced.
__global__ void __launch_bounds__(256) rope_pack_kernel(const float* __restrict__ qkv, int64_t ldq,
                                                        const float* __restrict__ freqs, Geometry geo,
                                                        __half* __restrict__ qp, __half* __restrict__ kp,
                                                        __half* __restrict__ vt) {
    pdl_wait();
    pdl_trigger();
    __shared__ float vtile[64][kHeadDim + 1];
    const int chunk = blockIdx.x, h = blockIdx.y, g = blockIdx.z;
    const int E = geo.heads * kHeadDim;
    const int64_t gh = static_cast<int64_t>(g) * geo.heads + h;
    for (int u = threadIdx.x; u < 64 * 8; u += blockDim.x) {
        const int t = u >> 3, c8 = u & 7;
        const int n = chunk * 64 + t;
        if (n >= geo.group_n) continue;
        const int tok = group_token(geo, g, n);
        const float* row = qkv + static_cast<int64_t>(tok) * ldq + h * kHeadDim + c8 * 8;
        const float* fr = freqs + static_cast<int64_t>(n) * kHeadDim + c8 * 8;  // 4 (cos, sin) pairs
        const float4 f0 = __ldg(reinterpret_cast<const float4*>(fr));
        const float4 f1 = __ldg(reinterpret_cast<const float4*>(fr) + 1);
        const float cs[4] = {f0.x, f0.z, f1.x, f1.z}, sn[4] = {f0.y, f0.w, f1.y, f1.w};
#pragma unroll
        for (int which = 0; which < 2; ++which) {  // 0: Q, 1: K
            const float4 a = __ldg(reinterpret_cast<const float4*>(row + which * E));
            const float4 b = __ldg(reinterpret_cast<const float4*>(row + which * E) + 1);
            const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
            const float scale = which == 0 ? 0.125f : 1.0f;
            __align__(16) __half2 o[4];
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                const float re = __fsub_rn(__fmul_rn(x[2 * p], cs[p]), __fmul_rn(x[2 * p + 1], sn[p]));
                const float im = __fadd_rn(__fmul_rn(x[2 * p], sn[p]), __fmul_rn(x[2 * p + 1], cs[p]));
                o[p] = __floats2half2_rn(re * scale, im * scale);
            }
            __half* dst = (which == 0 ? qp : kp) + (gh * geo.group_n + n) * kHeadDim + c8 * 8;
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(o);
        }
    }
    // V: 64 tokens x 64 channels through shared memory.
    for (int u = threadIdx.x; u < 64 * 16; u += blockDim.x) {
        const int t = u >> 4, c4 = u & 15;
        const int n = chunk * 64 + t;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (n < geo.group_n) {
            const int tok = group_token(geo, g, n);
            v = __ldg(reinterpret_cast<const float4*>(qkv + static_cast<int64_t>(tok) * ldq + 2 * E + h * kHeadDim +
                                                      c4 * 4));
        }
        vtile[t][c4 * 4 + 0] = v.x;
        vtile[t][c4 * 4 + 1] = v.y;
        vtile[t][c4 * 4 + 2] = v.z;
        vtile[t][c4 * 4 + 3] = v.w;
    }
    __syncthreads();
    for (int u = threadIdx.x; u < 64 * 8; u += blockDim.x) {
        const int d = u >> 3, t8 = u & 7;  // channel row d, tokens t8*8 .. +8
        const int n0 = chunk * 64 + t8 * 8;
        if (n0 >= geo.group_n) continue;
        __align__(16) __half2 o[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) o[p] = __floats2half2_rn(vtile[t8 * 8 + 2 * p][d], vtile[t8 * 8 + 2 * p + 1][d]);
        __half* dst = vt + (gh * kHeadDim + d) * geo.group_n + n0;
        if (n0 + 8 <= geo.group_n) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(o);
        } else {
            const __half* oh = reinterpret_cast<const __half*>(o);
            for (int i = 0; n0 + i < geo.group_n; ++i) dst[i] = oh[i];
        }
    }
}

// ---------------------------------------------------------------- attention

// 2^x is ex2_mufu (samq_device.cuh): PTX ex2.approx.ftz, relative error ~2^-22,
// far below the f16 rounding of P; ex2(-inf) = +0, which masks keys for free.

// Rows keep a reference maximum m (log2 units) and only move it when a block's
// maximum exceeds it by more than this, so P = 2^(s - m) <= 2^8 (exact in
// f16 range terms) and O is rescaled in TMEM only a few times per row instead
// of at nearly every block.  The final O / l is the same softmax either way.
constexpr float kLazyRescale = 8.0f;

// Shared memory: 14 mbarriers + the TMEM slot in the first 128 bytes of the
// dynamic window, then the tiles at the next 1024-byte boundary (SW128
// atoms).  112 KB of tiles + 1 KB of slack keeps two CTAs resident per SM.
struct AttnSmem {
    static constexpr int q_off = 0;                              // 128 x 128 B
    static constexpr int k_off = q_off + kQTile * 128;           // 2 stages x 128 keys x 128 B
    static constexpr int v_off = k_off + 2 * kKvTile * 128;      // 2 stages x 2 halves x 64 ch x 128 B
    static constexpr int p_off = v_off + 2 * 2 * kHeadDim * 128; // 2 halves x 128 rows x 128 B
    static constexpr int tiles = p_off + 2 * kQTile * 128;
    static constexpr int header = 128;
    static constexpr int total = tiles + 1024;
};

__global__ void __launch_bounds__(kAttnThreads, 2)
attention_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, Geometry geo, float* __restrict__ out,
                 __half* __restrict__ out_h, int64_t ldo, DeviceStatus* status) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const uintptr_t raw = reinterpret_cast<uintptr_t>(smem_raw);
    const uintptr_t aligned = (raw + AttnSmem::header + 1023) & ~uintptr_t(1023);
    if (aligned + AttnSmem::tiles > raw + AttnSmem::total) {  // uniform over the CTA: no access made
        if (threadIdx.x == 0) atomicOr(&status->flags, kStatusLayout);
        return;
    }
    uint8_t* smem = reinterpret_cast<uint8_t*>(aligned);
    uint8_t* sq = smem + AttnSmem::q_off;
    uint8_t* sk = smem + AttnSmem::k_off;
    uint8_t* sv = smem + AttnSmem::v_off;
    uint8_t* sp = smem + AttnSmem::p_off;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);
    // K stages are released by the S MMA that read them, V stages by the PV
    // MMA, so K(j + 1) streams in while PV(j - 1) is still pending.
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;   // [2]
    uint64_t* k_empty = bars + 3;  // [2]
    uint64_t* v_full = bars + 5;   // [2]
    uint64_t* v_empty = bars + 7;  // [2]
    uint64_t* s_full = bars + 9;
    uint64_t* s_free = bars + 10;
    uint64_t* p_full = bars + 11;
    uint64_t* o_done = bars + 12;
    uint64_t* drain = bars + 13;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q_tile = blockIdx.x;
    const int gh = blockIdx.y;  // group * heads + head
    const int g = gh / geo.heads, h = gh % geo.heads;
    const int n_kv = (geo.group_n + kKvTile - 1) / kKvTile;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&k_full[b], 1);
            mbar_init(&k_empty[b], 1);
            mbar_init(&v_full[b], 1);
            mbar_init(&v_empty[b], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, 4);
        mbar_init(p_full, 4);
        mbar_init(o_done, 1);
        mbar_init(drain, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
    }
    if (warp == 1) tmem_alloc(tmem_slot, 256);  // S: columns 0..127, O: columns 128..191
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            bool ok = true;
            mbar_arrive_expect_tx(q_full, kQTile * 128);
            tma_load_3d(sq, &tm_q, q_full, 0, q_tile * kQTile, gh);
            // Bit b of k_issued / v_issued: stage b has a load in flight whose
            // phase parity is the same bit of *_phase.
            uint32_t k_issued = 0, k_phase = 0, v_issued = 0, v_phase = 0;
            for (int j = 0; j < n_kv && ok; ++j) {
                const int b = j & 1;
                const uint32_t par = static_cast<uint32_t>(j >> 1) & 1u;
                if (!mbar_wait(&k_empty[b], par ^ 1u, status, 21)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&k_full[b], kKvTile * 128);
                tma_load_3d(sk + b * kKvTile * 128, &tm_k, &k_full[b], 0, j * kKvTile, gh);
                k_issued |= 1u << b;
                k_phase = (k_phase & ~(1u << b)) | (par << b);
                if (!mbar_wait(&v_empty[b], par ^ 1u, status, 28)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&v_full[b], 2 * kHeadDim * 128);
                uint8_t* vb = sv + b * 2 * kHeadDim * 128;
                tma_load_3d(vb, &tm_v, &v_full[b], j * kKvTile, 0, gh);
                tma_load_3d(vb + kHeadDim * 128, &tm_v, &v_full[b], j * kKvTile + 64, 0, gh);
                v_issued |= 1u << b;
                v_phase = (v_phase & ~(1u << b)) | (par << b);
            }
            pdl_trigger();
            if (!ok) {  // let the loads in flight land before the CTA exits
                mbar_wait(q_full, 0, status, 25);
                for (int b = 0; b < 2; ++b) {
                    if (k_issued & (1u << b)) mbar_wait(&k_full[b], (k_phase >> b) & 1u, status, 25);
                    if (v_issued & (1u << b)) mbar_wait(&v_full[b], (v_phase >> b) & 1u, status, 25);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_f16_f32(kQTile, kKvTile);
            constexpr uint32_t idesc_o = idesc_f16_f32(kQTile, kHeadDim);
            const uint32_t tmem_s = tmem_base, tmem_o = tmem_base + 128;
            const uint32_t q_addr = smem_u32(sq);
            const uint32_t p_addr = smem_u32(sp);
            auto issue_s = [&](int j) {
                const uint32_t k_addr = smem_u32(sk + (j & 1) * kKvTile * 128);
#pragma unroll
                for (int kk = 0; kk < kHeadDim / 16; ++kk)
                    tc_mma_f16(tmem_s, smem_desc_sw128(q_addr + kk * 32), smem_desc_sw128(k_addr + kk * 32), idesc_s,
                               kk != 0 ? 1u : 0u);
                tc_commit(s_full);
                tc_commit(&k_empty[j & 1]);
            };
            // S(j + 1) is issued as soon as the softmax warps have copied S(j)
            // out of TMEM, so it runs under their exponentials; PV(j) follows
            // once P(j) is in shared memory.
            bool ok = mbar_wait(q_full, 0, status, 22) && mbar_wait(&k_full[0], 0, status, 23);
            if (ok) {
                tc_fence_after();
                issue_s(0);
            }
            for (int j = 0; j < n_kv && ok; ++j) {
                if (j + 1 < n_kv) {
                    if (!mbar_wait(&k_full[(j + 1) & 1], static_cast<uint32_t>((j + 1) >> 1) & 1u, status, 23) ||
                        !mbar_wait(s_free, static_cast<uint32_t>(j) & 1u, status, 24))
                        break;
                    tc_fence_after();
                    issue_s(j + 1);
                }
                if (!mbar_wait(p_full, static_cast<uint32_t>(j) & 1u, status, 26) ||
                    !mbar_wait(&v_full[j & 1], static_cast<uint32_t>(j >> 1) & 1u, status, 29))
                    break;
                tc_fence_after();
                const uint32_t v_addr = smem_u32(sv + (j & 1) * 2 * kHeadDim * 128);
#pragma unroll
                for (int kk = 0; kk < kKvTile / 16; ++kk) {
                    const uint32_t half = static_cast<uint32_t>(kk >> 2), off = static_cast<uint32_t>(kk & 3) * 32;
                    tc_mma_f16(tmem_o, smem_desc_sw128(p_addr + half * kQTile * 128 + off),
                               smem_desc_sw128(v_addr + half * kHeadDim * 128 + off), idesc_o,
                               (j > 0 || kk > 0) ? 1u : 0u);
                }
                tc_commit(o_done);
                tc_commit(&v_empty[j & 1]);
            }
            tc_commit(drain);
            mbar_wait(drain, 0, status, 27);
        }
    } else {
        // Softmax warps: TMEM lane quarter warp % 4 -> query rows 32*quarter + lane.
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t tmem_s = tmem_base + lane_off, tmem_o = tmem_base + 128 + lane_off;
        float m = -INFINITY, l = 0.0f;
        bool ok = true;
        uint8_t* prow0 = sp + row * 128;                 // keys 0..63
        uint8_t* prow1 = sp + kQTile * 128 + row * 128;  // keys 64..127
        for (int j = 0; j < n_kv; ++j) {
            // Warp-uniform decisions: the tcgen05.ld / st below are warp-collective.
            if (!__all_sync(0xffffffffu, mbar_wait(s_full, static_cast<uint32_t>(j) & 1u, status, 31))) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t s[4][32];
#pragma unroll
            for (int c = 0; c < 4; ++c) tc_ld_32x32b_x32(tmem_s + c * 32, s[c]);
            tc_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free);
            const int valid = geo.group_n - j * kKvTile;
            if (valid < kKvTile) {  // last block of a ragged group (same for the whole CTA)
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (c * 32 + i >= valid) s[c][i] = __float_as_uint(-INFINITY);
            }
            float mx4[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                mx4[c] = __uint_as_float(s[c][0]);
#pragma unroll
                for (int i = 1; i < 32; ++i) mx4[c] = fmaxf(mx4[c], __uint_as_float(s[c][i]));
            }
            const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * kLog2e;
            // First block: m = -inf, so the row always takes its maximum and
            // alpha = 2^-inf = 0 (l is still 0, and PV(0) overwrites O).
            const bool move = mx > m + kLazyRescale;
            const float m_new = move ? mx : m;
            const float alpha = move ? ex2_mufu(m - m_new) : 1.0f;
            m = m_new;
            // P = 2^(s log2e - m) as f16, kept in registers until PV(j-1) has
            // released P's shared-memory tile.
            const float neg_m = -m;
            float rs[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            uint32_t packed[16][4];
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const int c = u >> 2, base_i = (u & 3) * 8;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float x0 = fmaf(__uint_as_float(s[c][base_i + 2 * e]), kLog2e, neg_m);
                    const float x1 = fmaf(__uint_as_float(s[c][base_i + 2 * e + 1]), kLog2e, neg_m);
                    const float p0 = ex2_mufu(x0);
                    const float p1 = ex2_mufu(x1);
                    rs[e] += p0 + p1;
                    const __half2 hp = __floats2half2_rn(p0, p1);
                    packed[u][e] = *reinterpret_cast<const uint32_t*>(&hp);
                }
            }
            if (j > 0) {
                // PV(j-1) has finished: P's tile is free and O is stable.
                if (!__all_sync(0xffffffffu, mbar_wait(o_done, static_cast<uint32_t>(j - 1) & 1u, status, 32))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
            }
            // P row into the swizzled A tile: keys 0..63 in the first 128-byte
            // row, 64..127 in the second, 16-byte units permuted by row & 7.
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                uint8_t* base = u < 8 ? prow0 : prow1;
                *reinterpret_cast<uint4*>(base + (((u & 7) ^ (row & 7)) << 4)) =
                    make_uint4(packed[u][0], packed[u][1], packed[u][2], packed[u][3]);
            }
            l = l * alpha + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
            // O rescale after P is out (S no longer live): rows whose reference
            // maximum stayed scale by exactly 1; the warp takes the branch if
            // any of its rows moved.
            if (j > 0 && __any_sync(0xffffffffu, move)) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    uint32_t o[32];
                    tc_ld_32x32b_x32(tmem_o + c * 32, o);
                    tc_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tc_st_32x32b_x32(tmem_o + c * 32, o);
                }
                tc_wait_st();
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        if (__all_sync(0xffffffffu, ok && mbar_wait(o_done, static_cast<uint32_t>(n_kv - 1) & 1u, status, 33))) {
            tc_fence_after();
            const int n = q_tile * kQTile + row;
            const float inv = 1.0f / l;
            uint32_t o[2][32];
            tc_ld_32x32b_x32(tmem_o, o[0]);
            tc_ld_32x32b_x32(tmem_o + 32, o[1]);
            tc_wait_ld();
            const bool valid_row = n < geo.group_n;
            const int64_t tok = valid_row ? group_token(geo, g, n) : 0;
            if (out_h != nullptr) {
                // Q8_1 operand of the proj linear, staged from the f32 values
                // the f32 path would store (two 32-channel blocks per row).
                uint4* dst = reinterpret_cast<uint4*>(out_h + tok * ldo + h * kHeadDim);
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    float v[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(o[c][i]) * inv;
                    uint32_t packed[16];
                    const bool bad = stage_q8_1<1, 32>(v, packed);
                    record_range(bad && valid_row, status);
                    if (valid_row) {
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            dst[c * 4 + j] = make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
                    }
                }
            } else if (valid_row) {
                float* dst = out + tok * ldo + h * kHeadDim;
#pragma unroll
                for (int c = 0; c < 2; ++c)
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4*>(dst + c * 32 + i) =
                            make_float4(__uint_as_float(o[c][i]) * inv, __uint_as_float(o[c][i + 1]) * inv,
                                        __uint_as_float(o[c][i + 2]) * inv, __uint_as_float(o[c][i + 3]) * inv);
            }
        }
        tc_fence_before();
    }
    // Reconverge each warp before the aligned CTA barrier (lane-0 role loops).
    __syncwarp();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 256);
    }
}

// A batch of images is one grid of grid_w x (batch * grid_h) tokens (images
// stacked vertically): windows never straddle two images since the window
// divides grid_h; a global block attends within each image (one group each).
Geometry make_geometry(int grid_w, int grid_h, int heads, int window, int batch) {
    Geometry geo{grid_w, grid_h * batch, heads, window, batch, grid_w * grid_h};
    if (window > 0) {
        geo.groups = (grid_w / window) * (grid_h * batch / window);
        geo.group_n = window * window;
    }
    return geo;
}

}  // namespace

size_t attention_scratch_bytes(int grid_w, int grid_h, int heads) {
    return static_cast<size_t>(3) * grid_w * grid_h * heads * kHeadDim * sizeof(__half) + 256;
}

void launch_attention_packed(const __half* qp, const __half* kp, const __half* vt, int grid_w, int grid_h, int heads,
                             int window, int batch, float* out, __half* out_h, int64_t ldo, DeviceState& state,
                             cudaStream_t stream) {
    const Geometry geo = make_geometry(grid_w, grid_h, heads, window, batch);
    const uint64_t gh = static_cast<uint64_t>(geo.groups) * heads;
    CUtensorMap tq, tk, tv;
    encode_tensor_map_3d(&tq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, qp, kHeadDim, geo.group_n, gh, kHeadDim * 2,
                         static_cast<uint64_t>(geo.group_n) * kHeadDim * 2, kHeadDim, kQTile,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    encode_tensor_map_3d(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kp, kHeadDim, geo.group_n, gh, kHeadDim * 2,
                         static_cast<uint64_t>(geo.group_n) * kHeadDim * 2, kHeadDim, kKvTile,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    encode_tensor_map_3d(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, vt, geo.group_n, kHeadDim, gh,
                         static_cast<uint64_t>(geo.group_n) * 2, static_cast<uint64_t>(geo.group_n) * kHeadDim * 2,
                         64, kHeadDim, CU_TENSOR_MAP_SWIZZLE_128B);
    set_smem_limit_once(state, reinterpret_cast<const void*>(attention_kernel), AttnSmem::total,
                        "cudaFuncSetAttribute(attention smem)");
    launch_pdl(attention_kernel, dim3((geo.group_n + kQTile - 1) / kQTile, static_cast<unsigned>(gh)),
               dim3(kAttnThreads), AttnSmem::total, stream, "attention_kernel launch", tq, tk, tv, geo, out, out_h, ldo,
               state.status);
}

void launch_vit_attention(const float* qkv, int64_t ldq, int grid_w, int grid_h, int heads, int window,
                          const float* freqs, float* out, int64_t ldo, void* packed, DeviceState& state,
                          cudaStream_t stream) {
    const Geometry geo = make_geometry(grid_w, grid_h, heads, window, 1);
    const int64_t per = static_cast<int64_t>(geo.groups) * heads * geo.group_n * kHeadDim;
    __half* qp = static_cast<__half*>(packed);
    __half* kp = qp + per;
    __half* vt = kp + per;
    launch_pdl(rope_pack_kernel, dim3((geo.group_n + 63) / 64, heads, geo.groups), dim3(256), 0, stream,
               "rope_pack_kernel launch", qkv, ldq, freqs, geo, qp, kp, vt);
    launch_attention_packed(qp, kp, vt, grid_w, grid_h, heads, window, 1, out, nullptr, ldo, state, stream);
}

}  // namespace samq
