// attention_tc.cu -- F32-precise attention on the sm_100a tensor cores for
// large query and key counts: softmax(Q K^T * scale) V per head, no mask
// (the fusion encoder's self-attention over the image tokens,
// src/models/sam3/fusion_encoder.hpp:60-90, kept at F32 precision by the
// reference in both CUDA compute modes, src/runtime/ggml/backends/cuda.hpp:86-91).
//
// F32 accuracy from TF32 MMAs (the split of dense.cu): every operand x is
// split once into hi = rna_tf32(x) and lo = rna_tf32(x - hi), and each product
// is hi*hi + hi*lo + lo*hi.  The hi*hi terms and the two correction terms
// accumulate in separate TMEM regions and are added in registers with f32
// round-to-nearest (the tensor core's accumulation rounds toward zero per MMA).
//   S = Q K^T:  M = 128 queries, N = 64 keys, K = head dim (32 / 64)
//   O = P V:    M = 128 queries, N = head dim, K = 64 keys
// The online softmax runs in f32 registers of the softmax warps (one query row
// per thread, read from TMEM); P goes back to TMEM as its hi / lo split and is
// the A operand of P V straight from there, so the P V MMAs read only V from
// shared memory (with 4-byte operands, shared-memory bandwidth for A would
// otherwise bound every MMA).
// Per 64-key tile the output O_t is a fresh accumulator and the softmax warps
// add it as o = o * alpha + O_t (the blocked sum of the SIMT kernel).
//
// One CTA per (128 queries, head), 224 threads (7 warps, so no SM
// sub-partition holds more than two and every thread may use 255 registers):
//   warps 0-1  loaders: Q once (split into hi / lo), then the K and V^T tiles:
//              either TMA loads of the TF32 hi / lo planes that split_kv_kernel
//              wrote once per call (one thread; the launchers' default when the
//              caller gives plane scratch), or reading the f32 rows and
//              splitting every tile themselves (128-byte swizzle either way)
//   warp 2     TMEM owner and MMA issuer (S and P V in readiness order)
//   warps 3-6  softmax (TMEM lane quarter = warp % 4)
// Measured on B200: splitting every tile in the loader warps bounded the kernel
// (~9000 cycles per 64-key tile at head dim 64); the TMA-fed form runs the
// fusion self-attention (5184^2 x 8 x 32) in 478 us against 675.
// No TMA multicast; every mbarrier wait is bounded (kStatusTimeout on expiry).
#include <algorithm>
#include <cmath>

#include "samq_internal.hpp"

namespace samq {
namespace {

constexpr int kQ = 128;          // queries per CTA
constexpr int kKeys = 64;        // keys per tile
constexpr int kLoaders = 2;     // loader warps
constexpr int kMmaWarp = kLoaders;
constexpr int kTcThreads = 32 * (kLoaders + 1 + 4);  // 7 warps: at most 2 per SM sub-partition

__host__ __device__ constexpr uint32_t idesc_tf32_mn(int m, int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D (+)= A(tmem) * B(smem desc)^T, kind::tf32: A is M lanes x K columns of TMEM.
__device__ __forceinline__ void mma_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

template <int HD>
struct TcLayout {
    static constexpr int stages = HD == 32 ? 4 : 2;           // K / V tiles in flight
    static constexpr int p_bufs = 1;                          // P (TMEM), S and O: one buffer each
    static constexpr int s_bufs = 1;
    static constexpr int o_bufs = 1;
    static constexpr int chunks = HD / 32;                    // 128-byte swizzle rows along the head dim
    static constexpr int q_bytes = chunks * kQ * 128;         // one of hi / lo
    static constexpr int k_bytes = chunks * kKeys * 128;      // K tile [64 keys][HD], one of hi / lo
    static constexpr int v_bytes = 2 * HD * 128;              // V^T tile [HD][64 keys], one of hi / lo
    static constexpr int q_off = 0;
    static constexpr int k_off = q_off + 2 * q_bytes;
    static constexpr int v_off = k_off + stages * 2 * k_bytes;
    static constexpr int bar_off = v_off + stages * 2 * v_bytes;
    static constexpr int bars = 1 + 2 * stages + 2 * s_bufs + p_bufs + 2 * o_bufs + 1;
    static constexpr int total = bar_off + bars * 8 + 16 + 1024;
    // TMEM columns: P hi, P lo (64 each), S as three accumulators (hi*hi,
    // hi*lo, lo*hi: independent MMA chains), O likewise.
    static constexpr uint32_t p_col = 0;
    __host__ __device__ static constexpr uint32_t s_col(int b) {
        return static_cast<uint32_t>(2 * kKeys + b * 3 * kKeys);
    }
    __host__ __device__ static constexpr uint32_t o_col(int b) {
        return static_cast<uint32_t>(2 * kKeys + s_bufs * 3 * kKeys + b * 3 * HD);
    }
    static_assert(2 * kKeys + s_bufs * 3 * kKeys + o_bufs * 3 * HD <= 512, "TMEM columns");
};

// Byte offset of element (row, k) of a K-major operand tile stored as
// 128-byte-swizzled chunks of 32 f32 along k, `rows` rows per chunk.
__device__ __forceinline__ uint32_t sw_off(int row, int k, int rows) {
    const int chunk = k >> 5, kin = k & 31;
    return static_cast<uint32_t>(chunk * rows * 128 + row * 128 + ((((kin >> 2) ^ (row & 7)) << 4) | ((kin & 3) << 2)));
}

struct TcArgs {
    const float* q;
    const float* k;
    const float* v;
    float* out;
    int64_t ldq, ldk, ldv, ldo;
    int lq, lk;
    // Groups (blockIdx.z): independent attention problems of lq queries / lk
    // keys whose rows follow each other in q, k, v (ViT windows or images).
    // Output row of (group g, query n): g * lq + n, or with out_window > 0 the
    // raster token of window g in a grid out_grid_w wide (ggml_win_unpart).
    int out_window, out_grid_w;
    float scale_log2e;  // softmax scale x log2(e)
    DeviceStatus* status;
    // Key split (one group only): with `part`, CTA z covers keys
    // [z kps, (z + 1) kps) (kps a multiple of 64) and writes its unnormalized
    // O, row maximum (natural-log units) and row sum to part
    // [splits][heads][lq][HD + 2] for launch_attention_combine.
    float* part = nullptr;
    int kps = 0;
};

// K and V^T of every (group, head) split once into TF32 hi / lo planes for the
// TMA-fed kernel (attention_tc_kernel<HD, true>): K planes [p][gh][lk][HD] and
// V^T planes [p][gh][HD][lk], p = 0 hi, 1 lo, gh = g * heads + h; a group's
// key rows follow each other in k / v with strides ldk / ldv (lk % 4 == 0).  One block
// per (64 keys, head, group); V goes through shared memory so that V^T rows
// (keys contiguous) are written coalesced.
template <int HD>
__global__ void __launch_bounds__(256) split_kv_kernel(const float* __restrict__ k, int64_t ldk,
                                                       const float* __restrict__ v, int64_t ldv, int lk, int heads,
                                                       int groups, float* __restrict__ kp, float* __restrict__ vtp) {
    pdl_wait();
    pdl_trigger();
    __shared__ float vt[64][HD + 1];
    const int n0 = blockIdx.x * 64, h = blockIdx.y, g = blockIdx.z;
    const int64_t gh = static_cast<int64_t>(g) * heads + h;
    const int64_t plane_k = static_cast<int64_t>(groups) * heads * lk * HD;  // elements per hi / lo plane
    const float* kg = k + static_cast<int64_t>(g) * lk * ldk + h * HD;
    const float* vg = v + static_cast<int64_t>(g) * lk * ldv + h * HD;
    for (int u = threadIdx.x; u < 64 * (HD / 4); u += blockDim.x) {
        const int r = u / (HD / 4), d4 = u % (HD / 4), n = n0 + r;
        float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (n < lk) {
            const float4 xk = __ldg(reinterpret_cast<const float4*>(kg + static_cast<int64_t>(n) * ldk) + d4);
            float4 hi, lo;
            split_tf32(xk.x, hi.x, lo.x);
            split_tf32(xk.y, hi.y, lo.y);
            split_tf32(xk.z, hi.z, lo.z);
            split_tf32(xk.w, hi.w, lo.w);
            const int64_t o = (gh * lk + n) * HD + 4 * d4;
            *reinterpret_cast<float4*>(kp + o) = hi;
            *reinterpret_cast<float4*>(kp + plane_k + o) = lo;
            xv = __ldg(reinterpret_cast<const float4*>(vg + static_cast<int64_t>(n) * ldv) + d4);
        }
        vt[r][4 * d4] = xv.x;
        vt[r][4 * d4 + 1] = xv.y;
        vt[r][4 * d4 + 2] = xv.z;
        vt[r][4 * d4 + 3] = xv.w;
    }
    __syncthreads();
    for (int u = threadIdx.x; u < HD * 16; u += blockDim.x) {  // HD rows x 16 groups of 4 keys
        const int d = u / 16, k4 = u % 16, n = n0 + 4 * k4;
        if (n >= lk) continue;  // lk % 4 == 0: a group of 4 keys is wholly in or out
        float4 hi, lo;
        split_tf32(vt[4 * k4][d], hi.x, lo.x);
        split_tf32(vt[4 * k4 + 1][d], hi.y, lo.y);
        split_tf32(vt[4 * k4 + 2][d], hi.z, lo.z);
        split_tf32(vt[4 * k4 + 3][d], hi.w, lo.w);
        const int64_t o = (gh * HD + d) * lk + n;
        *reinterpret_cast<float4*>(vtp + o) = hi;
        *reinterpret_cast<float4*>(vtp + plane_k + o) = lo;
    }
}

// Softmax warps: wait for P_j V_j (O buffer j % 2), add it as
// o = o * alpha + (hi*hi + corrections), release the buffer.
template <int HD, class L>
__device__ __forceinline__ bool take_o(float (&o)[HD], float alpha, int j, uint64_t* o_full, uint64_t* o_empty,
                                       uint32_t tmem_lane, int lane, DeviceStatus* status) {
    const int b = j % L::o_bufs;
    if (!__all_sync(0xffffffffu, mbar_poll(&o_full[b], (j / L::o_bufs) & 1u, status, 88))) return false;
    tc_fence_after();
#pragma unroll
    for (int c0 = 0; c0 < HD; c0 += 32) {
        uint32_t o0[32], o1[32], o2[32];
        tc_ld_32x32b_x32(tmem_lane + L::o_col(b) + c0, o0);
        tc_ld_32x32b_x32(tmem_lane + L::o_col(b) + HD + c0, o1);
        tc_ld_32x32b_x32(tmem_lane + L::o_col(b) + 2 * HD + c0, o2);
        tc_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c)
            o[c0 + c] = fmaf(o[c0 + c], alpha,
                             __uint_as_float(o0[c]) + (__uint_as_float(o1[c]) + __uint_as_float(o2[c])));
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&o_empty[b]);
    return true;
}

// SPLIT: K and V^T come as the TF32 hi / lo planes of split_kv_kernel through
// TMA (tm_k: [2 x groups x heads][lk][HD], tm_vt: [2 x groups x heads][HD][lk],
// boxes of 32 f32 x 64 keys / HD channels, 128-byte swizzle), issued by one
// thread of loader warp 0; otherwise the two loader warps read the f32 rows
// and split them.  Q is read and split by the loader warps in both forms.
template <int HD, bool SPLIT>
__global__ void __launch_bounds__(kTcThreads, 1) attention_tc_kernel(const TcArgs a,
                                                                     const __grid_constant__ CUtensorMap tm_k,
                                                                     const __grid_constant__ CUtensorMap tm_vt) {
    using L = TcLayout<HD>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::bar_off);
    uint64_t* q_full = bars;
    uint64_t* kv_full = q_full + 1;
    uint64_t* kv_empty = kv_full + L::stages;
    uint64_t* s_full = kv_empty + L::stages;
    uint64_t* s_empty = s_full + L::s_bufs;
    uint64_t* p_full = s_empty + L::s_bufs;
    uint64_t* o_full = p_full + L::p_bufs;
    uint64_t* o_empty = o_full + L::o_bufs;
    uint64_t* drain = o_empty + L::o_bufs;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    DeviceStatus* status = a.status;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * kQ, h = blockIdx.y;
    const int g = a.part ? 0 : static_cast<int>(blockIdx.z);
    const int split = a.part ? static_cast<int>(blockIdx.z) : 0;
    // This CTA's key tiles: all of them, or its split's range [t_begin, +tiles).
    const int all_tiles = (a.lk + kKeys - 1) / kKeys;
    const int t_begin = a.part ? split * (a.kps / kKeys) : 0;
    const int tiles = a.part ? max(0, min(all_tiles, t_begin + a.kps / kKeys) - t_begin) : all_tiles;
    const int key_base = t_begin * kKeys;
    const float* gq = a.q + int64_t(g) * a.lq * a.ldq;
    const float* gk = a.k + int64_t(g) * a.lk * a.ldk;
    const float* gv = a.v + int64_t(g) * a.lk * a.ldv;

    if (threadIdx.x == 0) {
        mbar_init(q_full, kLoaders);
        for (int s = 0; s < L::stages; ++s) {
            mbar_init(&kv_full[s], SPLIT ? 1 : kLoaders);
            mbar_init(&kv_empty[s], 1);
        }
        for (int b = 0; b < L::s_bufs; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&s_empty[b], 4);
        }
        for (int b = 0; b < L::o_bufs; ++b) {
            mbar_init(&o_full[b], 1);
            mbar_init(&o_empty[b], 4);
        }
        for (int b = 0; b < L::p_bufs; ++b) mbar_init(&p_full[b], 4);
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == kMmaWarp) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();

    if (warp < kLoaders) {
        // ---- loaders ---------------------------------------------------------
        const int t = threadIdx.x;  // 0 .. 32 kLoaders - 1
        uint8_t* qh = smem + L::q_off;
        uint8_t* ql = qh + L::q_bytes;
        // Every load of a tile is issued before any of them is used, so a
        // tile costs one global latency, not one per float4.
        constexpr int kLt = 32 * kLoaders;
        constexpr int kQLoads = kQ * (HD / 4) / kLt, kKvLoads = kKeys * (HD / 4) / kLt;
        {
            float4 x[kQLoads];
#pragma unroll
            for (int i = 0; i < kQLoads; ++i) {
                const int idx = t + kLt * i, r = idx / (HD / 4), d4 = idx % (HD / 4), n = q0 + r;
                x[i] = n < a.lq ? __ldg(reinterpret_cast<const float4*>(gq + int64_t(n) * a.ldq + h * HD) + d4)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < kQLoads; ++i) {
                const int idx = t + kLt * i, r = idx / (HD / 4), d4 = idx % (HD / 4);
                float4 hi, lo;
                split_tf32(x[i].x, hi.x, lo.x);
                split_tf32(x[i].y, hi.y, lo.y);
                split_tf32(x[i].z, hi.z, lo.z);
                split_tf32(x[i].w, hi.w, lo.w);
                const uint32_t off = sw_off(r, 4 * d4, kQ);
                *reinterpret_cast<float4*>(qh + off) = hi;
                *reinterpret_cast<float4*>(ql + off) = lo;
            }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_full);
        if constexpr (SPLIT) {
            if (warp == 0 && lane == 0) {
                const int gh = g * gridDim.y + h, planes = (a.part ? 1 : gridDim.z) * gridDim.y;
                uint32_t issued = 0, issued_phase = 0;  // per stage: loads in flight and their phase parity
                for (int j = 0; j < tiles; ++j) {
                    const int s = j % L::stages, key0 = key_base + j * kKeys;
                    const uint32_t par = static_cast<uint32_t>(j / L::stages) & 1u;
                    if (!mbar_wait(&kv_empty[s], par ^ 1u, status, 81)) break;
                    mbar_arrive_expect_tx(&kv_full[s], 2 * L::k_bytes + 2 * L::v_bytes);
                    uint8_t* kh = smem + L::k_off + s * 2 * L::k_bytes;
                    uint8_t* vh = smem + L::v_off + s * 2 * L::v_bytes;
#pragma unroll
                    for (int pl = 0; pl < 2; ++pl) {
#pragma unroll
                        for (int c = 0; c < HD / 32; ++c)
                            tma_load_3d(kh + pl * L::k_bytes + c * kKeys * 128, &tm_k, &kv_full[s], c * 32, key0,
                                        gh + pl * planes);
#pragma unroll
                        for (int c = 0; c < kKeys / 32; ++c)
                            tma_load_3d(vh + pl * L::v_bytes + c * HD * 128, &tm_vt, &kv_full[s], key0 + c * 32, 0,
                                        gh + pl * planes);
                    }
                    issued |= 1u << s;
                    issued_phase = (issued_phase & ~(1u << s)) | (par << s);
                }
                // Let every copy in flight land before the CTA can exit.
                for (int s = 0; s < L::stages; ++s)
                    if (issued & (1u << s)) mbar_wait(&kv_full[s], (issued_phase >> s) & 1u, status, 81);
            }
        }
        for (int j = 0; j < tiles && !SPLIT; ++j) {
            const int s = j % L::stages;
            const int key0 = key_base + j * kKeys;
            float4 xk[kKvLoads], xv[kKvLoads];
#pragma unroll
            for (int i = 0; i < kKvLoads; ++i) {
                const int idx = t + kLt * i;
                const int rk = idx / (HD / 4), dk = idx % (HD / 4), nk = key0 + rk;
                const int rv = idx % kKeys, dv = idx / kKeys, nv = key0 + rv;
                xk[i] = nk < a.lk ? __ldg(reinterpret_cast<const float4*>(gk + int64_t(nk) * a.ldk + h * HD) + dk)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
                xv[i] = nv < a.lk ? __ldg(reinterpret_cast<const float4*>(gv + int64_t(nv) * a.ldv + h * HD) + dv)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if (!__all_sync(0xffffffffu, mbar_poll(&kv_empty[s], ((j / L::stages) & 1u) ^ 1u, status, 81))) break;
            uint8_t* kh = smem + L::k_off + s * 2 * L::k_bytes;
            uint8_t* kl = kh + L::k_bytes;
            uint8_t* vh = smem + L::v_off + s * 2 * L::v_bytes;
            uint8_t* vl = vh + L::v_bytes;
#pragma unroll
            for (int i = 0; i < kKvLoads; ++i) {
                const int idx = t + kLt * i, r = idx / (HD / 4), d4 = idx % (HD / 4);
                float4 hi, lo;
                split_tf32(xk[i].x, hi.x, lo.x);
                split_tf32(xk[i].y, hi.y, lo.y);
                split_tf32(xk[i].z, hi.z, lo.z);
                split_tf32(xk[i].w, hi.w, lo.w);
                const uint32_t off = sw_off(r, 4 * d4, kKeys);
                *reinterpret_cast<float4*>(kh + off) = hi;
                *reinterpret_cast<float4*>(kl + off) = lo;
            }
            // V^T: row = channel d, k index = key; lanes run along the keys.
#pragma unroll
            for (int i = 0; i < kKvLoads; ++i) {
                const int idx = t + kLt * i, r = idx % kKeys, d4 = idx / kKeys;
                const float xs[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float hi, lo;
                    split_tf32(xs[e], hi, lo);
                    const uint32_t off = sw_off(4 * d4 + e, r, HD);
                    *reinterpret_cast<float*>(vh + off) = hi;
                    *reinterpret_cast<float*>(vl + off) = lo;
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&kv_full[s]);
        }
    } else if (warp == kMmaWarp) {
        // ---- MMA issuer --------------------------------------------------------
        if (lane == 0) {
            constexpr uint32_t id_s = idesc_tf32_mn(kQ, kKeys);
            constexpr uint32_t id_o = idesc_tf32_mn(kQ, HD);
            const uint32_t qh = smem_u32(smem + L::q_off), ql = qh + L::q_bytes;
            bool ok = mbar_wait(q_full, 0, status, 82);
            // Issue S_js and P_jo V_jo in whichever order their inputs become
            // ready (S_{j+1} runs ahead of P_j V_j by at most one tile).  The
            // readiness probes do not block; the loop is bounded by the wait
            // timeout like every other wait.
            auto issue_s = [&](int j) {
                const int s = j % L::stages, b = j % L::s_bufs;
                const uint32_t kh = smem_u32(smem + L::k_off + s * 2 * L::k_bytes), kl = kh + L::k_bytes;
                const uint32_t d0 = tmem_base + L::s_col(b), d1 = d0 + kKeys, d2 = d0 + 2 * kKeys;
#pragma unroll
                for (int t = 0; t < HD / 8; ++t) {
                    const uint32_t qo = (t >> 2) * kQ * 128 + (t & 3) * 32, ko = (t >> 2) * kKeys * 128 + (t & 3) * 32;
                    const uint32_t acc = t != 0 ? 1u : 0u;
                    mma_tf32(d0, smem_desc_sw128(qh + qo), smem_desc_sw128(kh + ko), id_s, acc);
                    mma_tf32(d1, smem_desc_sw128(qh + qo), smem_desc_sw128(kl + ko), id_s, acc);
                    mma_tf32(d2, smem_desc_sw128(ql + qo), smem_desc_sw128(kh + ko), id_s, acc);
                }
                tc_commit(&s_full[b]);
            };
            auto issue_o = [&](int j) {
                const int s = j % L::stages, b = j % L::o_bufs;
                const uint32_t vh = smem_u32(smem + L::v_off + s * 2 * L::v_bytes), vl = vh + L::v_bytes;
                const uint32_t ph = tmem_base + L::p_col, pl = ph + kKeys;
                const uint32_t d0 = tmem_base + L::o_col(b), d1 = d0 + HD, d2 = d0 + 2 * HD;
#pragma unroll
                for (int t = 0; t < kKeys / 8; ++t) {
                    const uint32_t vo = (t >> 2) * HD * 128 + (t & 3) * 32;
                    const uint32_t acc = t != 0 ? 1u : 0u;
                    mma_tf32_ts(d0, ph + 8 * t, smem_desc_sw128(vh + vo), id_o, acc);
                    mma_tf32_ts(d1, ph + 8 * t, smem_desc_sw128(vl + vo), id_o, acc);
                    mma_tf32_ts(d2, pl + 8 * t, smem_desc_sw128(vh + vo), id_o, acc);
                }
                tc_commit(&o_full[b]);
                tc_commit(&kv_empty[s]);
            };
            int js = 0, jo = 0;  // next S / next P V to issue
            uint64_t last = global_timer_ns();  // time of the last issue
            uint32_t spin = 0;
            while (ok && jo < tiles) {
                bool progressed = false;
                // S_js needs its K tile, a free S buffer, and (to keep at most one
                // tile of lookahead over P V) js <= jo + 1.
                if (js < tiles && js <= jo + 1 && mbar_test_wait(&kv_full[js % L::stages], (js / L::stages) & 1u) &&
                    mbar_test_wait(&s_empty[js % L::s_bufs], ((js / L::s_bufs) & 1u) ^ 1u)) {
                    tc_fence_after();
                    issue_s(js++);
                    progressed = true;
                }
                if (jo < js && mbar_test_wait(&p_full[jo % L::p_bufs], (jo / L::p_bufs) & 1u) &&
                    mbar_test_wait(&o_empty[jo % L::o_bufs], ((jo / L::o_bufs) & 1u) ^ 1u)) {
                    tc_fence_after();
                    issue_o(jo++);
                    progressed = true;
                }
                if (progressed) {
                    spin = 0;
                } else if ((++spin & 63u) == 0) {
                    const uint64_t now = global_timer_ns();
                    if (spin == 64) last = now;  // first check of this stall
                    if (now - last > kWaitTimeoutNs) {  // no issue possible for a whole wait limit
                        atomicOr(&status->flags, kStatusTimeout);
                        atomicExch(&status->timeout_site, 83u);
                        ok = false;
                    }
                }
            }
            tc_commit(drain);
            mbar_wait(drain, 0, status, 87);
        }
    } else {
        // ---- softmax -----------------------------------------------------------
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;  // query q0 + row
        const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
        float o[HD], m = -INFINITY, l = 0.0f, alpha_prev = 1.0f;
#pragma unroll
        for (int c = 0; c < HD; ++c) o[c] = 0.0f;
        bool ok = true;
        for (int j = 0; j < tiles && ok; ++j) {
            const int b = j % L::s_bufs;
            if (!__all_sync(0xffffffffu, mbar_poll(&s_full[b], (j / L::s_bufs) & 1u, status, 89))) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sv[kKeys];  // raw scores Q . K (scale applied in the exponent)
#pragma unroll
            for (int c0 = 0; c0 < kKeys; c0 += 32) {
                uint32_t s0[32], s1[32], s2[32];
                tc_ld_32x32b_x32(tmem_base + lane_addr + L::s_col(b) + c0, s0);
                tc_ld_32x32b_x32(tmem_base + lane_addr + L::s_col(b) + kKeys + c0, s1);
                tc_ld_32x32b_x32(tmem_base + lane_addr + L::s_col(b) + 2 * kKeys + c0, s2);
                tc_wait_ld();
#pragma unroll
                for (int c = 0; c < 32; ++c)
                    sv[c0 + c] = __uint_as_float(s0[c]) + (__uint_as_float(s1[c]) + __uint_as_float(s2[c]));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_empty[b]);
            const int key0 = key_base + j * kKeys;
            if (key0 + kKeys > a.lk) {
#pragma unroll
                for (int c = 0; c < kKeys; ++c)
                    if (key0 + c >= a.lk) sv[c] = -INFINITY;
            }
            float pm[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) pm[i] = sv[i];
#pragma unroll
            for (int c = 8; c < kKeys; ++c) pm[c & 7] = fmaxf(pm[c & 7], sv[c]);
            const float mx = fmaxf(fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])), fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7]))), m);
            // exp(scale (s - m)) = 2^(s c - m c), c = scale log2(e): one FMA and the
            // MUFU exponential (relative error ~2^-22) per score.
            const float m_use = mx == -INFINITY ? 0.0f : mx;
            const float mc = m_use * a.scale_log2e;
            const float alpha = ex2_mufu(fmaf(m, a.scale_log2e, -mc));
            float ps[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) ps[i] = 0.0f;
#pragma unroll
            for (int c = 0; c < kKeys; ++c) {
                sv[c] = ex2_mufu(fmaf(sv[c], a.scale_log2e, -mc));
                ps[c & 7] += sv[c];
            }
            const float sum = ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
            l = fmaf(l, alpha, sum);
            m = mx;
            // P (TMEM) is free once P_{j-1} V_{j-1} is done: take O_{j-1} first.
            if (j > 0) {
                if (!take_o<HD, L>(o, alpha_prev, j - 1, o_full, o_empty, tmem_base + lane_addr, lane, status)) {
                    ok = false;
                    break;
                }
            }
            alpha_prev = alpha;
#pragma unroll
            for (int c0 = 0; c0 < kKeys; c0 += 32) {
                uint32_t hi[32], lo[32];
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    float h, lw;
                    split_tf32(sv[c0 + c], h, lw);
                    hi[c] = __float_as_uint(h);
                    lo[c] = __float_as_uint(lw);
                }
                tc_st_32x32b_x32(tmem_base + lane_addr + L::p_col + c0, hi);
                tc_st_32x32b_x32(tmem_base + lane_addr + L::p_col + kKeys + c0, lo);
            }
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[0]);
        }
        if (ok && tiles > 0)
            ok = take_o<HD, L>(o, alpha_prev, tiles - 1, o_full, o_empty, tmem_base + lane_addr, lane, status);
        pdl_trigger();
        const int n = q0 + row;
        if (ok && n < a.lq && a.part != nullptr) {
            // Key-split partial: O unnormalized, the row maximum in natural-log
            // units (P = 2^((s - m) c) = e^((s - m) scale)), the row sum.
            float* dst = a.part + ((int64_t(split) * gridDim.y + h) * a.lq + n) * (HD + 2);
#pragma unroll
            for (int c = 0; c < HD; ++c) dst[c] = o[c];
            dst[HD] = m == -INFINITY ? -INFINITY : m * (a.scale_log2e * 0.6931471805599453f);
            dst[HD + 1] = l;
        } else if (ok && n < a.lq) {
            int64_t orow = int64_t(g) * a.lq + n;
            if (a.out_window > 0) {
                const int per_row = a.out_grid_w / a.out_window;
                const int wy = g / per_row, wx = g % per_row, ly = n / a.out_window, lx = n % a.out_window;
                orow = int64_t(wy * a.out_window + ly) * a.out_grid_w + wx * a.out_window + lx;
            }
            float* dst = a.out + orow * a.ldo + h * HD;
#pragma unroll
            for (int c4 = 0; c4 < HD / 4; ++c4) {
                float4 r4;
                r4.x = l > 0.0f ? __fdiv_rn(o[4 * c4], l) : 0.0f;
                r4.y = l > 0.0f ? __fdiv_rn(o[4 * c4 + 1], l) : 0.0f;
                r4.z = l > 0.0f ? __fdiv_rn(o[4 * c4 + 2], l) : 0.0f;
                r4.w = l > 0.0f ? __fdiv_rn(o[4 * c4 + 3], l) : 0.0f;
                reinterpret_cast<float4*>(dst)[c4] = r4;
            }
        }
    }
    tc_fence_before();
    // Reconverge each warp before the aligned CTA barrier (lane-0 role loops).
    __syncwarp();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 512);
    }
}

}  // namespace

template <int HD, bool SPLIT>
void launch_tc(const TcArgs& a, int heads, int groups, const CUtensorMap& tm_k, const CUtensorMap& tm_vt,
               DeviceState& state, cudaStream_t stream) {
    using L = TcLayout<HD>;
    static_assert(L::total <= 232448, "shared memory budget");
    auto kernel = attention_tc_kernel<HD, SPLIT>;
    set_smem_limit_once(state, reinterpret_cast<const void*>(kernel), L::total,
                        "cudaFuncSetAttribute(attention_tc smem)");
    const dim3 grid((a.lq + kQ - 1) / kQ, heads, groups);
    launch_pdl(kernel, grid, dim3(kTcThreads), L::total, stream, "attention_tc_kernel launch", a, tm_k, tm_vt);
}

bool attention_tc_eligible(int lq, int lk, int head_dim, int causal, const float* bias, const float* out,
                           int64_t ldo) {
    return (head_dim == 32 || head_dim == 64) && !causal && bias == nullptr && lq >= 1024 && lk >= 256 &&
           ldo % 4 == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
}

size_t attention_tc_plane_bytes(int groups, int group_n, int heads, int head_dim) {
    return static_cast<size_t>(4) * groups * group_n * heads * head_dim * sizeof(float);
}

// Key splits of the one-group form: CTAs run one per SM, so a grid of a few
// waves loses its last wave's idle SMs.  s splits make waves of 1 / s of a
// CTA's keys (plus a fixed per-CTA start, ~3 % of a full CTA at the fusion
// shape); the smallest s within 2 % of the least critical path is taken, with
// at least 8 key tiles per split.
constexpr int kMaxKeySplits = 4;

static int tc_key_splits(int lq, int lk, int heads, int sms) {
    const int64_t ctas = int64_t((lq + kQ - 1) / kQ) * heads;
    const int tiles = (lk + kKeys - 1) / kKeys;
    double cost[kMaxKeySplits + 1] = {};
    double best = 1e30;
    for (int s = 1; s <= kMaxKeySplits; ++s) {
        if (s > 1 && tiles / s < 8) break;
        const int64_t waves = (ctas * s + sms - 1) / sms;
        cost[s] = static_cast<double>(waves) * (1.0 / s + 0.03);
        best = std::min(best, cost[s]);
    }
    for (int s = 1; s <= kMaxKeySplits; ++s)
        if (cost[s] > 0.0 && cost[s] <= best * 1.02) return s;
    return 1;
}

static size_t tc_partial_floats(int lq, int heads, int head_dim) {
    return static_cast<size_t>(kMaxKeySplits) * heads * lq * (head_dim + 2);
}

template <int HD>
static void launch_groups(TcArgs a, int heads, int groups, float* planes, float* part, DeviceState& state,
                   cudaStream_t stream) {
    const int lk = a.lk;
    int splits = 1;
    if (part != nullptr && groups == 1 && a.out_window == 0) splits = tc_key_splits(a.lq, lk, heads, state.sm_count);
    float* out = a.out;
    const int64_t ldo = a.ldo;
    int z = groups;
    if (splits > 1) {
        const int tiles = (lk + kKeys - 1) / kKeys;
        a.kps = (tiles + splits - 1) / splits * kKeys;
        splits = (tiles * kKeys + a.kps - 1) / a.kps;  // splits actually holding keys
        a.part = part;
        z = splits;
    }
    if (planes == nullptr || lk % 4 != 0 || (reinterpret_cast<uintptr_t>(planes) & 15u) != 0) {
        CUtensorMap none{};  // not read by the loader-fed kernel
        launch_tc<HD, false>(a, heads, z, none, none, state, stream);
    } else {
        // K / V^T split once into TF32 hi / lo planes, then loaded by TMA.
        const uint64_t gh2 = static_cast<uint64_t>(2) * groups * heads;
        float* kp = planes;
        float* vtp = planes + static_cast<int64_t>(2) * groups * heads * lk * HD;
        launch_pdl(split_kv_kernel<HD>, dim3((lk + 63) / 64, heads, groups), dim3(256), 0, stream,
                   "split_kv_kernel launch", a.k, a.ldk, a.v, a.ldv, lk, heads, groups, kp, vtp);
        CUtensorMap tm_k, tm_vt;
        encode_tensor_map_3d(&tm_k, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, kp, HD, lk, gh2, HD * 4,
                             static_cast<uint64_t>(lk) * HD * 4, 32, kKeys, CU_TENSOR_MAP_SWIZZLE_128B);
        encode_tensor_map_3d(&tm_vt, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, vtp, lk, HD, gh2, static_cast<uint64_t>(lk) * 4,
                             static_cast<uint64_t>(lk) * HD * 4, 32, HD, CU_TENSOR_MAP_SWIZZLE_128B);
        launch_tc<HD, true>(a, heads, z, tm_k, tm_vt, state, stream);
    }
    if (splits > 1) launch_attention_combine(part, splits, heads, a.lq, HD, out, ldo, stream);
}

void launch_attention_tc(const float* q, int64_t ldq, const float* k, int64_t ldk, const float* v, int64_t ldv,
                         int lq, int lk, int heads, int head_dim, float scale, float* out, int64_t ldo, float* scratch,
                         DeviceState& state, cudaStream_t stream) {
    TcArgs a{q, k, v, out, ldq, ldk, ldv, ldo, lq, lk, 0, 0, scale * 1.4426950408889634f, state.status};
    // scratch: the K / V^T planes, then the key-split partials (attention_tc_scratch_bytes).
    float* part = nullptr;
    if (scratch != nullptr)
        part = scratch + (attention_tc_plane_bytes(1, lk, heads, head_dim) + 255) / 256 * 64;  // 256-byte aligned
    if (head_dim == 64)
        launch_groups<64>(a, heads, 1, scratch, part, state, stream);
    else
        launch_groups<32>(a, heads, 1, scratch, part, state, stream);
}

size_t attention_tc_scratch_bytes(int lq, int lk, int heads, int head_dim) {
    return (attention_tc_plane_bytes(1, lk, heads, head_dim) + 255) / 256 * 256 +
           tc_partial_floats(lq, heads, head_dim) * sizeof(float);
}

void launch_attention_tc_groups(const float* qkv, int64_t ldq, int64_t embed, int groups, int group_n, int heads,
                                int head_dim, float scale, float* out, int64_t ldo, int out_window, int out_grid_w,
                                float* planes, DeviceState& state, cudaStream_t stream) {
    TcArgs a{qkv, qkv + embed, qkv + 2 * embed, out, ldq, ldq, ldq, ldo, group_n, group_n, out_window, out_grid_w,
             scale * 1.4426950408889634f, state.status};
    if (head_dim == 64)
        launch_groups<64>(a, heads, groups, planes, nullptr, state, stream);
    else
        launch_groups<32>(a, heads, groups, planes, nullptr, state, stream);
}

}  // namespace samq
