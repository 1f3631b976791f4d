// samq_device.cuh -- sm_100a device primitives used by the samq kernels:
// mbarriers with bounded waits, TMA tensor copies (no cluster multicast),
// tcgen05 tensor-memory allocation / MMA / loads, and the device status word.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace samq {

// Device status word layout (one uint32 array per device, see DeviceStatus).
enum : uint32_t {
    kStatusRange = 1u,    // activation block non-finite or beyond the f16 operand range
    kStatusTimeout = 2u,  // a bounded mbarrier wait gave up
    kStatusLayout = 4u,   // dynamic shared memory base too poorly aligned for the kernel's layout
};

// Round to TF32 (10 stored mantissa bits), nearest, ties away from zero.
__device__ __forceinline__ float rna_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// The F32-semantics GEMM operand split: hi = rna_tf32(x), lo = rna_tf32(x - hi)
// (x - hi is exact in f32).
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
    hi = rna_tf32(x);
    lo = rna_tf32(x - hi);
}

struct DeviceStatus {
    uint32_t flags;       // OR of kStatus*
    uint32_t timeout_site;
    uint32_t range_blocks;
    uint32_t pad;
};

// A wait that has not completed after this many nanoseconds of %globaltimer is
// abandoned: the kernel records kStatusTimeout, skips its remaining work and
// returns, so a broken pipeline can never hang the GPU.
constexpr uint64_t kWaitTimeoutNs = 1000000000ull;
// Each mbarrier test suspends the thread at most this long (ns) before it
// re-checks, so the timeout above is observed within a few microseconds.
constexpr uint32_t kSuspendHintNs = 1000u;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return done != 0;
}

// One probe of the phase that returns at once (no suspend hint).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded polling wait (test_wait, %globaltimer checked every 64 probes): for
// short pipeline hand-offs where a suspended thread's wake-up would cost more
// than the step it waits for.
__device__ __forceinline__ bool mbar_poll(uint64_t* bar, uint32_t parity, DeviceStatus* status, uint32_t site) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t start = global_timer_ns();
    for (uint32_t spin = 1;; ++spin) {
        if (mbar_test_wait(bar, parity)) return true;
        if ((spin & 63u) == 0 && global_timer_ns() - start > kWaitTimeoutNs) {
            if (status) {
                atomicOr(&status->flags, kStatusTimeout);
                atomicExch(&status->timeout_site, site);
            }
            return false;
        }
    }
}

// Bounded wait for the phase with parity `parity`.  Returns false (and records
// the site) when the wait is abandoned.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, DeviceStatus* status, uint32_t site) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_timer_ns();
    for (uint32_t spin = 1;; ++spin) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((spin & 15u) == 0 && global_timer_ns() - start > kWaitTimeoutNs) {
            if (status) {
                atomicOr(&status->flags, kStatusTimeout);
                atomicExch(&status->timeout_site, site);
            }
            return false;
        }
    }
}

// ---- Q8_1 activation operand ---------------------------------------------
// The staging rule of GGML CUDA's quantize_q8_1 as pinned by SAM.cpp's
// verifiers (tools/validation/verify_q8_rhs_staging.py:24-83) and scale patch
// (cmake/patches/ggml-precise-cuda.patch:623-633), restated per 32-value block:
//   amax = max |x|, d = amax / 127 (IEEE), q = round_half_away(x * (127/amax)),
// and the tensor-core A operand is f16(f32(f16(d)) * q).  Shared by K1 and by
// the fused producers (LayerNorm, GEMM and attention epilogues) so that every
// path stages bit-identically from the same f32 values.

// |x| above this could overflow the f16 operand (65504) after rounding.
constexpr float kOperandLimit = 65000.0f;

// roundf() for |y| < 2^22 without float/int conversions: round half away
// from zero is trunc(|y| + 0.5) with the sign of y; the sum is taken rounding
// toward zero (so 0.49999997 + 0.5 stays below 1) and the truncation is the
// exact round-toward-zero add/subtract of 2^23.  Adding +0 at the end turns a
// negative zero into +0, as the integer code it stands for has no sign.
__device__ __forceinline__ float round_half_away(float y) {
    const float t = __fadd_rz(fabsf(y), 0.5f);
    const float whole = __fsub_rz(__fadd_rz(t, 8388608.0f), 8388608.0f);
    return __fadd_rn(copysignf(whole, y), 0.0f);
}

// Stages V consecutive values of one thread whose 32-value block is spread
// over LANES aligned neighbouring lanes (V * LANES == 32; every lane of the
// warp must call it).  out[j] holds the f16 operand pair of v[2j], v[2j+1].
// Returns true when a value is non-finite or beyond kOperandLimit.
template <int LANES, int V>
__device__ __forceinline__ bool stage_q8_1(const float (&v)[V], uint32_t (&out)[V / 2]) {
    static_assert(LANES * V == 32, "one Q8_1 block is 32 values");
    float amax = 0.0f;
    bool bad = false;
#pragma unroll
    for (int j = 0; j < V; ++j) {
        amax = fmaxf(amax, fabsf(v[j]));
        bad |= !(fabsf(v[j]) <= kOperandLimit);
    }
#pragma unroll
    for (int o = 1; o < LANES; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float dq = __half2float(__float2half_rn(__fdiv_rn(amax, 127.0f)));
    const float inv = amax == 0.0f ? 0.0f : __fdiv_rn(127.0f, amax);
#pragma unroll
    for (int j = 0; j < V / 2; ++j) {
        const float q0 = round_half_away(__fmul_rn(v[2 * j], inv));
        const float q1 = round_half_away(__fmul_rn(v[2 * j + 1], inv));
        const __half2 h = __floats2half2_rn(__fmul_rn(dq, q0), __fmul_rn(dq, q1));
        out[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return bad;
}

// Records a range failure once per warp (every lane must call it).
__device__ __forceinline__ void record_range(bool bad, DeviceStatus* status) {
    const unsigned any = __ballot_sync(0xffffffffu, bad);
    if (any && (threadIdx.x & 31) == __ffs(any) - 1 && status) {
        atomicOr(&status->flags, kStatusRange);
        atomicAdd(&status->range_blocks, 1u);
    }
}

// erf-GELU, 0.5 x (1 + erf(x / sqrt 2)), from Abramowitz & Stegun 7.1.26:
// for z >= 0, erf(z) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) e^(-z^2)
// with t = 1 / (1 + p z), |error| <= 1.5e-7.  With q = (1 - erf(|x|/sqrt 2)) / 2,
// GELU(x) = x (1 - q) for x >= 0 and x q for x < 0.  The reciprocal and the
// exponential go to the MUFU pipe (rcp.approx, ex2.approx: relative errors
// ~2^-22), the rest is 11 FMA-pipe operations: about half the issue cost of
// a polynomial erf of the same accuracy, in the epilogue that bounds fc1.
__device__ __forceinline__ float rcp_mufu(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float ex2_mufu(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float gelu_erf(float x) {
    // a_i / 2 (the 1/2 of q folded in), p, 1/sqrt(2), -log2(e)/2.
    constexpr float b1 = 0.127414796f, b2 = -0.142248368f, b3 = 0.7107068705f, b4 = -0.7265760135f,
                    b5 = 0.5307027145f, p = 0.3275911f;
    const float z = fabsf(x) * 0.70710678118654752f;
    const float t = rcp_mufu(fmaf(p, z, 1.0f));
    float poly = fmaf(b5, t, b4);
    poly = fmaf(poly, t, b3);
    poly = fmaf(poly, t, b2);
    poly = fmaf(poly, t, b1);
    poly *= t;
    const float q = poly * ex2_mufu((x * x) * -0.72134752044448170f);
    return x * (x >= 0.0f ? 1.0f - q : q);
}

// ---- programmatic dependent launch ---------------------------------------
// Kernels launched with cudaLaunchAttributeProgrammaticStreamSerialization may
// start before the previous kernel on the stream has finished; each of them
// calls pdl_wait() before touching memory the predecessor may write or read,
// and pdl_trigger() once its own dependents may be scheduled.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- TMA tensor copies (cp.async.bulk.tensor); plain loads, no multicast --

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
            "r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// 1-D bulk copy global -> shared of `bytes` (multiple of 16, both addresses
// 16-byte aligned), completing on `bar` (expect_tx must cover it).  No multicast.
__device__ __forceinline__ void bulk_load_1d(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y, int32_t z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
            "r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(smem_src)), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Generic-proxy writes to shared memory become visible to the async proxy
// (TMA store, tcgen05.mma operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tcgen05 ------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f16 (f16 or bf16 inputs).
__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns: register i of lane l holds
// column (col + i) of TMEM lane (lane_base + l).
__device__ __forceinline__ void tc_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Store 32 consecutive 32-bit columns of this warp's 32 TMEM lanes (inverse of
// tc_ld_32x32b_x32).
__device__ __forceinline__ void tc_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
        "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
        "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t desc = 0;
    desc |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);      // start address
    desc |= static_cast<uint64_t>(1u) << 16;                       // leading byte offset (unused for SW128 K-major)
    desc |= static_cast<uint64_t>(1024u >> 4) << 32;               // stride byte offset: 8 rows x 128 B
    desc |= static_cast<uint64_t>(1u) << 46;                       // descriptor version (sm_100)
    desc |= static_cast<uint64_t>(2u) << 61;                       // SWIZZLE_128B
    return desc;
}

// Instruction descriptor: kind::f16, A/B f16, D f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
    return (1u << 4)                                   // D format f32
           | (0u << 7) | (0u << 10)                    // A, B f16
           | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
           | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

// ---- CTA pairs (cluster of 2, tcgen05 cta_group::2) ----------------------
// Two CTAs on the two SMs of a TPC share one M = 256 tile: each holds 128 rows
// of A and half of B's rows in its own shared memory, and its own 128 rows of
// the accumulator in TMEM.  Every TMA load below is a plain load into the
// issuing CTA's own shared memory (no multicast); only its completion may be
// signalled on the other CTA's mbarrier.

__device__ __forceinline__ uint32_t cluster_cta_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// shared::cluster address of the variable at `local` in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(const void* local, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(local)), "r"(rank));
    return out;
}

// Cluster-wide barrier (aligned: every warp executes it converged).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive (count 1) on an mbarrier given by its shared::cluster address.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// mbar_try_wait with cluster-scope acquire: for barriers that threads of the
// other CTA of the pair arrive on.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return done != 0;
}

// Bounded wait (as mbar_wait) with cluster-scope acquire.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, DeviceStatus* status,
                                                  uint32_t site) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t start = global_timer_ns();
    for (uint32_t spin = 1;; ++spin) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((spin & 15u) == 0 && global_timer_ns() - start > kWaitTimeoutNs) {
            if (status) {
                atomicOr(&status->flags, kStatusTimeout);
                atomicExch(&status->timeout_site, site);
            }
            return false;
        }
    }
}

// 2-D tile load into this CTA's shared memory whose completion is signalled on
// an mbarrier of either CTA of the pair (cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster_addr,
                                                 int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
            "r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Pair MMA issued by one thread of the even CTA: A rows and B rows are split
// across the two CTAs' shared memory at the same offsets, D is each CTA's TMEM.
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on the mbarrier at `bar_cluster_addr` (either CTA of the pair) once
// every pair MMA issued so far by this thread is complete.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster_addr) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar_cluster_addr)
                 : "memory");
}

}  // namespace samq
