// Shared device helpers for the hq4 kernels (sm_100a only).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "hq4 kernels are written for sm_100a (B200) only"
#endif

namespace hq4 {

constexpr int kWarp = 32;

// ---- programmatic dependent launch -------------------------------------
// launch_dependents lets the next kernel in the stream be scheduled while this
// one drains; wait blocks until the previous kernel has completed and its
// writes are visible.  Both are no-ops when the launch carries no
// programmatic dependency.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---- global loads -------------------------------------------------------
// Streaming 256-bit load of packed weights: read once, do not keep in L1.
__device__ __forceinline__ void ldg256_stream(const uint32_t* p, uint32_t (&v)[8]) {
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]),
                   "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "l"(p));
}
__device__ __forceinline__ void ldg128_stream(const uint32_t* p, uint32_t (&v)[4]) {
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "l"(p));
}
// Scales/biases: 16-bit, re-used by neighbouring units through L1.
__device__ __forceinline__ uint32_t ldg_u16(const uint16_t* p) {
    unsigned short v;
    asm volatile("ld.global.nc.L1::evict_last.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}
// 8-byte read-only load (4 fp16 scales or biases), kept in L1 for the
// neighbouring rows' threads.
__device__ __forceinline__ uint2 ldg_u32x2(const uint16_t* p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
// 16-byte streaming load straight into four caller registers (a prefetch
// target must be the asm output itself: any select or copy of the result
// would wait for the load where it is issued).
__device__ __forceinline__ void ldg128_into(const uint32_t* p, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "l"(p));
}
// Four consecutive fp16 values (8-byte aligned) into four 16-bit registers.
__device__ __forceinline__ void ldg_u16x4_into(const uint16_t* p, unsigned short& a, unsigned short& b,
                                               unsigned short& c, unsigned short& d) {
    asm volatile("ld.global.nc.v4.u16 {%0,%1,%2,%3}, [%4];" : "=h"(a), "=h"(b), "=h"(c), "=h"(d) : "l"(p));
}
__device__ __forceinline__ void ldg_u16_into(const uint16_t* p, unsigned short& a) {
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(a) : "l"(p));
}
// Coherent (L1-bypassing) load for values written by other CTAs this launch.
__device__ __forceinline__ float ldcg_f32(const float* p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}

// ---- int4 -> fp16 exact dequantisation ---------------------------------
// d = (a & b) | c
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// From one packed word w (nibbles q0..q7, low first) produce the half2 pairs
//   lo = {q0, q4}   hi = {q1, q5}
// exactly: OR-ing a nibble into the mantissa of 1024.0h gives 1024+q, and a
// nibble at bits 4..7 gives 1024+16q, which *1/16 - 64 maps back to q.
__device__ __forceinline__ void dq_pair(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t kMagic = 0x64006400u;      // {1024, 1024}
    const uint32_t kSixteenth = 0x2C002C00u;  // {1/16, 1/16}
    const uint32_t kNeg64 = 0xD400D400u;      // {-64, -64}
    lo = h2_sub(lop3_and_or(w, 0x000F000Fu, kMagic), kMagic);
    hi = h2_fma(lop3_and_or(w, 0x00F000F0u, kMagic), kSixteenth, kNeg64);
}

// ---- int4 -> u8 unpack ----------------------------------------------------
// One packed word w (nibbles q0..q7, low first) -> two u8x4 registers
//   even = {q0, q2, q4, q6}   odd = {q1, q3, q5, q7}
__device__ __forceinline__ void unpack_u8(uint32_t w, uint32_t& even, uint32_t& odd) {
    even = w & 0x0F0F0F0Fu;
    odd = (w >> 4) & 0x0F0F0F0Fu;
}

// ---- tensor core --------------------------------------------------------
// D(16x8,s32) += A(16x32,u8,row) * B(32x8,s8,col): exact integer products/sums
__device__ __forceinline__ void mma_u8s8_16832(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D(16x8,s32) = A(16x32,u8,row) * B(32x8,s8,col): the first MMA of a chain
// (no accumulator to clear)
__device__ __forceinline__ void mma_u8s8_16832_first(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                     uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
// D(16x8,f32) += A(16x16,f16,row) * B(16x8,f16,col)
__device__ __forceinline__ void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D(16x8,f32) = A(16x16,bf16,row) * B(16x8,bf16,col) + C
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)bits16));
}

// ---- x as a per-group fixed-point integer ------------------------------
// Exponent E with amax < 2^E (E = floor(log2 amax) + 1 for normal amax), so
// that v = rint(x * 2^(22-E)) satisfies |v| <= 2^22.  Clamped so both
// 2^(22-E) and 2^(E-22) are normal fp32; groups below 2^-100 round to zero.
constexpr int kXBits = 22;
__device__ __forceinline__ int group_exponent(float amax) {
    if (!(amax > 0.0f)) return 0;
    int e = (int)((__float_as_uint(amax) >> 23) & 0xFF) - 126;
    if (e < -100) e = -100;
    if (e > 127) e = 127;
    return e;
}

// The three balanced base-256 digits of v = rint(x * up), |v| <= 2^22, as the
// low three bytes of one word: v = d2*2^16 + d1*2^8 + d0 with d0, d1 in
// [-128, 127] and d2 in [-64, 64], each byte the digit's two's complement.
// fma(x, up, 1.5*2^23) rounds x*up to the nearest integer (ties to even) and
// leaves it in the low mantissa bits: bits = 0x4B400000 + v (at v = 2^22 the
// mantissa carry lands in the exponent and the identity still holds).  Adding
// 0x808080 makes every byte the biased digit d+128; xor 0x808080 unbiases.
__device__ __forceinline__ uint32_t digits3(float x, float up) {
    const float f = fmaf(x, up, 12582912.0f);
    return (__float_as_uint(f) + (0x808080u - 0x4B400000u)) ^ 0x808080u;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// ---- thread-block cluster / mbarrier / bulk copy (sm_90+) ----------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}
// fp32 load from a cluster peer's shared memory (address from map_to_rank).
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Initialise without the fence; the caller issues mbar_init_fence() once
// after the last of several initialisations.
__device__ __forceinline__ void mbar_init_nofence(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
// Bounded wait for phase `parity` of an mbarrier; false if the bound ran out.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int max_iters) {
    for (int i = 0; i < max_iters; i++) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done) : "r"(bar), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}
// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (bulk copies) issued afterwards.
// Wait for phase `parity` of an mbarrier for at most `limit_ns` of wall
// time (%globaltimer); false if the limit ran out.  Bounds the wait however
// long each try_wait suspends.
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done) : "r"(bar), "r"(parity) : "memory");
    return done != 0;
}
// Wall-clock-bounded wait.  The timer is read only once the barrier has
// been found incomplete (reading %globaltimer is slow), and each further
// try_wait may suspend the thread in hardware (up to ~1 ms) until the phase
// completes.
__device__ __forceinline__ bool mbar_wait_ns(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done) : "r"(bar), "r"(parity), "r"(1000000u) : "memory");
        if (done) return true;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}
// Bounded wait without the timer (for hot loops): try_wait with a suspend-
// time hint of hint_ns, at most `tries` times; false if none succeeded.
__device__ __forceinline__ bool mbar_wait_tries(uint32_t bar, uint32_t parity, uint32_t hint_ns, int tries) {
    for (int i = 0; i < tries; i++) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done) : "r"(bar), "r"(parity), "r"(hint_ns) : "memory");
        if (done) return true;
    }
    return false;
}
// Tight poll for the thread on the critical path (the MMA issuer): plain
// try_wait, the timer read once every 1024 polls.
__device__ __forceinline__ bool mbar_wait_spin(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t n = 1;; n++) {
        if (mbar_try(bar, parity)) return true;
        if ((n & 1023) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
    }
}
// The same wait for helper threads that are usually far ahead (loaders, the
// MMA issuer): poll, then sleep `nap_ns` between polls so the waiting warp
// leaves the issue slots to the warps sharing its scheduler.
__device__ __forceinline__ bool mbar_wait_nap(uint32_t bar, uint32_t parity, uint64_t limit_ns, uint32_t nap_ns) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        __nanosleep(nap_ns);
        if (mbar_try(bar, parity)) return true;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// 2D tensor copy global -> this CTA's shared memory (no multicast), completing
// on the mbarrier `bar`; (x, y) is the box origin in elements.  x times the
// element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tm, int x, int y, uint32_t bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(bar), "l"(policy)
        : "memory");
}
// 3D tensor copy, as tma_load_2d with box origin (x, y, z).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* tm, int x, int y, int z, uint32_t bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy)
        : "memory");
}
// Bring a 2D box of a tensor map into L2 ahead of its copy (a hint: no
// shared memory, no completion to wait for).  x as in tma_load_2d.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* tm, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(tm)),
                 "r"(x), "r"(y)
                 : "memory");
}
// Fetch a tensor map's descriptor ahead of its first use.
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* tm) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Copy `bytes` from this CTA's shared memory to a peer CTA's shared memory
// (both 16-byte aligned, bytes % 16 == 0), signalling the peer's mbarrier.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                                  uint32_t peer_bar_cluster) {
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst_cluster), "r"(src_cta), "r"(bytes), "r"(peer_bar_cluster) : "memory");
}
// L2 policy for data many CTAs re-read (the activation row).
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// L2 policy for data read exactly once (the packed weights).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// Bulk copy global -> this CTA's shared memory (16-byte aligned, bytes % 16
// == 0), completing on the mbarrier `bar` (a shared::cta address).
__device__ __forceinline__ void bulk_load_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(policy) : "memory");
}
__device__ __forceinline__ void bulk_commit_and_wait_read() {
    asm volatile("cp.async.bulk.commit_group;\n cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ float exp2i(int e) {  // 2^e for |e| <= 126
    return __uint_as_float((uint32_t)(e + 127) << 23);
}

}  // namespace hq4
