// W4A16 GEMM on the fifth-generation tensor cores (tcgen05 + TMEM):
// out[t][n] = sum_k x[t][k] * (q[n][k] * scale[n][g] + bias[n][g]),
// for token counts where the product is a real dense contraction (microbatched
// decode, prefill).  The reference computes the same product in
// QLinear._gemm (hetero/cpu_model.py:118-136) as fp32 dequantisation of
// 512-row blocks (kernel/q4gemv.c:311-379) followed by a BLAS matmul.
//
// Two launches per call:
//
//  1. xprep: the activations (bf16 or fp32) become fp16 in a caller-owned
//     workspace laid out as the exact shared-memory image of the B operand --
//     per (token tile, 64-wide k-block) one contiguous [T][64] fp16 block,
//     K-major with the 128-byte swizzle.  A B stage is then one bulk copy.
//  2. the GEMM.  One CTA owns 128 weight rows (the MMA's M) x T <= 256 tokens
//     (its N) x a contiguous range of k-blocks:
//       warps 0-7  dequantise: two threads per weight row, each turning 16
//                  packed bytes of a k-block into 32 fp16 values (q as fp16
//                  through the 0x6400 exponent trick, then one fma with the
//                  group's scale and bias: a single rounding of q*s+b),
//                  written K-major with the 128-byte swizzle; packed words are
//                  prefetched in registers 4 k-blocks at a time, kSbPre
//                  such groups ahead.  After the
//                  mainloop the same warps read the fp32 accumulator out of
//                  TMEM (warp w owns lanes 32(w%4)..+31).
//       warp 8     one thread streams the workspace blocks into the B stages
//                  (cp.async.bulk, completing on the stage's mbarrier).
//       warp 9     allocates TMEM and, from one thread, issues
//                  tcgen05.mma.cta_group::1.kind::f16 (K=16 per instruction)
//                  once a stage is full, releasing it through tcgen05.commit.
//
// Inside a 64-wide k-block the k order is permuted identically for weights
// and activations (word j of a row holds k = 8j..8j+7; its values are stored
// as k 8j+{0,4,1,5,2,6,3,7}), which is what the nibble-to-fp16 trick
// produces directly; a dot product does not depend on the order.
//
// Splitting K over a thread-block cluster (grid y) fills the SMs when there
// are few row tiles (the 3584-row down projection has 28): every CTA of the
// cluster stores its fp32 partial tile in its own shared memory, and after a
// cluster barrier CTA j sums token slice j over the cluster ranks in rank
// order (distributed shared memory loads).  Deterministic, no atomics.
//
// Precision: weights are rounded once to fp16 (relative error <= 2^-11),
// activations are converted to fp16 (exact for bf16 x with |x| < 65520;
// larger magnitudes set status bit 2), products and sums are fp32.  Relative
// L2 error vs the reference's fp32 path is ~3e-4 (acceptance bar 1e-3).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "hq4_common.cuh"
#include "hq4.h"

namespace hq4 {

int check_device_cap();
int* status_word();

constexpr int kGemmRows = 128;                          // MMA M
constexpr int kAWarps = 8;                              // dequant + epilogue
constexpr int kLoadWarp = kAWarps;                      // warp 8: B-stage bulk copies
constexpr int kMmaWarp = kAWarps + 1;                   // warp 9: TMEM + MMA issue
constexpr int kGemmThreads = (kAWarps + 2) * 32;
constexpr int kAStageBytes = kGemmRows * 128;           // 128 rows x 64 fp16
constexpr int kSbPre = 3;                               // super-blocks (4 k-blocks) in flight per thread
constexpr uint64_t kGemmWaitNs = 1000000000ull;         // 1 s: a correct kernel never waits this long
constexpr int kMaxTile = 256;
constexpr int kGemmSmemMax = 220 * 1024;
constexpr int kPrepThreads = 256;

struct GemmParams {
    const uint32_t* w;
    const uint16_t* sc;
    const uint16_t* bi;
    const unsigned char* xw;   // prepared activations (workspace)
    float* out;
    const float* row_add;
    const float* residual;
    int n_out, n_in, m;
    int n_sg;       // groups per row
    int gs_shift;   // log2(gs / 64)
    int nkb;        // k-blocks per row (n_in / 64)
    int ks;         // CTAs of a cluster along K
    int t_tile;     // tokens per CTA (multiple of 16)
    int stages;
    uint32_t tmem_cols;
    int* status;
};

// ---- tcgen05 / TMEM wrappers --------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T, fp16 operands, fp32 accumulator.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
        : "memory");
}
// Arrive once on an mbarrier when every tcgen05.mma issued so far has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, rows of 128 B
// in 8-row atoms of 1024 B (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    const uint32_t lo = ((smem_addr & 0x3FFFFu) >> 4) | (1u << 16);
    const uint32_t hi = (1024u >> 4) | (1u << 14) | (2u << 29);
    return ((uint64_t)hi << 32) | lo;
}
// Byte offset of 16-byte chunk c of row r in a K-major 128B-swizzled tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
    return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// 8 nibbles of w -> fp16 q*s+b in the order n0,n4,n1,n5,n2,n6,n3,n7.
// A nibble in bits 0-3 of a 16-bit half OR-ed into 0x6400 (1024.0) reads as
// 1024 + q; in bits 4-7 OR-ed into 0x5400 (64.0, whose mantissa LSB is 1/16)
// as 64 + q.  Subtracting the magic is exact, and one fma then rounds q*s+b
// once.  One shift per word (for nibbles 2, 3, 6, 7).
__device__ __forceinline__ uint4 dequant_word(uint32_t w, __half2 s2, __half2 b2) {
    const __half2 k1024 = bits_h2(0x64006400u), k64 = bits_h2(0x54005400u);
    const uint32_t w8 = w >> 8;
    const uint32_t p0 = lop3_and_or(w, 0x000F000Fu, 0x64006400u);   // n0, n4
    const uint32_t p1 = lop3_and_or(w, 0x00F000F0u, 0x54005400u);   // n1, n5
    const uint32_t p2 = lop3_and_or(w8, 0x000F000Fu, 0x64006400u);  // n2, n6
    const uint32_t p3 = lop3_and_or(w8, 0x00F000F0u, 0x54005400u);  // n3, n7
    uint4 o;
    o.x = h2_bits(__hfma2(__hsub2(bits_h2(p0), k1024), s2, b2));
    o.y = h2_bits(__hfma2(__hsub2(bits_h2(p1), k64), s2, b2));
    o.z = h2_bits(__hfma2(__hsub2(bits_h2(p2), k1024), s2, b2));
    o.w = h2_bits(__hfma2(__hsub2(bits_h2(p3), k64), s2, b2));
    return o;
}

// ---- activation preparation ---------------------------------------------------
// One thread per (token, 8-value word): x[t][8j..8j+7] -> fp16 in the order
// x0,x4,x1,x5,x2,x6,x3,x7, stored in block (t / T, j / 8) of the workspace at
// row t % T, chunk j % 8 (128-byte swizzle).  Tokens past m are zeros.
template <bool XF32>
__global__ void __launch_bounds__(kPrepThreads) gemm_xprep_kernel(const void* __restrict__ x,
                                                                unsigned char* __restrict__ ws, int m, int m_pad,
                                                                int n_in, int t_tile, int* status) {
    pdl_launch_dependents();
    pdl_wait();  // x comes from the previous kernel; the workspace may still be read by the previous GEMM
    const int wpr = n_in >> 3, nkb = n_in >> 6;
    const long long total = (long long)m_pad * wpr;
    float amax = 0.0f;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / wpr), j = (int)(i - (long long)t * wpr);
        float f[8];
        if (t < m) {
            if constexpr (XF32) {
                const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) +
                                                                  (size_t)t * n_in + (size_t)j * 8);
                const float4 a = __ldg(p), b = __ldg(p + 1);
                f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
                f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
            } else {
                const uint4 a = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) +
                                                                     (size_t)t * n_in + (size_t)j * 8));
                const uint32_t v[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int u = 0; u < 4; u++) {  // bf16 pair -> two fp32 (exact)
                    f[2 * u] = __uint_as_float(v[u] << 16);
                    f[2 * u + 1] = __uint_as_float(v[u] & 0xFFFF0000u);
                }
            }
        } else {
#pragma unroll
            for (int u = 0; u < 8; u++) f[u] = 0.0f;
        }
        uint32_t o[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            amax = fmaxf(amax, fmaxf(fabsf(f[u]), fabsf(f[u + 4])));
            o[u] = h2_bits(__floats2half2_rn(f[u], f[u + 4]));  // low half = f[u]
        }
        const int tt = t / t_tile, tin = t - tt * t_tile, kb = j >> 3, c = j & 7;
        const size_t blk = ((size_t)tt * nkb + kb) * (size_t)(t_tile * 128);
        *reinterpret_cast<uint4*>(ws + blk + sw128_off(tin, c)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    if (amax >= 65520.0f && status) atomicOr(status, 4);
}

// ---- the GEMM -------------------------------------------------------------------------
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_w4a16_kernel(const GemmParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // SW128 atoms need 1024-byte alignment
    unsigned char* sm = smem_raw + (base - raw);
    const int S = p.stages, T = p.t_tile;
    const int b_stage = T * 128;
    const uint32_t a_base = base, b_base = base + (uint32_t)(S * kAStageBytes);
    const uint32_t bar0 = b_base + (uint32_t)(S * b_stage);
    auto full_bar = [&](int s) { return bar0 + 8u * (uint32_t)s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (uint32_t)(S + s); };
    const uint32_t accum_bar = bar0 + 16u * (uint32_t)S;
    const uint32_t tmem_slot = accum_bar + 8u;
    volatile uint32_t* tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(sm + (tmem_slot - base));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * kGemmRows;
    const int kr = blockIdx.y;  // K-split rank (= cluster rank: the cluster spans grid y)
    const int tt = blockIdx.z, tok0 = tt * T;
    const int mt = min(T, p.m - tok0);
    const int kb0 = (int)((long long)kr * p.nkb / p.ks), kb1 = (int)((long long)(kr + 1) * p.nkb / p.ks);
    const int nk = kb1 - kb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(full_bar(s), kAWarps + 1);  // one arrive per dequant warp + the copy's expect_tx
            mbar_init(empty_bar(s), 1);
        }
        mbar_init(accum_bar, 1);
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, p.tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot_ptr;
    pdl_launch_dependents();

    bool fail = false;
    if (warp < kAWarps) {
        // ---- dequantise weights -------------------------------------------------------------
        // Every dequant thread takes part in every k-block, in order (each
        // waits for consecutive completions of each stage barrier, so none can
        // be satisfied by an older phase of the same parity).  Thread (r, h):
        // weight row r, words 4h..4h+3 of each k-block; warps 0-3 are h = 0,
        // warps 4-7 h = 1.  Packed words are fetched a super-block (4
        // k-blocks) at a time, so the two threads of a row request its 128
        // contiguous bytes together -- one burst per row, as DRAM wants.
        const int h = warp >> 2;
        const int r = (warp & 3) * 32 + lane;
        const int grow = row0 + r;
        const bool rok = grow < p.n_out;
        const size_t wpr = (size_t)(p.n_in >> 3);
        const uint32_t* wrow = p.w + (size_t)(rok ? grow : 0) * wpr + 4 * h;
        const uint16_t* srow = p.sc + (size_t)(rok ? grow : 0) * p.n_sg;
        const uint16_t* brow = p.bi + (size_t)(rok ? grow : 0) * p.n_sg;
        // gs = 64 with 8-byte aligned scale rows: 4 scales (biases) in one load
        const bool vec_sb = p.gs_shift == 0 && (p.n_sg & 3) == 0 && (kb0 & 3) == 0 &&
                            (((uintptr_t)p.sc | (uintptr_t)p.bi) & 7) == 0;
        const int nsb = (nk + 3) >> 2;  // super-blocks in this CTA's K range
        uint32_t q[kSbPre][16];
        unsigned short sv[kSbPre][4], bv[kSbPre][4];
        // Loads go straight into the ring registers, unconditionally: past
        // the end of the range (or for a row past n_out) the address is
        // clamped to valid data that is then not used.
        auto fetch = [&](int sb, uint32_t (&qq)[16], unsigned short (&ss)[4], unsigned short (&bb)[4]) {
            const int kbs = kb0 + 4 * min(sb, nsb - 1);  // first k-block of the super-block
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int kb = min(kbs + u, kb1 - 1);
                ldg128_into(wrow + (size_t)kb * 8, qq[4 * u], qq[4 * u + 1], qq[4 * u + 2], qq[4 * u + 3]);
            }
            if (vec_sb && kbs + 3 < kb1) {
                ldg_u16x4_into(srow + kbs, ss[0], ss[1], ss[2], ss[3]);
                ldg_u16x4_into(brow + kbs, bb[0], bb[1], bb[2], bb[3]);
            } else {
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int g = min(kbs + u, kb1 - 1) >> p.gs_shift;
                    ldg_u16_into(srow + g, ss[u]);
                    ldg_u16_into(brow + g, bb[u]);
                }
            }
        };
#pragma unroll
        for (int d = 0; d < kSbPre; d++) fetch(d, q[d], sv[d], bv[d]);
        for (int sbb = 0; sbb < nsb && !fail; sbb += kSbPre) {
#pragma unroll
            for (int d = 0; d < kSbPre; d++) {
                const int sb = sbb + d;
                if (sb < nsb && !fail) {
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int i = 4 * sb + u;  // local k-block
                        if (i < nk && !fail) {
                            const int s = i % S;
                            if (i >= S &&
                                !mbar_wait_ns(empty_bar(s), (uint32_t)((i / S) - 1) & 1u, kGemmWaitNs)) {
                                fail = true;
                            } else {
                                const __half2 s2 = __half2half2(__ushort_as_half(sv[d][u]));
                                const __half2 b2 = __half2half2(__ushort_as_half(bv[d][u]));
                                unsigned char* dst = sm + (a_base - base) + (size_t)s * kAStageBytes;
#pragma unroll
                                for (int c = 0; c < 4; c++) {
                                    const uint4 v = rok ? dequant_word(q[d][4 * u + c], s2, b2)
                                                        : make_uint4(0, 0, 0, 0);
                                    *reinterpret_cast<uint4*>(dst + sw128_off(r, 4 * h + c)) = v;
                                }
                                fence_proxy_async_smem();
                                __syncwarp();
                                if (lane == 0) mbar_arrive(full_bar(s));
                            }
                        }
                    }
                    fetch(sb + kSbPre, q[d], sv[d], bv[d]);
                }
            }
        }
    } else if (warp == kLoadWarp) {
        // ---- B stages: one bulk copy of a prepared block each ---------------------------
        if (lane == 0) {
            pdl_wait();  // the workspace is written by the preparation kernel
            const uint64_t pol = l2_policy_evict_last();
            const unsigned char* src = p.xw + ((size_t)tt * p.nkb + kb0) * (size_t)b_stage;
            for (int i = 0; i < nk; i++) {
                const int s = i % S;
                if (i >= S && !mbar_wait_ns(empty_bar(s), (uint32_t)((i / S) - 1) & 1u, kGemmWaitNs)) {
                    fail = true;
                    break;
                }
                mbar_arrive_expect_tx(full_bar(s), (uint32_t)b_stage);
                bulk_load_g2s(b_base + (uint32_t)(s * b_stage), src + (size_t)i * b_stage, (uint32_t)b_stage,
                              full_bar(s), pol);
            }
        }
    } else if (lane == 0) {
        // ---- MMA issue ------------------------------------------------------------------
        const uint32_t idesc = (1u << 4)                        // D fp32
                               | ((uint32_t)(T >> 3) << 17)     // N
                               | ((uint32_t)(kGemmRows >> 4) << 24);  // M
        for (int i = 0; i < nk; i++) {
            const int s = i % S;
            if (!mbar_wait_ns(full_bar(s), (uint32_t)(i / S) & 1u, kGemmWaitNs)) {
                fail = true;
                break;
            }
            tc_fence_after();
            const uint64_t ad = sw128_desc(a_base + (uint32_t)(s * kAStageBytes));
            const uint64_t bd = sw128_desc(b_base + (uint32_t)(s * b_stage));
#pragma unroll
            for (int kk = 0; kk < 4; kk++)  // 16 k per instruction: +32 bytes = +2 descriptor units
                umma_f16(tmem, ad + 2u * kk, bd + 2u * kk, idesc, (i | kk) != 0);
            umma_commit(empty_bar(s));
        }
        umma_commit(accum_bar);
    }
    if (fail && p.status) atomicOr(p.status, 1);

    // ---- epilogue: TMEM -> out ---------------------------------------------------------
    // warp w reads TMEM lanes 32(w%4).. (its quadrant) for the 32-column chunks
    // with index = w/4 (mod 2)
    const bool epi = warp < kAWarps;
    const int er = (warp & 3) * 32 + lane;
    const int grow = row0 + er;
    float* part = reinterpret_cast<float*>(sm);  // split-K partial tile [T][128], reuses the rings
    if (epi) {
        pdl_wait();
        const bool ok = mbar_wait_ns(accum_bar, 0, kGemmWaitNs);
        if (!ok && p.status) atomicOr(p.status, 1);
        __syncwarp();  // tcgen05.ld is warp-aligned
        tc_fence_after();
        const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        for (int c0 = (warp >> 2) * 32; c0 < T; c0 += 64) {
            uint32_t v[32];
            tmem_ld32(trow + (uint32_t)c0, v);
            tmem_wait_ld();
            if (p.ks == 1) {
                if (ok && grow < p.n_out) {
                    const float add = p.row_add ? p.row_add[grow] : 0.0f;
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        const int t = c0 + j;
                        if (t < mt) {
                            const size_t o = (size_t)(tok0 + t) * p.n_out + grow;
                            float y = __uint_as_float(v[j]) + add;
                            if (p.residual) y += p.residual[o];
                            p.out[o] = y;
                        }
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++)
                    if (c0 + j < T) part[(c0 + j) * kGemmRows + er] = __uint_as_float(v[j]);
            }
        }
    }
    __syncwarp();  // the cluster barriers below are warp-aligned
    if (p.ks > 1) {
        // every thread of every CTA of the cluster takes both barriers
        cluster_sync();
        const int t_lo = (int)((long long)kr * mt / p.ks), t_hi = (int)((long long)(kr + 1) * mt / p.ks);
        const int n_el = (t_hi - t_lo) * kGemmRows;
        const uint32_t part_addr = base;
        for (int e = threadIdx.x; e < n_el; e += kGemmThreads) {
            const int t = t_lo + e / kGemmRows, rr = e % kGemmRows;
            const int gr = row0 + rr;
            const uint32_t off = (uint32_t)((t * kGemmRows + rr) * 4);
            float y = 0.0f;
            for (int j = 0; j < p.ks; j++) y += ld_cluster_f32(map_to_rank(part_addr + off, (uint32_t)j));
            if (gr < p.n_out) {
                const size_t o = (size_t)(tok0 + t) * p.n_out + gr;
                if (p.row_add) y += p.row_add[gr];
                if (p.residual) y += p.residual[o];
                p.out[o] = y;
            }
        }
        cluster_sync();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        __syncwarp();
        tmem_dealloc(tmem, p.tmem_cols);
    }
}

// ---- host side --------------------------------------------------------------------------
struct GemmPlan {
    int t_tile, n_tt, row_tiles, ks, stages;
    uint32_t tmem_cols;
    size_t smem;
    size_t ws_bytes;
};

static int sm_count_gemm() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

static size_t gemm_smem(int t_tile, int stages) {
    return 1024 + (size_t)stages * (kAStageBytes + t_tile * 128) + 16 * (size_t)stages + 16;
}

static GemmPlan plan_gemm(int n_out, int n_in, int m) {
    GemmPlan pl{};
    pl.n_tt = (m + kMaxTile - 1) / kMaxTile;
    const int per = (m + pl.n_tt - 1) / pl.n_tt;             // balance the token tiles
    pl.t_tile = std::min(kMaxTile, (per + 15) / 16 * 16);
    pl.row_tiles = (n_out + kGemmRows - 1) / kGemmRows;
    const int stage_bytes = kAStageBytes + pl.t_tile * 128;
    pl.stages = std::min(8, (int)((kGemmSmemMax - 1024 - 256) / stage_bytes));
    pl.smem = gemm_smem(pl.t_tile, pl.stages);
    uint32_t c = 32;
    while ((int)c < pl.t_tile) c <<= 1;
    pl.tmem_cols = c;
    const int sms = sm_count_gemm();
    const int ctas = pl.row_tiles * pl.n_tt;
    const int nkb = n_in / 64;
    int ks = 1;
    if (ctas < sms) ks = std::min({8, nkb, std::max(1, sms / ctas)});
    pl.ks = ks;
    pl.ws_bytes = (size_t)pl.n_tt * pl.t_tile * (size_t)n_in * 2;
    return pl;
}

static cudaLaunchAttribute pdl_attribute() {
    cudaLaunchAttribute a;
    a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a.val.programmaticStreamSerializationAllowed = 1;
    return a;
}

static int launch_gemm(const GemmParams& prm, const GemmPlan& pl, cudaStream_t st) {
    // the shared-memory opt-in is a per-device function attribute
    static bool attr_done[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HQ4_ERR_LAUNCH;
    if (!attr_done[dev]) {
        if (cudaFuncSetAttribute(gemm_w4a16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmSmemMax) !=
            cudaSuccess)
            return HQ4_ERR_LAUNCH;
        attr_done[dev] = true;
    }
    // split-K partial tile [t_tile][128] fp32 lives in the (drained) rings
    if ((size_t)pl.t_tile * kGemmRows * 4 > (size_t)pl.stages * (kAStageBytes + pl.t_tile * 128) ||
        pl.smem > (size_t)kGemmSmemMax)
        return HQ4_ERR_SHAPE;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na++] = pdl_attribute();
    if (pl.ks > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = (unsigned)pl.ks;
        attr[na].val.clusterDim.z = 1;
        na++;
    }
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)pl.row_tiles, (unsigned)pl.ks, (unsigned)pl.n_tt);
    lc.blockDim = dim3(kGemmThreads);
    lc.dynamicSmemBytes = pl.smem;
    lc.stream = st;
    lc.attrs = attr;
    lc.numAttrs = na;
    return cudaLaunchKernelEx(&lc, gemm_w4a16_kernel, prm) == cudaSuccess ? HQ4_OK : HQ4_ERR_LAUNCH;
}

static int launch_xprep(const void* x, bool xf32, unsigned char* ws, int m, const GemmPlan& pl, int n_in,
                        int* status, cudaStream_t st) {
    const int m_pad = pl.n_tt * pl.t_tile;
    const long long total = (long long)m_pad * (n_in >> 3);
    const int blocks = (int)std::min<long long>((total + kPrepThreads - 1) / kPrepThreads, 4L * sm_count_gemm());
    cudaLaunchAttribute attr[1] = {pdl_attribute()};
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)blocks);
    lc.blockDim = dim3(kPrepThreads);
    lc.stream = st;
    lc.attrs = attr;
    lc.numAttrs = 1;
    cudaError_t e = xf32 ? cudaLaunchKernelEx(&lc, gemm_xprep_kernel<true>, x, ws, m, m_pad, n_in, pl.t_tile, status)
                         : cudaLaunchKernelEx(&lc, gemm_xprep_kernel<false>, x, ws, m, m_pad, n_in, pl.t_tile, status);
    return e == cudaSuccess ? HQ4_OK : HQ4_ERR_LAUNCH;
}

}  // namespace hq4

using namespace hq4;

static bool gemm_shape_ok(int n_out, int n_in, int gs, int m) {
    return n_out > 0 && n_in > 0 && m > 0 && gs >= 64 && gs % 64 == 0 && (gs & (gs - 1)) == 0 && n_in % gs == 0;
}

extern "C" long long hq4_gemm_workspace_bytes(int n_out, int n_in, int m) {
    if (n_out <= 0 || n_in <= 0 || m <= 0 || n_in % 64) return HQ4_ERR_SHAPE;
    return (long long)plan_gemm(n_out, n_in, m).ws_bytes;
}

extern "C" int hq4_gemm_w4a16(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, const void* x,
                              int x_is_f32, float* out, int n_out, int n_in, int gs, int m,
                              const float* row_add, const float* residual, void* workspace,
                              long long workspace_bytes, void* stream) {
    if (int rc = check_device_cap()) return rc;
    if (!gemm_shape_ok(n_out, n_in, gs, m)) return HQ4_ERR_SHAPE;
    if (((uintptr_t)w & 31) || ((uintptr_t)x & 15) || ((uintptr_t)out & 3) || ((uintptr_t)scales & 1) ||
        ((uintptr_t)biases & 1) || ((uintptr_t)workspace & 127))
        return HQ4_ERR_ALIGN;
    const GemmPlan pl = plan_gemm(n_out, n_in, m);
    if (!workspace || workspace_bytes < (long long)pl.ws_bytes) return HQ4_ERR_SHAPE;
    int* status = status_word();
    if (!status) return HQ4_ERR_LAUNCH;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    if (int rc = launch_xprep(x, x_is_f32 != 0, ws, m, pl, n_in, status, st)) return rc;
    GemmParams prm{};
    prm.w = w;
    prm.sc = scales;
    prm.bi = biases;
    prm.xw = ws;
    prm.out = out;
    prm.row_add = row_add;
    prm.residual = residual;
    prm.n_out = n_out;
    prm.n_in = n_in;
    prm.m = m;
    prm.n_sg = n_in / gs;
    int sh = 0;
    while ((64 << sh) < gs) sh++;
    prm.gs_shift = sh;
    prm.nkb = n_in / 64;
    prm.ks = pl.ks;
    prm.t_tile = pl.t_tile;
    prm.stages = pl.stages;
    prm.tmem_cols = pl.tmem_cols;
    prm.status = status;
    return launch_gemm(prm, pl, st);
}

extern "C" int hq4_gemm_plan(int n_out, int n_in, int m, int x_is_f32, int* info) {
    (void)x_is_f32;
    if (n_out <= 0 || n_in <= 0 || m <= 0 || n_in % 64 || !info) return HQ4_ERR_SHAPE;
    const GemmPlan pl = plan_gemm(n_out, n_in, m);
    info[0] = pl.row_tiles;
    info[1] = pl.ks;
    info[2] = pl.n_tt;
    info[3] = pl.t_tile;
    info[4] = pl.stages;
    info[5] = (int)pl.smem;
    info[6] = (int)pl.tmem_cols;
    info[7] = kGemmThreads;
    return HQ4_OK;
}
