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
//     (its N) x a contiguous range of k-blocks, in super-blocks of 4 k-blocks:
//       warp 8     streams each super-block's packed weights (128 rows x 128
//                  bytes, 128-byte swizzle) and its scale and bias tiles into
//                  a ring in shared memory with 2D TMA (cp.async.bulk.tensor);
//       warp 9     streams the prepared activation blocks into the B stages
//                  (cp.async.bulk);
//       warps 0-7  dequantise: two threads per weight row, each turning 16
//                  packed bytes of a k-block (read from the ring) into 32
//                  fp16 values (q as fp16 through exponent tricks, then one
//                  fma with the group's scale and bias: a single rounding of
//                  q*s+b), stored straight into the A operand in TMEM
//                  (tcgen05.st); no global loads, no shared-memory round trip
//                  for A.  After the mainloop the same warps read the fp32
//                  accumulator out of TMEM (warp w owns lanes 32(w%4)..+31);
//       warp 10    allocates TMEM and, from one thread, issues
//                  tcgen05.mma.cta_group::1.kind::f16 with A in TMEM and B in
//                  shared memory (K=16 per instruction) once a stage is full,
//                  releasing it through tcgen05.commit.
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

#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "hq4_common.cuh"
#include "hq4_gemv_dev.cuh"
#include "hq4_host.cuh"
#include "hq4_mt.cuh"
#include "hq4_tmap.cuh"
#include "hq4.h"

namespace hq4 {

int check_device_cap();
int* status_word();
int gemv_stream_m1(const uint32_t* w, const uint16_t* sc, const uint16_t* bi, const void* x, bool x_bf16,
                   float* out, int n_out, int n_in, int gs, const float* row_add, const float* residual,
                   cudaStream_t st, bool* used);
bool gemv_stream_fits_gs64(int n_out, int n_in);

constexpr int kGemmRows = 128;                          // MMA M
constexpr int kAWarps = 8;                              // dequant + epilogue
constexpr int kLoadWarp = kAWarps;                      // warp 8: all TMA / bulk copies, in order
constexpr int kMmaWarp = kAWarps + 1;                   // warp 9: TMEM + MMA issue
constexpr int kGemmThreads = (kAWarps + 2) * 32;
constexpr int kWTileBytes = kGemmRows * 128;            // packed super-block: 128 rows x 4 k-blocks
constexpr int kSTileBytes = kGemmRows * 16;             // 8 groups of fp16 scales per row
constexpr int kWSlotBytes = kWTileBytes + 2 * kSTileBytes;
constexpr int kTmemCols = 512;
constexpr uint64_t kGemmWaitNs = 1000000000ull;         // 1 s: a correct kernel never waits this long
constexpr int kMaxTile = 256;
constexpr int kGemmSmemMax = 220 * 1024;
constexpr int kPrepThreads = 256;

struct GemmParams {
    const unsigned char* xw;   // prepared activations (workspace)
    float* out;
    const float* row_add;
    const float* residual;
    int n_out, n_in, m;
    int gs_shift;   // log2(gs / 64)
    int nkb;        // k-blocks per row (n_in / 64)
    int ks;         // CTAs of a cluster along K
    int t_tile;     // tokens per CTA (multiple of 16)
    int stages;     // B (shared memory) k-block stages
    int astages;    // A (TMEM) super-block stages, 128 columns each
    int nacc;       // independent TMEM accumulators the MMAs rotate over
    int acc_stride; // TMEM columns per accumulator (t_tile rounded up to 32)
    int wslots;     // packed super-block slots
    int sb_tma;     // scales/biases by TMA (else the dequant threads load them)
    int n_sg;
    const uint16_t* sc;
    const uint16_t* bi;
    int* status;
};

// ---- tcgen05 / TMEM / TMA wrappers ----------------------------------------------
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
// D[tmem] (+)= A[tmem] . B[smem]^T, fp16 operands, fp32 accumulator.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
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
// 16 consecutive TMEM columns of this warp's 32 lanes <- 16 registers per thread.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
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
// fp16 number idx (0..7) of an 8-value row, replicated into both halves.
__device__ __forceinline__ __half2 half_at(const uint4& v, int idx) {
    const uint32_t lo = (idx & 2) ? v.y : v.x, hi = (idx & 2) ? v.w : v.z;
    const uint32_t wd = (idx & 4) ? hi : lo;
    const uint32_t h = (idx & 1) ? (wd >> 16) : (wd & 0xFFFFu);
    return bits_h2(h | (h << 16));
}

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
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_w4a16_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s,
                      const __grid_constant__ CUtensorMap tm_b, const GemmParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // SW128 atoms need 1024-byte alignment
    unsigned char* sm = smem_raw + (base - raw);
    const int S = p.stages, T = p.t_tile, DW = p.wslots, SA = p.astages;
    const int b_stage = T * 128;
    const uint32_t w_base = base;                                  // packed super-block ring
    const uint32_t b_base = base + (uint32_t)(DW * kWSlotBytes);   // activation stages
    const uint32_t bar0 = b_base + (uint32_t)(S * b_stage);
    auto full_bar = [&](int s) { return bar0 + 8u * (uint32_t)s; };                 // B stage filled
    auto empty_bar = [&](int s) { return bar0 + 8u * (uint32_t)(S + s); };          // B stage consumed
    auto wfull_bar = [&](int j) { return bar0 + 8u * (uint32_t)(2 * S + j); };
    auto wempty_bar = [&](int j) { return bar0 + 8u * (uint32_t)(2 * S + DW + j); };
    auto afull_bar = [&](int a) { return bar0 + 8u * (uint32_t)(2 * S + 2 * DW + a); };
    auto aempty_bar = [&](int a) { return bar0 + 8u * (uint32_t)(2 * S + 2 * DW + SA + a); };
    const uint32_t accum_bar = bar0 + 8u * (uint32_t)(2 * S + 2 * DW + 2 * SA);
    const uint32_t tmem_slot = accum_bar + 8u;
    volatile uint32_t* tmem_slot_ptr = reinterpret_cast<volatile uint32_t*>(sm + (tmem_slot - base));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * kGemmRows;
    const int kr = blockIdx.y;  // K-split rank (= cluster rank: the cluster spans grid y)
    const int tt = blockIdx.z, tok0 = tt * T;
    const int mt = min(T, p.m - tok0);
    // K range in whole super-blocks, so each super-block's groups sit in one
    // 8-group scale tile
    const int nsb_all = (p.nkb + 3) >> 2;
    const int sb0 = (int)((long long)kr * nsb_all / p.ks), sb1 = (int)((long long)(kr + 1) * nsb_all / p.ks);
    const int kb0 = 4 * sb0, kb1 = min(p.nkb, 4 * sb1);
    const int nk = kb1 - kb0, nsb = sb1 - sb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(full_bar(s), 1);            // the copy's expect_tx
            mbar_init(empty_bar(s), 1);           // MMA commit
        }
        for (int j = 0; j < DW; j++) {
            mbar_init(wfull_bar(j), 1);           // the TMA's expect_tx
            mbar_init(wempty_bar(j), kAWarps);    // one arrive per dequant warp
        }
        for (int a = 0; a < SA; a++) {
            mbar_init(afull_bar(a), kAWarps);     // one arrive per dequant warp
            mbar_init(aempty_bar(a), 1);          // MMA commit
        }
        mbar_init(accum_bar, 1);
    }
    if (warp == kMmaWarp) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // TMEM: A stages at columns [0, 128 SA), then nacc accumulators of
    // acc_stride columns.  Consecutive MMAs go to different accumulators so
    // small-N MMAs do not wait on one another's accumulation; the epilogue
    // adds the accumulators in a fixed order.
    const uint32_t tmem = *tmem_slot_ptr;
    const uint32_t acc_col = (uint32_t)(128 * SA);
    const int NACC = p.nacc, ACS = p.acc_stride;
    pdl_launch_dependents();

    bool fail = false;
    if (warp < kAWarps) {
        // ---- dequantise weights into the TMEM A stages ----------------------------------
        // Thread (r, h): weight row r, words 4h..4h+3 of each k-block (warps
        // 0-3 are h = 0, warps 4-7 h = 1; warp w writes TMEM lanes of
        // quadrant w % 4 = its rows).  Every dequant thread takes part in
        // every k-block, in order.
        const int h = warp >> 2;
        const int r = (warp & 3) * 32 + lane;
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        for (int j = 0; j < nsb && !fail; j++) {
            const int slot = j % DW, a = j % SA;
            if (!mbar_wait_ns(wfull_bar(slot), (uint32_t)(j / DW) & 1u, kGemmWaitNs)) {
                fail = true;
                break;
            }
            const unsigned char* wt = sm + (w_base - base) + (size_t)slot * kWSlotBytes;
            const int kbf = kb0 + 4 * j;
            int g_start;
            uint4 s8, b8;
            if (p.sb_tma) {
                g_start = (kbf >> p.gs_shift) & ~7;
                s8 = *reinterpret_cast<const uint4*>(wt + kWTileBytes + r * 16);
                b8 = *reinterpret_cast<const uint4*>(wt + kWTileBytes + kSTileBytes + r * 16);
            } else {
                // scale rows whose stride TMA cannot take: this row's (up to)
                // 4 groups of the super-block straight from global memory
                g_start = kbf >> p.gs_shift;
                const int grow_c = min(row0 + r, p.n_out - 1);
                const uint16_t* sr = p.sc + (size_t)grow_c * p.n_sg;
                const uint16_t* br = p.bi + (size_t)grow_c * p.n_sg;
                uint32_t sw[4], bw[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int g = min(g_start + u, p.n_sg - 1);
                    sw[u] = ldg_u16(sr + g);
                    bw[u] = ldg_u16(br + g);
                }
                s8 = make_uint4(sw[0] | (sw[1] << 16), sw[2] | (sw[3] << 16), 0, 0);
                b8 = make_uint4(bw[0] | (bw[1] << 16), bw[2] | (bw[3] << 16), 0, 0);
            }
            uint4 wv[4];
#pragma unroll
            for (int u = 0; u < 4; u++) wv[u] = *reinterpret_cast<const uint4*>(wt + sw128_off(r, 2 * u + h));
            // the TMEM A stage must have been consumed by the MMAs of super-block j - SA
            if (j >= SA && !mbar_wait_ns(aempty_bar(a), (uint32_t)((j / SA) - 1) & 1u, kGemmWaitNs)) {
                fail = true;
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int u = 0; u < 4; u++) {  // all 4 k-blocks (past the range: unused columns)
                const int gi = ((kbf + u) >> p.gs_shift) - g_start;
                const __half2 s2 = half_at(s8, min(gi, 7)), b2 = half_at(b8, min(gi, 7));
                uint32_t v[16];
                const uint4 d0 = dequant_word(wv[u].x, s2, b2), d1 = dequant_word(wv[u].y, s2, b2);
                const uint4 d2 = dequant_word(wv[u].z, s2, b2), d3 = dequant_word(wv[u].w, s2, b2);
                v[0] = d0.x; v[1] = d0.y; v[2] = d0.z; v[3] = d0.w;
                v[4] = d1.x; v[5] = d1.y; v[6] = d1.z; v[7] = d1.w;
                v[8] = d2.x; v[9] = d2.y; v[10] = d2.z; v[11] = d2.w;
                v[12] = d3.x; v[13] = d3.y; v[14] = d3.z; v[15] = d3.w;
                tmem_st16(tmem + lane_base + (uint32_t)(a * 128 + u * 32 + 16 * h), v);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(afull_bar(a));
                mbar_arrive(wempty_bar(slot));  // this warp is done reading the slot
            }
        }
    } else if (warp == kLoadWarp) {
        // ---- one loader, issuing in consumption order --------------------------------
        // per super-block j: its packed weights, scales and biases (2D TMA),
        // then the prepared activation blocks of its k-blocks (bulk copies).
        // One queue in consumption order keeps an activation copy from
        // waiting behind weight loads issued for later super-blocks.
        if (lane == 0) {
            const uint64_t pol_w = l2_policy_evict_first();
            const uint64_t pol_x = l2_policy_evict_last();
            const unsigned char* src = p.xw + ((size_t)tt * p.nkb + kb0) * (size_t)b_stage;
            bool waited = false;
            for (int j = 0; j < nsb && !fail; j++) {
                const int slot = j % DW;
                if (j >= DW && !mbar_wait_nap(wempty_bar(slot), (uint32_t)((j / DW) - 1) & 1u, kGemmWaitNs, 64)) {
                    fail = true;
                    break;
                }
                const uint32_t dst = w_base + (uint32_t)(slot * kWSlotBytes);
                const int kbf = kb0 + 4 * j;
                const int g_start = (kbf >> p.gs_shift) & ~7;
                mbar_arrive_expect_tx(wfull_bar(slot), (uint32_t)(p.sb_tma ? kWSlotBytes : kWTileBytes));
                tma_load_2d(dst, &tm_w, kbf * 8, row0, wfull_bar(slot), pol_w);
                if (p.sb_tma) {
                    tma_load_2d(dst + kWTileBytes, &tm_s, g_start, row0, wfull_bar(slot), pol_w);
                    tma_load_2d(dst + kWTileBytes + kSTileBytes, &tm_b, g_start, row0, wfull_bar(slot), pol_w);
                }
                if (!waited) {
                    pdl_wait();  // the activation workspace is written by the preparation kernel
                    waited = true;
                }
                for (int u = 0; u < 4; u++) {
                    const int i = 4 * j + u;
                    if (i >= nk) break;
                    const int s = i % S;
                    if (i >= S && !mbar_wait_nap(empty_bar(s), (uint32_t)((i / S) - 1) & 1u, kGemmWaitNs, 64)) {
                        fail = true;
                        break;
                    }
                    mbar_arrive_expect_tx(full_bar(s), (uint32_t)b_stage);
                    bulk_load_g2s(b_base + (uint32_t)(s * b_stage), src + (size_t)i * b_stage, (uint32_t)b_stage,
                                  full_bar(s), pol_x);
                }
                // the weight ring is full: ask L2 for the rest of this CTA's rows
                // now, so each row is read from DRAM in one pass
                if (j + 1 == min(DW, nsb))
                    for (int jj = DW; jj < nsb; jj++) tma_prefetch_l2_2d(&tm_w, (kb0 + 4 * jj) * 8, row0);
            }
        }
    } else if (lane == 0) {
        // ---- MMA issue ------------------------------------------------------------------
        const uint32_t idesc = (1u << 4)                        // D fp32
                               | ((uint32_t)(T >> 3) << 17)     // N
                               | ((uint32_t)(kGemmRows >> 4) << 24);  // M
        // stage / phase counters instead of divisions: this loop paces the MMAs
        int a = 0, s = 0, acc = 0;
        uint32_t pa = 0, pb = 0;
        bool first = true;
        uint32_t dcol = tmem + acc_col;  // current accumulator
        for (int j = 0; j < nsb && !fail; j++) {
            if (!mbar_wait_spin(afull_bar(a), pa, kGemmWaitNs)) {
                fail = true;
                break;
            }
            const uint32_t abase = tmem + (uint32_t)(a * 128);
            const int nu = min(4, nk - 4 * j);
            for (int u = 0; u < nu; u++) {
                if (!mbar_wait_spin(full_bar(s), pb, kGemmWaitNs)) {
                    fail = true;
                    break;
                }
                tc_fence_after();
                const uint64_t bd = sw128_desc(b_base + (uint32_t)(s * b_stage));
                const uint32_t acol = abase + (uint32_t)(u * 32);
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {  // 16 k per instruction: A +8 TMEM columns, B +32 bytes
                    umma_f16_ts(dcol, acol + 8u * kk, bd + 2u * kk, idesc, first ? 0u : 1u);
                    dcol += (uint32_t)ACS;
                    if (++acc == NACC) {
                        acc = 0;
                        dcol = tmem + acc_col;
                        first = false;
                    }
                }
                umma_commit(empty_bar(s));
                if (++s == S) {
                    s = 0;
                    pb ^= 1u;
                }
            }
            umma_commit(aempty_bar(a));
            if (++a == SA) {
                a = 0;
                pa ^= 1u;
            }
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
        const uint32_t trow = tmem + acc_col + ((uint32_t)((warp & 3) * 32) << 16);
        for (int c0 = (warp >> 2) * 32; c0 < T; c0 += 64) {
            uint32_t v[32];
            tmem_ld32(trow + (uint32_t)c0, v);
            tmem_wait_ld();
            for (int c = 1; c < NACC; c++) {  // accumulators in a fixed order
                uint32_t w2[32];
                tmem_ld32(trow + (uint32_t)(c * ACS + c0), w2);
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 32; q++) v[q] = __float_as_uint(__uint_as_float(v[q]) + __uint_as_float(w2[q]));
            }
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
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---- host side --------------------------------------------------------------------------
struct GemmPlan {
    int t_tile, n_tt, row_tiles, ks, stages, astages, wslots, nacc, acc_stride;
    size_t smem;
    size_t ws_bytes;
};

static int sm_count_gemm() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

static size_t gemm_smem(int t_tile, int stages, int wslots, int astages) {
    return 1024 + (size_t)wslots * kWSlotBytes + (size_t)stages * t_tile * 128 +
           8 * (size_t)(2 * stages + 2 * wslots + 2 * astages + 1) + 16;
}

static GemmPlan plan_gemm(int n_out, int n_in, int m) {
    GemmPlan pl{};
    pl.n_tt = (m + kMaxTile - 1) / kMaxTile;
    const int per = (m + pl.n_tt - 1) / pl.n_tt;             // balance the token tiles
    pl.t_tile = std::min(kMaxTile, (per + 15) / 16 * 16);
    pl.row_tiles = (n_out + kGemmRows - 1) / kGemmRows;
    // TMEM (512 columns): 128 per A stage + nacc accumulators of t_tile
    // rounded up to 32
    pl.acc_stride = (pl.t_tile + 31) / 32 * 32;
    if (pl.acc_stride <= 32) {
        pl.astages = 3;
        pl.nacc = 4;
    } else if (pl.acc_stride <= 64) {
        pl.astages = 2;
        pl.nacc = 4;
    } else if (pl.acc_stride <= 128) {
        pl.astages = 2;
        pl.nacc = 2;
    } else {
        pl.astages = 2;
        pl.nacc = 1;
    }
    // the loader runs min(weight slots, activation stages / 4) super-blocks
    // ahead: give both rings that depth, as deep as shared memory allows
    pl.wslots = 6;
    pl.stages = 24;
    while (gemm_smem(pl.t_tile, pl.stages, pl.wslots, pl.astages) > (size_t)kGemmSmemMax) {
        if (pl.stages > 4 * pl.wslots - 4 || pl.wslots <= 2) {
            if (pl.stages > 4) pl.stages -= 4;
            else break;
        } else {
            pl.wslots--;
        }
    }
    pl.smem = gemm_smem(pl.t_tile, pl.stages, pl.wslots, pl.astages);
    const int sms = sm_count_gemm();
    const int ctas = pl.row_tiles * pl.n_tt;
    const int nsb = (n_in / 64 + 3) / 4;
    int ks = 1;
    if (ctas < sms) {
        static SplitPicker picker;
        ks = picker.pick((const void*)gemm_w4a16_kernel, kGemmThreads, pl.smem, kGemmSmemMax, ctas,
                         std::min({8, nsb, std::max(1, sms / ctas)}));
    }
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

// ---- tensor maps (hq4_tmap.cuh)
// rows x cols 2D map of `elem`-byte elements, box (box_cols x 128 rows)
static bool make_map(CUtensorMap* tm, const void* ptr, CUtensorMapDataType dt, int elem, long long rows,
                     long long cols, int box_cols, bool swizzle128) {
    return make_map_2d(tm, ptr, dt, elem, rows, cols, box_cols, kGemmRows, swizzle128);
}

struct WeightMaps {
    const void* w;
    const void* s;
    const void* b;
    int n_out, n_in, n_sg, dev;
    bool sb_tma;
    CUtensorMap tw, ts, tb;
};

// The three maps of a weight matrix, cached by (pointers, shape, device).
static bool weight_maps(const uint32_t* w, const uint16_t* sc, const uint16_t* bi, int n_out, int n_in, int n_sg,
                        WeightMaps* outm) {
    static std::mutex mu;
    static WeightMaps cache[64];
    static int used = 0, next = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> g(mu);
    for (int i = 0; i < used; i++) {
        const WeightMaps& c = cache[i];
        if (c.w == w && c.s == sc && c.b == bi && c.n_out == n_out && c.n_in == n_in && c.n_sg == n_sg &&
            c.dev == dev) {
            *outm = c;
            return true;
        }
    }
    WeightMaps m{};
    m.w = w;
    m.s = sc;
    m.b = bi;
    m.n_out = n_out;
    m.n_in = n_in;
    m.n_sg = n_sg;
    m.dev = dev;
    // scale tiles by TMA need a row stride (n_sg * 2 bytes) and base that are
    // multiples of 16 bytes
    m.sb_tma = n_sg % 8 == 0 && (((uintptr_t)sc | (uintptr_t)bi) & 15) == 0;
    if (!make_map(&m.tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, n_out, n_in / 8, 32, true)) return false;
    if (m.sb_tma) {
        if (!make_map(&m.ts, sc, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, n_out, n_sg, 8, false) ||
            !make_map(&m.tb, bi, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, n_out, n_sg, 8, false))
            return false;
    } else {
        m.ts = m.tw;  // unused
        m.tb = m.tw;
    }
    const int at = used < 64 ? used++ : (next++ & 63);
    cache[at] = m;
    *outm = m;
    return true;
}

static int launch_gemm(const WeightMaps& wm, const GemmParams& prm, const GemmPlan& pl, cudaStream_t st) {
    // the shared-memory opt-in is a per-device function attribute
    static PerDeviceOnce attr_once;
    if (smem_opt_in(attr_once, gemm_w4a16_kernel, kGemmSmemMax) != cudaSuccess) return HQ4_ERR_LAUNCH;
    // split-K partial tile [t_tile][128] fp32 lives in the (drained) rings;
    // A stages + accumulator fit the 512 TMEM columns
    if ((size_t)pl.t_tile * kGemmRows * 4 > (size_t)pl.wslots * kWSlotBytes + (size_t)pl.stages * pl.t_tile * 128 ||
        pl.smem > (size_t)kGemmSmemMax || 128 * pl.astages + pl.nacc * pl.acc_stride > kTmemCols)
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
    return cudaLaunchKernelEx(&lc, gemm_w4a16_kernel, wm.tw, wm.ts, wm.tb, prm) == cudaSuccess ? HQ4_OK
                                                                                             : HQ4_ERR_LAUNCH;
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


// ===========================================================================
// Small token counts: register-path MMAs on the same weight stream.
//
// For m up to 16 (bf16 x) the tensor work per weight byte is small and the
// cost of issuing tcgen05.mma from one thread dominates, so here every
// consumer warp issues its own warp-level MMAs (mma.sync m16n8k16, bf16 in,
// fp32 accumulate) on the packed weights the loader streams in by TMA:
//
//   * warp w (0-7) owns CTA rows 16w..16w+15; lane (g, t) = (lane/4, lane%4)
//     holds rows g and g+8;
//   * weights enter the MMA as 128+q in bf16 (exact: nibble OR 0x4300), so a
//     64-wide group's product is D = sum (128+q) x, folded per group into
//     fp32 accumulators as  acc += s*D + (b - 128 s) * X,  X = sum of the
//     group's x (exact in fp32 up to summation order);
//   * lane t uses words 2t, 2t+1 of each group; k-step kk takes nibbles
//     (kk, kk+4) of each word, so x is pre-arranged (xprep_frag) in exactly
//     that order: per (group, 8-token tile) 32 bytes per lane, then the
//     tile's 8 group sums;
//   * fp32 x becomes two bf16 "virtual tokens" (hi, x - hi), placed in the
//     two C columns a lane owns and added at the end (16 significant bits).
// ===========================================================================
constexpr int kFragBlock = 1024 + 32;   // per (group, 8-token tile): fragments + 8 group sums

__device__ __forceinline__ uint32_t bf16_bits(float f) {  // round to nearest even (finite inputs)
    const uint32_t u = __float_as_uint(f);
    return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}
__device__ __forceinline__ float bf16_to_f(uint32_t h) { return __uint_as_float(h << 16); }

// x [m][n_in] (bf16 or fp32) -> per (super-block, group u, tile n, lane) fragments.
// Thread per (group G, tile n, lane l): 16 values + (lane < 8) the group sum of token n*8+lane.
template <bool XF32>
__global__ void __launch_bounds__(kPrepThreads) gemm_xprep_frag_kernel(const void* __restrict__ x,
                                                                     unsigned char* __restrict__ ws, int m,
                                                                     int n_in, int nt, int* status) {
    pdl_launch_dependents();
    pdl_wait();
    const int ng = n_in >> 6;
    const long long total = (long long)ng * nt * 32;
    float amax = 0.0f;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int l = (int)(i & 31);
        const int n = (int)((i >> 5) % nt);
        const int G = (int)((i >> 5) / nt);
        const int g = l >> 2, t = l & 3;
        // virtual token v of this lane's column: tile n, column g
        const int v = n * 8 + g;
        const int tok = XF32 ? (v >> 1) : v;
        const bool lo_part = XF32 && (v & 1);
        const bool live = tok < m;
        auto xval = [&](int k) -> float {  // the virtual token's value at group-local k, exactly bf16
            if (!live) return 0.0f;
            const size_t e = (size_t)tok * n_in + (size_t)G * 64 + k;
            float f;
            if constexpr (XF32) {
                const float xf = __ldg(reinterpret_cast<const float*>(x) + e);
                const float hi = bf16_to_f(bf16_bits(xf));
                f = lo_part ? bf16_to_f(bf16_bits(xf - hi)) : hi;
                amax = fmaxf(amax, fabsf(xf));
            } else {
                f = bf16_to_f(__ldg(reinterpret_cast<const unsigned short*>(x) + e));
            }
            return f;
        };
        uint32_t o[8];
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            const float a = xval(16 * t + kk), b = xval(16 * t + kk + 4);
            const float c = xval(16 * t + 8 + kk), d = xval(16 * t + 12 + kk);
            o[2 * kk] = bf16_bits(a) | (bf16_bits(b) << 16);
            o[2 * kk + 1] = bf16_bits(c) | (bf16_bits(d) << 16);
        }
        const int sb = G >> 2, u = G & 3;
        unsigned char* blk = ws + (((size_t)sb * 4 + u) * nt + n) * kFragBlock;
        uint4* dst = reinterpret_cast<uint4*>(blk + l * 32);
        dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
        dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        if (l < 8) {  // group sum X of virtual token n*8 + l, from the same bf16 values
            const int vv = n * 8 + l;
            const int tk = XF32 ? (vv >> 1) : vv;
            float sum = 0.0f;
            if (tk < m) {
                for (int k = 0; k < 64; k++) {
                    const size_t e = (size_t)tk * n_in + (size_t)G * 64 + k;
                    float f;
                    if constexpr (XF32) {
                        const float xf = __ldg(reinterpret_cast<const float*>(x) + e);
                        const float hi = bf16_to_f(bf16_bits(xf));
                        f = (vv & 1) ? bf16_to_f(bf16_bits(xf - hi)) : hi;
                    } else {
                        f = bf16_to_f(__ldg(reinterpret_cast<const unsigned short*>(x) + e));
                    }
                    sum += f;
                }
            }
            reinterpret_cast<float*>(blk + 1024)[l] = sum;
        }
    }
    (void)status;
    (void)amax;
}

struct SmallParams {
    const unsigned char* xw;
    float* out;
    const float* row_add;
    const float* residual;
    int n_out, n_in, m, nkb, ks, nt, xf32, gs_shift;
    int bstages, wslots, sb_tma, n_sg;
    const uint16_t* sc;
    const uint16_t* bi;
    int* status;
};

template <int NT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_small_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s,
                      const __grid_constant__ CUtensorMap tm_b, const SmallParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* sm = smem_raw + (base - raw);
    const int DW = p.wslots;
    // one ring slot per super-block: packed weights | scales | biases | activation fragments
    const int b_bytes = 4 * NT * kFragBlock;
    const int slot_bytes = (kWSlotBytes + b_bytes + 1023) & ~1023;
    const uint32_t w_base = base;
    const uint32_t bar0 = base + (uint32_t)(DW * slot_bytes);
    auto full_bar = [&](int j) { return bar0 + 8u * (uint32_t)j; };
    auto empty_bar = [&](int j) { return bar0 + 8u * (uint32_t)(DW + j); };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * kGemmRows;
    const int kr = blockIdx.y;
    const int nsb_all = (p.nkb + 3) >> 2;
    const int sb0 = (int)((long long)kr * nsb_all / p.ks), sb1 = (int)((long long)(kr + 1) * nsb_all / p.ks);
    const int kb0 = 4 * sb0, kb1 = min(p.nkb, 4 * sb1);
    const int nk = kb1 - kb0, nsb = sb1 - sb0;

    if (threadIdx.x == 0) {
        for (int j = 0; j < DW; j++) {
            mbar_init(full_bar(j), 1);           // the loader's expect_tx
            mbar_init(empty_bar(j), kAWarps);    // one arrive per consumer warp
        }
    }
    __syncthreads();
    pdl_launch_dependents();

    bool fail = false;
    const int g = lane >> 2, t = lane & 3;
    float acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++)
#pragma unroll
        for (int q = 0; q < 4; q++) acc[n][q] = 0.0f;

    if (warp < kAWarps) {
        const int R0 = warp * 16 + g, R1 = R0 + 8;  // CTA rows of this lane
        int slot = 0;
        uint32_t ph = 0;
        for (int j = 0; j < nsb && !fail; j++) {
            if (!mbar_wait_ns(full_bar(slot), ph, kGemmWaitNs)) {
                fail = true;
                break;
            }
            const unsigned char* wt = sm + (size_t)slot * slot_bytes;
            const unsigned char* xt = wt + kWSlotBytes;
            const int kbf = kb0 + 4 * j;
            const int nu = min(4, nk - 4 * j);
            int g_start;
            uint4 s0, s1, c0, c1;  // scales / biases of rows R0, R1 (8 groups)
            if (p.sb_tma) {
                g_start = (kbf >> p.gs_shift) & ~7;
                s0 = *reinterpret_cast<const uint4*>(wt + kWTileBytes + R0 * 16);
                s1 = *reinterpret_cast<const uint4*>(wt + kWTileBytes + R1 * 16);
                c0 = *reinterpret_cast<const uint4*>(wt + kWTileBytes + kSTileBytes + R0 * 16);
                c1 = *reinterpret_cast<const uint4*>(wt + kWTileBytes + kSTileBytes + R1 * 16);
            } else {
                g_start = kbf >> p.gs_shift;
                uint32_t a[4], b[4], cc[4], d[4];
                const int r0c = min(row0 + R0, p.n_out - 1), r1c = min(row0 + R1, p.n_out - 1);
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int gg = min(g_start + u, p.n_sg - 1);
                    a[u] = ldg_u16(p.sc + (size_t)r0c * p.n_sg + gg);
                    b[u] = ldg_u16(p.sc + (size_t)r1c * p.n_sg + gg);
                    cc[u] = ldg_u16(p.bi + (size_t)r0c * p.n_sg + gg);
                    d[u] = ldg_u16(p.bi + (size_t)r1c * p.n_sg + gg);
                }
                s0 = make_uint4(a[0] | (a[1] << 16), a[2] | (a[3] << 16), 0, 0);
                s1 = make_uint4(b[0] | (b[1] << 16), b[2] | (b[3] << 16), 0, 0);
                c0 = make_uint4(cc[0] | (cc[1] << 16), cc[2] | (cc[3] << 16), 0, 0);
                c1 = make_uint4(d[0] | (d[1] << 16), d[2] | (d[3] << 16), 0, 0);
            }
            // A fragments of all 4 groups first (128+q as bf16 pairs): pair kk of a
            // word = nibbles (kk, kk+4); words 2t, 2t+1 of each group, rows R0, R1
            uint32_t A[4][4][4];  // [group u][kk][a0..a3]
            float sr0[4], sr1[4], br0[4], br1[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int cidx = 2 * u + (t >> 1);
                const uint2 w0 = *reinterpret_cast<const uint2*>(wt + R0 * 128 + ((cidx ^ (R0 & 7)) << 4) + (t & 1) * 8);
                const uint2 w1 = *reinterpret_cast<const uint2*>(wt + R1 * 128 + ((cidx ^ (R1 & 7)) << 4) + (t & 1) * 8);
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    A[u][kk][0] = lop3_and_or(w0.x >> (4 * kk), 0x000F000Fu, 0x43004300u);
                    A[u][kk][1] = lop3_and_or(w1.x >> (4 * kk), 0x000F000Fu, 0x43004300u);
                    A[u][kk][2] = lop3_and_or(w0.y >> (4 * kk), 0x000F000Fu, 0x43004300u);
                    A[u][kk][3] = lop3_and_or(w1.y >> (4 * kk), 0x000F000Fu, 0x43004300u);
                }
                const int gi = min(((kbf + u) >> p.gs_shift) - g_start, 7);
                sr0[u] = __half2float(__low2half(half_at(s0, gi)));
                sr1[u] = __half2float(__low2half(half_at(s1, gi)));
                br0[u] = fmaf(-128.0f, sr0[u], __half2float(__low2half(half_at(c0, gi))));
                br1[u] = fmaf(-128.0f, sr1[u], __half2float(__low2half(half_at(c1, gi))));
            }
#pragma unroll
            for (int n = 0; n < NT; n++) {
                // four independent MMA chains (one per group), interleaved
                float D[4][4];
                uint4 F0[4], F1[4];
                float2 X[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const unsigned char* fb = xt + (size_t)(u * NT + n) * kFragBlock;
                    F0[u] = *reinterpret_cast<const uint4*>(fb + lane * 32);
                    F1[u] = *reinterpret_cast<const uint4*>(fb + lane * 32 + 16);
                    X[u] = *reinterpret_cast<const float2*>(fb + 1024 + 8 * t);
#pragma unroll
                    for (int q = 0; q < 4; q++) D[u][q] = 0.0f;
                }
#pragma unroll
                for (int kk = 0; kk < 4; kk++)
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const uint32_t b0 = kk == 0 ? F0[u].x : kk == 1 ? F0[u].z : kk == 2 ? F1[u].x : F1[u].z;
                        const uint32_t b1 = kk == 0 ? F0[u].y : kk == 1 ? F0[u].w : kk == 2 ? F1[u].y : F1[u].w;
                        mma_bf16_16816(D[u], A[u][kk][0], A[u][kk][1], A[u][kk][2], A[u][kk][3], b0, b1);
                    }
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    if (u < nu) {  // D: (R0, col 2t), (R0, 2t+1), (R1, 2t), (R1, 2t+1)
                        acc[n][0] = fmaf(sr0[u], D[u][0], fmaf(br0[u], X[u].x, acc[n][0]));
                        acc[n][1] = fmaf(sr0[u], D[u][1], fmaf(br0[u], X[u].y, acc[n][1]));
                        acc[n][2] = fmaf(sr1[u], D[u][2], fmaf(br1[u], X[u].x, acc[n][2]));
                        acc[n][3] = fmaf(sr1[u], D[u][3], fmaf(br1[u], X[u].y, acc[n][3]));
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar(slot));
            if (++slot == DW) {
                slot = 0;
                ph ^= 1u;
            }
        }
    } else if (warp == kLoadWarp) {
        if (lane == 0) {
            const uint64_t pol_w = l2_policy_evict_first();
            const uint64_t pol_x = l2_policy_evict_last();
            bool waited = false;
            int slot = 0;
            uint32_t ph = 0;
            for (int j = 0; j < nsb && !fail; j++) {
                if (j >= DW && !mbar_wait_nap(empty_bar(slot), ph ^ 1u, kGemmWaitNs, 64)) {
                    fail = true;
                    break;
                }
                const uint32_t dst = w_base + (uint32_t)(slot * slot_bytes);
                const int kbf = kb0 + 4 * j;
                const int g_start = (kbf >> p.gs_shift) & ~7;
                mbar_arrive_expect_tx(full_bar(slot),
                                      (uint32_t)((p.sb_tma ? kWSlotBytes : kWTileBytes) + b_bytes));
                tma_load_2d(dst, &tm_w, kbf * 8, row0, full_bar(slot), pol_w);
                if (p.sb_tma) {
                    tma_load_2d(dst + kWTileBytes, &tm_s, g_start, row0, full_bar(slot), pol_w);
                    tma_load_2d(dst + kWTileBytes + kSTileBytes, &tm_b, g_start, row0, full_bar(slot), pol_w);
                }
                if (!waited) {
                    pdl_wait();  // the fragment workspace is written by the preparation kernel
                    waited = true;
                }
                bulk_load_g2s(dst + kWSlotBytes, p.xw + (size_t)(sb0 + j) * b_bytes, (uint32_t)b_bytes,
                              full_bar(slot), pol_x);
                // the ring is full: ask L2 for the rest of this CTA's rows now, so
                // each weight row is read from DRAM in one pass, not 128 bytes
                // per super-block as the ring drains
                if (j + 1 == min(DW, nsb))
                    for (int jj = DW; jj < nsb; jj++) tma_prefetch_l2_2d(&tm_w, (kb0 + 4 * jj) * 8, row0);
                if (++slot == DW) {
                    slot = 0;
                    ph ^= 1u;
                }
            }
        }
    }
    if (fail && p.status) atomicOr(p.status, 1);

    // ---- epilogue ------------------------------------------------------------------------
    // lane (g, t) of warp w holds rows 16w+g, 16w+g+8 x columns (2t, 2t+1) of each tile:
    // bf16 x: tokens 8n+2t, 8n+2t+1; fp32 x: token 4n+t (hi + lo columns added).
    float* part = reinterpret_cast<float*>(sm);  // split-K partials [tokens][128], reuses the ring
    const int tok_per_tile = p.xf32 ? 4 : 8;
    const int tcap = NT * tok_per_tile;
    if (warp < kAWarps) {
        pdl_wait();
        // the partials overwrite the ring: every consumer warp must be done
        // reading it first (named barrier 1 over the consumer warps)
        if (p.ks > 1) asm volatile("bar.sync 1, %0;" ::"r"(kAWarps * 32) : "memory");
        const int R0 = warp * 16 + g, R1 = R0 + 8;
#pragma unroll
        for (int n = 0; n < NT; n++) {
#pragma unroll
            for (int hc = 0; hc < 2; hc++) {  // column 2t + hc
                const int tok = p.xf32 ? n * 4 + t : n * 8 + 2 * t + hc;
                if (p.xf32 && hc == 1) continue;
                const float y0 = p.xf32 ? acc[n][0] + acc[n][1] : acc[n][hc];
                const float y1 = p.xf32 ? acc[n][2] + acc[n][3] : acc[n][2 + hc];
                if (p.ks == 1) {
                    if (tok < p.m) {
                        const int r[2] = {row0 + R0, row0 + R1};
                        const float yv[2] = {y0, y1};
#pragma unroll
                        for (int q = 0; q < 2; q++) {
                            if (r[q] < p.n_out) {
                                const size_t o = (size_t)tok * p.n_out + r[q];
                                float y = yv[q];
                                if (p.row_add) y += p.row_add[r[q]];
                                if (p.residual) y += p.residual[o];
                                p.out[o] = y;
                            }
                        }
                    }
                } else {
                    part[tok * kGemmRows + R0] = y0;
                    part[tok * kGemmRows + R1] = y1;
                }
            }
        }
    }
    __syncwarp();
    if (p.ks > 1) {
        cluster_sync();
        const int mt = min(p.m, tcap);
        const int t_lo = (int)((long long)kr * mt / p.ks), t_hi = (int)((long long)(kr + 1) * mt / p.ks);
        const int n_el = (t_hi - t_lo) * kGemmRows;
        for (int e = threadIdx.x; e < n_el; e += kGemmThreads) {
            const int tk = t_lo + e / kGemmRows, rr = e % kGemmRows;
            const int gr = row0 + rr;
            const uint32_t off = (uint32_t)((tk * kGemmRows + rr) * 4);
            float y = 0.0f;
            for (int q = 0; q < p.ks; q++) y += ld_cluster_f32(map_to_rank(base + off, (uint32_t)q));
            if (gr < p.n_out) {
                const size_t o = (size_t)tk * p.n_out + gr;
                if (p.row_add) y += p.row_add[gr];
                if (p.residual) y += p.residual[o];
                p.out[o] = y;
            }
        }
        cluster_sync();
    }
}

struct SmallPlan {
    int nt, row_tiles, ks, bstages, wslots;
    size_t smem, ws_bytes;
};

static size_t small_slot_bytes(int nt) { return ((size_t)kWSlotBytes + 4 * nt * kFragBlock + 1023) & ~(size_t)1023; }
static size_t small_smem(int nt, int bstages, int wslots) {
    (void)bstages;
    return 1024 + (size_t)wslots * small_slot_bytes(nt) + 16 * (size_t)wslots + 16;
}

static SmallPlan plan_small(int n_out, int n_in, int m, bool xf32) {
    SmallPlan pl{};
    const int v = xf32 ? 2 * m : m;
    pl.nt = v <= 8 ? 1 : v <= 16 ? 2 : v <= 32 ? 4 : 8;
    pl.row_tiles = (n_out + kGemmRows - 1) / kGemmRows;
    pl.wslots = 6;
    pl.bstages = 6;
    while (small_smem(pl.nt, pl.bstages, pl.wslots) > (size_t)kGemmSmemMax && pl.wslots > 2) {
        pl.wslots--;
        pl.bstages = pl.wslots;
    }
    pl.smem = small_smem(pl.nt, pl.bstages, pl.wslots);
    const int sms = sm_count_gemm();
    const int nsb = (n_in / 64 + 3) / 4;
    int ks = 1;
    if (pl.row_tiles < sms) {
        static SplitPicker picker;
        const void* kern = pl.nt == 1   ? (const void*)gemm_small_kernel<1>
                           : pl.nt == 2 ? (const void*)gemm_small_kernel<2>
                           : pl.nt == 4 ? (const void*)gemm_small_kernel<4>
                                        : (const void*)gemm_small_kernel<8>;
        ks = picker.pick(kern, kGemmThreads, pl.smem, kGemmSmemMax, pl.row_tiles,
                         std::min({8, nsb, std::max(1, sms / pl.row_tiles)}));
    }
    pl.ks = ks;
    pl.ws_bytes = (size_t)nsb * 4 * pl.nt * kFragBlock;
    return pl;
}

static bool use_small(int m, bool xf32) { return (xf32 ? 2 * m : m) <= 16; }

template <int NT>
static int launch_small_nt(const WeightMaps& wm, const SmallParams& prm, const SmallPlan& pl, cudaStream_t st) {
    static PerDeviceOnce attr_once;  // one per instantiation, as the attribute is per kernel
    if (smem_opt_in(attr_once, gemm_small_kernel<NT>, kGemmSmemMax) != cudaSuccess) return HQ4_ERR_LAUNCH;
    const int tcap = NT * (prm.xf32 ? 4 : 8);
    if (pl.smem > (size_t)kGemmSmemMax || (size_t)tcap * kGemmRows * 4 > (size_t)pl.wslots * small_slot_bytes(NT))
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
    lc.gridDim = dim3((unsigned)pl.row_tiles, (unsigned)pl.ks, 1);
    lc.blockDim = dim3(kGemmThreads);
    lc.dynamicSmemBytes = pl.smem;
    lc.stream = st;
    lc.attrs = attr;
    lc.numAttrs = na;
    return cudaLaunchKernelEx(&lc, gemm_small_kernel<NT>, wm.tw, wm.ts, wm.tb, prm) == cudaSuccess ? HQ4_OK
                                                                                               : HQ4_ERR_LAUNCH;
}

static int launch_small(const void* x, bool xf32, unsigned char* ws, const WeightMaps& wm, SmallParams prm,
                        const SmallPlan& pl, cudaStream_t st) {
    const long long total = (long long)(prm.n_in >> 6) * pl.nt * 32;
    const int blocks = (int)std::min<long long>((total + kPrepThreads - 1) / kPrepThreads, 4L * sm_count_gemm());
    cudaLaunchAttribute attr[1] = {pdl_attribute()};
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)blocks);
    lc.blockDim = dim3(kPrepThreads);
    lc.stream = st;
    lc.attrs = attr;
    lc.numAttrs = 1;
    cudaError_t e = xf32 ? cudaLaunchKernelEx(&lc, gemm_xprep_frag_kernel<true>, x, ws, prm.m, prm.n_in, pl.nt,
                                              prm.status)
                         : cudaLaunchKernelEx(&lc, gemm_xprep_frag_kernel<false>, x, ws, prm.m, prm.n_in, pl.nt,
                                              prm.status);
    if (e != cudaSuccess) return HQ4_ERR_LAUNCH;
    switch (pl.nt) {
        case 1: return launch_small_nt<1>(wm, prm, pl, st);
        case 2: return launch_small_nt<2>(wm, prm, pl, st);
        case 4: return launch_small_nt<4>(wm, prm, pl, st);
        default: return launch_small_nt<8>(wm, prm, pl, st);
    }
}

}  // namespace hq4

using namespace hq4;

static bool gemm_shape_ok(int n_out, int n_in, int gs, int m) {
    return n_out > 0 && n_in > 0 && m > 0 && gs >= 64 && gs % 64 == 0 && (gs & (gs - 1)) == 0 && n_in % gs == 0;
}

extern "C" long long hq4_gemm_workspace_bytes(int n_out, int n_in, int m) {
    if (n_out <= 0 || n_in <= 0 || m <= 0 || n_in % 64) return HQ4_ERR_SHAPE;
    // enough for either activation type
    size_t need = 0;
    for (int f = 0; f < 2; f++)
        need = std::max(need, use_small(m, f != 0) ? plan_small(n_out, n_in, m, f != 0).ws_bytes
                                                   : plan_gemm(n_out, n_in, m).ws_bytes);
    return (long long)need;
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
    const bool xf32 = x_is_f32 != 0;
    const bool small = use_small(m, xf32);
    const GemmPlan pl = plan_gemm(n_out, n_in, m);
    const SmallPlan sp = plan_small(n_out, n_in, m, xf32);
    if (!workspace || workspace_bytes < (long long)(small ? sp.ws_bytes : pl.ws_bytes)) return HQ4_ERR_SHAPE;
    if (m == 1) {  // one token: the streaming GEMV (the weights exact, x widened to fp32)
        bool used = false;
        const int rc = gemv_stream_m1(w, scales, biases, x, !xf32, out, n_out, n_in, gs, row_add, residual,
                                      static_cast<cudaStream_t>(stream), &used);
        if (rc || used) return rc;
    }
    if (m <= kMtMaxTok) {
        // a few tokens: the multi-token streaming kernel (the one-token
        // kernel's exact digit product, tokens sharing the weight fragments)
        MtParams mp = {};
        mp.w = w;
        mp.sc = scales;
        mp.bi = biases;
        mp.x = x;
        mp.x_stride = n_in;
        mp.x_bf16 = xf32 ? 0 : 1;
        mp.out = out;
        mp.out_stride = n_out;
        mp.n_out = n_out;
        mp.n_in = n_in;
        mp.m = m;
        mp.row_add = row_add;
        mp.residual = residual;
        mp.mode = kEpiPlain;
        bool used = false;
        const int rc = gemv_mt_pass(mp, gs, static_cast<cudaStream_t>(stream), &used);
        if (rc || used) return rc;
    }
    int* status = status_word();
    if (!status) return HQ4_ERR_LAUNCH;
    WeightMaps wm;
    if (!weight_maps(w, scales, biases, n_out, n_in, n_in / gs, &wm)) return HQ4_ERR_LAUNCH;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    int gsh = 0;
    while ((64 << gsh) < gs) gsh++;
    if (small) {
        SmallParams sprm{};
        sprm.xw = ws;
        sprm.out = out;
        sprm.row_add = row_add;
        sprm.residual = residual;
        sprm.n_out = n_out;
        sprm.n_in = n_in;
        sprm.m = m;
        sprm.nkb = n_in / 64;
        sprm.ks = sp.ks;
        sprm.nt = sp.nt;
        sprm.xf32 = xf32 ? 1 : 0;
        sprm.gs_shift = gsh;
        sprm.bstages = sp.bstages;
        sprm.wslots = sp.wslots;
        sprm.sb_tma = wm.sb_tma ? 1 : 0;
        sprm.n_sg = n_in / gs;
        sprm.sc = scales;
        sprm.bi = biases;
        sprm.status = status;
        return launch_small(x, xf32, ws, wm, sprm, sp, st);
    }
    if (int rc = launch_xprep(x, x_is_f32 != 0, ws, m, pl, n_in, status, st)) return rc;
    GemmParams prm{};
    prm.xw = ws;
    prm.out = out;
    prm.row_add = row_add;
    prm.residual = residual;
    prm.n_out = n_out;
    prm.n_in = n_in;
    prm.m = m;
    int sh = 0;
    while ((64 << sh) < gs) sh++;
    prm.gs_shift = sh;
    prm.nkb = n_in / 64;
    prm.ks = pl.ks;
    prm.t_tile = pl.t_tile;
    prm.stages = pl.stages;
    prm.astages = pl.astages;
    prm.nacc = pl.nacc;
    prm.acc_stride = pl.acc_stride;
    prm.wslots = pl.wslots;
    prm.sb_tma = wm.sb_tma ? 1 : 0;
    prm.n_sg = n_in / gs;
    prm.sc = scales;
    prm.bi = biases;
    prm.status = status;
    return launch_gemm(wm, prm, pl, st);
}

extern "C" int hq4_gemm_plan(int n_out, int n_in, int m, int x_is_f32, int* info) {
    if (n_out <= 0 || n_in <= 0 || m <= 0 || n_in % 64 || !info) return HQ4_ERR_SHAPE;
    if (m == 1 && gemv_stream_fits_gs64(n_out, n_in)) {
        for (int i = 0; i < 7; i++) info[i] = 0;
        info[7] = 2;  // streaming GEMV
        return HQ4_OK;
    }
    if (m >= 2 && gemv_mt_fits(n_out, n_in, 64, m)) {
        for (int i = 0; i < 7; i++) info[i] = 0;
        info[7] = 3;  // multi-token streaming kernel
        return HQ4_OK;
    }
    if (use_small(m, x_is_f32 != 0)) {
        const SmallPlan sp = plan_small(n_out, n_in, m, x_is_f32 != 0);
        info[0] = sp.row_tiles;
        info[1] = sp.ks;
        info[2] = 1;
        info[3] = sp.nt * 8;
        info[4] = sp.bstages;
        info[5] = (int)sp.smem;
        info[6] = sp.wslots;
        info[7] = 1;  // register-path MMAs
        return HQ4_OK;
    }
    const GemmPlan pl = plan_gemm(n_out, n_in, m);
    info[0] = pl.row_tiles;
    info[1] = pl.ks;
    info[2] = pl.n_tt;
    info[3] = pl.t_tile;
    info[4] = pl.stages;
    info[5] = (int)pl.smem;
    info[6] = pl.wslots;
    info[7] = 0;  // tcgen05 / TMEM
    return HQ4_OK;
}

// ---- allocation-free variant -------------------------------------------------
// The same GEMM with its workspace taken from a fixed area of this module's
// static device memory (one per device, allocated when the module loads), for
// callers that cannot allocate device memory.  Every call on a device uses the
// same area: calls queued on one stream are ordered and safe; calls that can
// overlap (different streams, or host threads without a common stream) race
// on it and must be serialised by the caller.
static __device__ __align__(256) unsigned char g_hq4_gemm_scratch[HQ4_GEMM_STATIC_SCRATCH_BYTES];

// Device address of g_hq4_gemm_scratch, resolved with cudaGetSymbolAddress
// once per device (the first call may load the module, so it must not happen
// while a stream is being captured); nullptr if the lookup fails.
static void* static_scratch() {
    static PerDeviceOnce once;
    static void* addr[kMaxDevices] = {nullptr};
    int dev = 0;
    const cudaError_t e = once.run([&](int d) {
        void* a = nullptr;
        const cudaError_t r = cudaGetSymbolAddress(&a, g_hq4_gemm_scratch);
        if (r != cudaSuccess || !a) {
            (void)cudaGetLastError();  // the failed lookup does not stick to later launches
            return r != cudaSuccess ? r : cudaErrorInvalidSymbol;
        }
        addr[d] = a;
        return cudaSuccess;
    });
    if (e != cudaSuccess || cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    return addr[dev];  // written before the once-flag's release store
}

extern "C" int hq4_gemm_w4a16_static(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                                     const void* x, int x_is_f32, float* out, int n_out, int n_in, int gs,
                                     int m, const float* row_add, const float* residual, void* stream) {
    if (int rc = check_device_cap()) return rc;
    const long long need = hq4_gemm_workspace_bytes(n_out, n_in, m);
    if (need < 0 || need > (long long)HQ4_GEMM_STATIC_SCRATCH_BYTES) return HQ4_ERR_SHAPE;
    void* ws = static_scratch();
    if (!ws) return HQ4_ERR_LAUNCH;
    return hq4_gemm_w4a16(w, scales, biases, x, x_is_f32, out, n_out, n_in, gs, m, row_add, residual, ws,
                          (long long)HQ4_GEMM_STATIC_SCRATCH_BYTES, stream);
}
