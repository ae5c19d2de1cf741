// W4A16 GEMM on the fifth-generation tensor cores (tcgen05 + TMEM):
// out[t][n] = sum_k x[t][k] * (q[n][k] * scale[n][g] + bias[n][g]),
// for token counts where the product is a real dense contraction (microbatched
// decode, prefill).  The reference computes the same product in
// QLinear._gemm (hetero/cpu_model.py:118-136) as fp32 dequantisation of
// 512-row blocks (kernel/q4gemv.c:311-379) followed by a BLAS matmul.
//
// One CTA owns 128 weight rows (the MMA's M) x up to 256 tokens (its N) and a
// contiguous range of 64-wide k-blocks:
//
//   warps 0-3   dequantise: thread = weight row; the row's 32 packed bytes of
//               a k-block become 64 fp16 values (q as fp16 through the 0x6400
//               exponent trick, then one fma with the group's scale and bias:
//               a single rounding of q*s+b), written K-major with the 128-byte
//               swizzle; after the mainloop the same warps read the fp32
//               accumulator out of TMEM (warp w owns lanes 32w..32w+31);
//   warps 4-11  convert the activation tile (bf16 or fp32) to fp16 in the
//               same layout;
//   warp 12     allocates TMEM and, from one thread, issues
//               tcgen05.mma.cta_group::1.kind::f16 (K=16 per instruction) on
//               each stage once both operands are in, releasing the stage
//               through tcgen05.commit.
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
// order (distributed shared memory loads).  Deterministic, no workspace, no
// atomics.
//
// Precision: weights are rounded once to fp16 (relative error <= 2^-11),
// activations are converted to fp16 exactly for bf16 input in fp16 range
// (|x| < 65520; larger magnitudes set status bit 2), products and sums are
// fp32.  Relative L2 error vs the reference's fp32 path is ~3e-4 for fp16
// weight rounding alone (acceptance bar 1e-3).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "hq4_common.cuh"
#include "hq4.h"

namespace hq4 {

int check_device_cap();
int* status_word();

constexpr int kGemmRows = 128;                          // MMA M
constexpr int kAWarps = 4;                              // dequant + epilogue
constexpr int kXWarps = 8;                              // activation conversion
constexpr int kMmaWarp = kAWarps + kXWarps;             // warp 12
constexpr int kGemmThreads = (kAWarps + kXWarps + 1) * 32;
constexpr int kAStageBytes = kGemmRows * 128;           // 128 rows x 64 fp16
constexpr int kWPre = 8;                                // packed k-blocks in flight per row
constexpr int kXPre = 2;                                // activation k-blocks in flight
constexpr uint64_t kGemmWaitNs = 1000000000ull;  // 1 s: a correct kernel never waits this long
constexpr int kMaxTileBf16 = 256, kMaxTileF32 = 128;
constexpr int kGemmSmemMax = 220 * 1024;

struct GemmParams {
    const uint32_t* w;
    const uint16_t* sc;
    const uint16_t* bi;
    const void* x;
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
__device__ __forceinline__ uint4 dequant_word(uint32_t w, __half2 s2, __half2 b2) {
    const __half2 k1024 = bits_h2(0x64006400u);
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t p = lop3_and_or(w >> (4 * j), 0x000F000Fu, 0x64006400u);
        o[j] = h2_bits(__hfma2(__hsub2(bits_h2(p), k1024), s2, b2));
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// 8 fp32 activations x0..x7 -> fp16 in the order x0,x4,x1,x5,x2,x6,x3,x7;
// amax tracks the largest magnitude seen (range check).
__device__ __forceinline__ uint4 pack_x8(const float (&f)[8], float& amax) {
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        amax = fmaxf(amax, fmaxf(fabsf(f[j]), fabsf(f[j + 4])));
        o[j] = h2_bits(__floats2half2_rn(f[j], f[j + 4]));  // low half = f[j]
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

template <bool XF32>
struct XChunk {
    uint32_t v[XF32 ? 8 : 4];
};

template <bool XF32>
__device__ __forceinline__ void load_x_chunk(const void* x, size_t elem, XChunk<XF32>& c) {
    if constexpr (XF32) {
        const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(x) + elem);
        const uint4 a = __ldg(p), b = __ldg(p + 1);
        c.v[0] = a.x; c.v[1] = a.y; c.v[2] = a.z; c.v[3] = a.w;
        c.v[4] = b.x; c.v[5] = b.y; c.v[6] = b.z; c.v[7] = b.w;
    } else {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(x) + elem));
        c.v[0] = a.x; c.v[1] = a.y; c.v[2] = a.z; c.v[3] = a.w;
    }
}

template <bool XF32>
__device__ __forceinline__ void chunk_floats(const XChunk<XF32>& c, float (&f)[8]) {
    if constexpr (XF32) {
#pragma unroll
        for (int j = 0; j < 8; j++) f[j] = __uint_as_float(c.v[j]);
    } else {
#pragma unroll
        for (int j = 0; j < 4; j++) {  // bf16 pair -> two fp32 (exact)
            f[2 * j] = __uint_as_float(c.v[j] << 16);
            f[2 * j + 1] = __uint_as_float(c.v[j] & 0xFFFF0000u);
        }
    }
}

template <bool XF32>
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
    const int tok0 = blockIdx.z * T;
    const int mt = min(T, p.m - tok0);
    const int kb0 = (int)((long long)kr * p.nkb / p.ks), kb1 = (int)((long long)(kr + 1) * p.nkb / p.ks);
    const int nk = kb1 - kb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(full_bar(s), kAWarps + kXWarps);
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
        // ---- dequantise weights: thread = row ------------------------------------
        const int r = warp * 32 + lane;
        const int grow = row0 + r;
        const bool rok = grow < p.n_out;
        const size_t wpr = (size_t)(p.n_in >> 3);
        const uint32_t* wrow = p.w + (size_t)(rok ? grow : 0) * wpr;
        const uint16_t* srow = p.sc + (size_t)(rok ? grow : 0) * p.n_sg;
        const uint16_t* brow = p.bi + (size_t)(rok ? grow : 0) * p.n_sg;
        uint32_t q[kWPre][8];
        uint32_t sb[kWPre];
        auto fetch = [&](int i, uint32_t (&qq)[8], uint32_t& sbv) {
            if (i < nk && rok) {
                const int kb = kb0 + i;
                ldg256_stream(wrow + (size_t)kb * 8, qq);
                const int g = kb >> p.gs_shift;
                sbv = (uint32_t)ldg_u16(srow + g) | ((uint32_t)ldg_u16(brow + g) << 16);
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) qq[j] = 0;
                sbv = 0;
            }
        };
#pragma unroll
        for (int d = 0; d < kWPre; d++) fetch(d, q[d], sb[d]);
        for (int ib = 0; ib < nk && !fail; ib += kWPre) {
#pragma unroll
            for (int d = 0; d < kWPre; d++) {
                const int i = ib + d;
                if (i < nk && !fail) {
                    const int s = i % S;
                    if (i >= S && !mbar_wait_ns(empty_bar(s), (uint32_t)((i / S) - 1) & 1u, kGemmWaitNs)) {
                        fail = true;
                    } else {
                        const __half2 s2 = __half2half2(__ushort_as_half((unsigned short)(sb[d] & 0xFFFFu)));
                        const __half2 b2 = __half2half2(__ushort_as_half((unsigned short)(sb[d] >> 16)));
                        unsigned char* dst = sm + (a_base - base) + (size_t)s * kAStageBytes;
#pragma unroll
                        for (int c = 0; c < 8; c++) {
                            const uint4 v = rok ? dequant_word(q[d][c], s2, b2) : make_uint4(0, 0, 0, 0);
                            *reinterpret_cast<uint4*>(dst + sw128_off(r, c)) = v;
                        }
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(full_bar(s));
                        fetch(i + kWPre, q[d], sb[d]);
                    }
                }
            }
        }
    } else if (warp < kMmaWarp) {
        // ---- activations -> fp16 B tile ----------------------------------------------
        pdl_wait();
        const int xi = threadIdx.x - kAWarps * 32;        // 0..255
        constexpr int kXThreads = kXWarps * 32;
        const int nchunks = T * 8;                        // (token, word) pairs per k-block
        constexpr int kMaxC = (XF32 ? kMaxTileF32 : kMaxTileBf16) * 8 / kXThreads;
        XChunk<XF32> xb[kXPre][kMaxC];
        float amax = 0.0f;
        auto fetch = [&](int i, XChunk<XF32> (&dst)[kMaxC]) {
#pragma unroll
            for (int j = 0; j < kMaxC; j++) {
                const int ch = xi + j * kXThreads;
                const int t = ch >> 3, c = ch & 7;
                if (i < nk && ch < nchunks && t < mt) {
                    const size_t elem = (size_t)(tok0 + t) * p.n_in + (size_t)(kb0 + i) * 64 + c * 8;
                    load_x_chunk<XF32>(p.x, elem, dst[j]);
                } else {
#pragma unroll
                    for (int u = 0; u < (XF32 ? 8 : 4); u++) dst[j].v[u] = 0;
                }
            }
        };
#pragma unroll
        for (int d = 0; d < kXPre; d++) fetch(d, xb[d]);
        for (int ib = 0; ib < nk && !fail; ib += kXPre) {
#pragma unroll
            for (int d = 0; d < kXPre; d++) {
                const int i = ib + d;
                if (i < nk && !fail) {
                    const int s = i % S;
                    if (i >= S && !mbar_wait_ns(empty_bar(s), (uint32_t)((i / S) - 1) & 1u, kGemmWaitNs)) {
                        fail = true;
                    } else {
                        unsigned char* dst = sm + (b_base - base) + (size_t)s * b_stage;
#pragma unroll
                        for (int j = 0; j < kMaxC; j++) {
                            const int ch = xi + j * kXThreads;
                            if (ch < nchunks) {
                                float f[8];
                                chunk_floats<XF32>(xb[d][j], f);
                                *reinterpret_cast<uint4*>(dst + sw128_off(ch >> 3, ch & 7)) = pack_x8(f, amax);
                            }
                        }
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(full_bar(s));
                        fetch(i + kXPre, xb[d]);
                    }
                }
            }
        }
        if (amax >= 65520.0f && p.status) atomicOr(p.status, 4);
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
    const bool epi = warp < kAWarps;
    const int r = warp * 32 + lane;
    const int grow = row0 + r;
    float* part = reinterpret_cast<float*>(sm);  // split-K partial tile [T][128], reuses the rings
    if (epi) {
        pdl_wait();
        const bool ok = mbar_wait_ns(accum_bar, 0, kGemmWaitNs);
        if (!ok && p.status) atomicOr(p.status, 1);
        __syncwarp();  // tcgen05.ld is warp-aligned
        tc_fence_after();
        const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
        for (int c0 = 0; c0 < T; c0 += 32) {
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
                    if (c0 + j < T) part[(c0 + j) * kGemmRows + r] = __uint_as_float(v[j]);
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

static GemmPlan plan_gemm(int n_out, int n_in, int m, bool xf32) {
    GemmPlan pl{};
    const int tmax = xf32 ? kMaxTileF32 : kMaxTileBf16;
    pl.n_tt = (m + tmax - 1) / tmax;
    const int per = (m + pl.n_tt - 1) / pl.n_tt;             // balance the token tiles
    pl.t_tile = std::min(tmax, (per + 15) / 16 * 16);
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
    return pl;
}

template <bool XF32>
static int launch_gemm(const GemmParams& prm, const GemmPlan& pl, cudaStream_t st) {
    // the shared-memory opt-in is a per-device function attribute
    static bool attr_done[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HQ4_ERR_LAUNCH;
    if (!attr_done[dev]) {
        if (cudaFuncSetAttribute(gemm_w4a16_kernel<XF32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kGemmSmemMax) != cudaSuccess)
            return HQ4_ERR_LAUNCH;
        attr_done[dev] = true;
    }
    // split-K partial tile [t_tile][128] fp32 lives in the (drained) rings
    if ((size_t)pl.t_tile * kGemmRows * 4 > (size_t)pl.stages * (kAStageBytes + pl.t_tile * 128) ||
        pl.smem > (size_t)kGemmSmemMax)
        return HQ4_ERR_SHAPE;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
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
    return cudaLaunchKernelEx(&lc, gemm_w4a16_kernel<XF32>, prm) == cudaSuccess ? HQ4_OK : HQ4_ERR_LAUNCH;
}

}  // namespace hq4

using namespace hq4;

extern "C" int hq4_gemm_w4a16(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, const void* x,
                              int x_is_f32, float* out, int n_out, int n_in, int gs, int m,
                              const float* row_add, const float* residual, void* stream) {
    if (int rc = check_device_cap()) return rc;
    if (n_out <= 0 || n_in <= 0 || m <= 0 || gs < 64 || gs % 64 || n_in % gs) return HQ4_ERR_SHAPE;
    if ((gs & (gs - 1)) != 0) return HQ4_ERR_SHAPE;
    if (((uintptr_t)w & 31) || ((uintptr_t)x & 15) || ((uintptr_t)out & 3) || ((uintptr_t)scales & 1) ||
        ((uintptr_t)biases & 1))
        return HQ4_ERR_ALIGN;
    const bool xf32 = x_is_f32 != 0;
    const GemmPlan pl = plan_gemm(n_out, n_in, m, xf32);
    GemmParams prm{};
    prm.w = w;
    prm.sc = scales;
    prm.bi = biases;
    prm.x = x;
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
    prm.status = status_word();
    if (!prm.status) return HQ4_ERR_LAUNCH;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return xf32 ? launch_gemm<true>(prm, pl, st) : launch_gemm<false>(prm, pl, st);
}

extern "C" int hq4_gemm_plan(int n_out, int n_in, int m, int x_is_f32, int* info) {
    if (n_out <= 0 || n_in <= 0 || m <= 0 || n_in % 64 || !info) return HQ4_ERR_SHAPE;
    const GemmPlan pl = plan_gemm(n_out, n_in, m, x_is_f32 != 0);
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
