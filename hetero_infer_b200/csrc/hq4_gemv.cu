// Fused int4 GEMV (decode, one token) and block dequantisation for sm_100a.
//
// Device-side replacement for the reference's q4_gemv / q4_dequant
// (hetero-infer kernel/q4gemv.c:232-301, 303-379).  Same packed layout, same
// per-group arithmetic:  y[o] = sum_g scale[o,g] * dot_g + bias[o,g] * xsum_g
// (kernel/q4gemv.c:15-17), with dot_g evaluated on the tensor cores.
//
// How one token's GEMV maps onto the hardware
// -------------------------------------------
// * A warp works on "tiles" of 16 output rows x 4 lane-groups (KG = 64 or 32
//   values of K each).  Lane (g = lane/4, t = lane%4) owns lane-group t of the
//   tile for rows g and g+8 and fetches those two group-rows (KG/2 bytes each)
//   with one 256-bit (or 128-bit) load each: the weight stream is fully
//   coalesced, one instruction per group-row.
// * Nibbles become u8 with three instructions per packed word (mask, shift,
//   mask) and are the A operand of the integer tensor-core MMA
//   mma.sync m16n8k32 (u8 x s8 -> s32).  Lane t feeds only its own group's k
//   positions, so one k-step mixes four groups.
// * The B operand holds x as a per-group fixed-point integer: with
//   2^(E-1) <= max|x_group| < 2^E, v = rint(x * 2^(22-E)) has 22 bits plus
//   sign and is split into three balanced s8 digits (v = d2*2^16 + d1*2^8 +
//   d0).  Columns 2t / 2t+1 of n-tile 0 carry d2 / d1 of lane-group t and
//   column 2t of n-tile 1 carries d0, zero elsewhere, so the C registers lane
//   t holds end the tile as the three exact integer digit-dots of its own
//   group for rows g and g+8.
// * The epilogue per group is fp32: dot = (C2*2^16 + C1*2^8 + C0) * 2^(E-22),
//   acc += scale * dot + bias * xsum, with xsum the group's fp32 sum of x
//   (kernel/q4gemv.c:244-248).  x is thereby represented to 2^-22 of its group
//   maximum and every product and integer sum is exact: the result agrees with
//   the reference float path to fp32 rounding.
// * Work split: every CTA owns a contiguous run of whole 16-row strips
//   (balanced to one strip); inside the CTA the (strip, tile) units are split
//   evenly and contiguously over its 8 warps.  A strip cut between two warps
//   is reduced through shared memory by the warp holding its last piece,
//   summing the pieces in warp order: deterministic, and no global scratch,
//   atomics or fences.
// * The first D tiles of weights are requested before griddepcontrol.wait,
//   so with programmatic dependent launch the weight stream starts while the
//   producer of x is still draining.
#include <algorithm>
#include <cstdio>
#include <functional>
#include <mutex>
#include <unordered_map>

#include "hq4_common.cuh"
#include "hq4_gemv_dev.cuh"
#include "hq4_host.cuh"
#include "hq4_mt.cuh"
#include "hq4_tmap.cuh"
#include "hq4.h"

namespace hq4 {

constexpr int kGemvThreads = 256;  // 8 warps
constexpr int kGemvWarps = kGemvThreads / kWarp;
constexpr int kPrefetch = 3;       // tiles of weights in flight per warp


// Shared memory: [ng x kImgStride x image][zero block 64 B]
//                [kGemvWarps x 2 x 16 floats: split-strip partials]
//                [mbarrier: x row][raw x row, fp32, when n_in <= 8192]
__host__ __device__ __forceinline__ size_t zero_block_offset(int ng, int stride) {
    return (size_t)ng * stride;
}
__host__ __device__ __forceinline__ size_t partial_offset(int ng, int stride) {
    return zero_block_offset(ng, stride) + 64;
}
__host__ __device__ __forceinline__ size_t mbar_offset(int ng, int stride) {
    return partial_offset(ng, stride) + (size_t)kGemvWarps * 2 * 16 * sizeof(float);
}
__host__ __device__ __forceinline__ size_t rawx_offset(int ng, int stride) {
    return mbar_offset(ng, stride) + 16;
}
constexpr int kMbarWaitIters = 1 << 22;  // bounded wait on the x-row bulk copy
constexpr int kRawXMax = 32 * 1024;      // x rows up to 8192 fp32 go through smem

// Sum a strip's lane partials across the 4 lanes t; store it when this warp
// owns the whole strip, else park it in the warp's head/tail smem slot.
__device__ __forceinline__ void flush_strip(const GemvM1Params& p, int s, bool full, float* slot,
                                            float acc0, float acc1, int lane) {
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    const int g = lane >> 2, t = lane & 3;
    if (t != 0) return;
    if (full) {
        store_pair(p, s, g, acc0, acc1);
    } else {
        slot[g] = acc0;
        slot[g + 8] = acc1;
    }
}

// x image: for every lane-group, three s8 digit blocks (d2, d1, d0) of KG
// bytes, each in k-step order with the values of a packed word permuted as
// the u8 unpack produces them ({0,2,4,6} then {1,3,5,7}), followed by
// (2^(E-22), xsum).  This builds lane-groups [g_lo, g_hi) only, from the fp32
// values of those groups already in shared memory (xs); the CTAs of a cluster
// each build one slice and exchange them.
template <int KG>
__device__ __forceinline__ void build_x_slice(const float* xs, int g_lo, int g_hi,
                                              unsigned char* img, float norm_r,
                                              const float* __restrict__ norm_w) {
    using C = M1<KG>;
    constexpr int kPer = KG / 4;  // values per thread: 4 threads per lane-group
    const int ntask = (g_hi - g_lo) * 4;
    for (int base = 0; base < ntask; base += kGemvThreads) {
        const int task = base + threadIdx.x;
        const bool ok = task < ntask;
        const int G = g_lo + (task >> 2), qq = task & 3;
        float v[kPer];
        if (ok) {
            const float4* xp = reinterpret_cast<const float4*>(xs + (size_t)(G - g_lo) * KG + qq * kPer);
#pragma unroll
            for (int i = 0; i < kPer / 4; i++) {
                float4 f = xp[i];
                v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < kPer; i++) v[i] = 0.0f;
        }
        if (norm_w && ok) {
            // hetero/cpu_model.py:164-166: (x * (1/sqrt(mean(x^2)+eps))) * w
            const float4* wp = reinterpret_cast<const float4*>(norm_w + (size_t)G * KG + qq * kPer);
#pragma unroll
            for (int i = 0; i < kPer / 4; i++) {
                const float4 nw = wp[i];
                v[4 * i] = __fmul_rn(__fmul_rn(v[4 * i], norm_r), nw.x);
                v[4 * i + 1] = __fmul_rn(__fmul_rn(v[4 * i + 1], norm_r), nw.y);
                v[4 * i + 2] = __fmul_rn(__fmul_rn(v[4 * i + 2], norm_r), nw.z);
                v[4 * i + 3] = __fmul_rn(__fmul_rn(v[4 * i + 3], norm_r), nw.w);
            }
        }
        float amax = 0.0f, s = 0.0f;
#pragma unroll
        for (int i = 0; i < kPer; i++) {
            amax = fmaxf(amax, fabsf(v[i]));
            s += v[i];
        }
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        const int E = group_exponent(amax);
        const float up = exp2i(kXBits - E);
        if (ok) {
            unsigned char* gbase = img + (size_t)G * C::kImgStride;
#pragma unroll
            for (int j = 0; j < kPer / 8; j++) {
                const int word = qq * (kPer / 8) + j;
                uint32_t r[8];
#pragma unroll
                for (int k = 0; k < 8; k++) r[k] = digits3(v[8 * j + k], up);
                // even values {0,2,4,6} then odd {1,3,5,7}; byte k of r = digit k
                const uint32_t e01 = prmt(prmt(r[0], r[2], 0x5140), prmt(r[4], r[6], 0x5140), 0x5410);
                const uint32_t e11 = prmt(prmt(r[0], r[2], 0x5140), prmt(r[4], r[6], 0x5140), 0x7632);
                const uint32_t e21 = prmt(prmt(r[0], r[2], 0x0062), prmt(r[4], r[6], 0x0062), 0x5410);
                const uint32_t o01 = prmt(prmt(r[1], r[3], 0x5140), prmt(r[5], r[7], 0x5140), 0x5410);
                const uint32_t o11 = prmt(prmt(r[1], r[3], 0x5140), prmt(r[5], r[7], 0x5140), 0x7632);
                const uint32_t o21 = prmt(prmt(r[1], r[3], 0x0062), prmt(r[5], r[7], 0x0062), 0x5410);
                *reinterpret_cast<uint2*>(gbase + 0 * KG + word * 8) = make_uint2(e21, o21);
                *reinterpret_cast<uint2*>(gbase + 1 * KG + word * 8) = make_uint2(e11, o11);
                *reinterpret_cast<uint2*>(gbase + 2 * KG + word * 8) = make_uint2(e01, o01);
            }
            if (qq == 0)
                *reinterpret_cast<float2*>(gbase + C::kMetaOff) = make_float2(exp2i(E - kXBits), s);
        }
    }
}

template <int KG>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_m1_kernel(const GemvM1Params p) {
    using C = M1<KG>;
    constexpr int D = kPrefetch;
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* img = smem;
    const uint32_t bar_x = smem_u32(smem + mbar_offset(p.ng, C::kImgStride));  // x row arrival
    // rows short enough get the x row through one bulk copy into shared memory
    const bool x_via_smem = p.n_in * (int)sizeof(float) <= kRawXMax;
    float* rawx = reinterpret_cast<float*>(smem + rawx_offset(p.ng, C::kImgStride));
    if (threadIdx.x == 0) mbar_init(bar_x, 1);

    pdl_launch_dependents();

    const int lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int wj = threadIdx.x >> 5;
    // this CTA's strips, and this warp's contiguous share of their units
    const int s0 = (int)(blockIdx.x * (uint32_t)p.n_strips / gridDim.x);
    const int s1 = (int)((blockIdx.x + 1) * (uint32_t)p.n_strips / gridDim.x);
    const int cu0 = s0 * p.nq, nunits = (s1 - s0) * p.nq;
    const int wa = nunits < kGemvWarps ? nunits : kGemvWarps;  // warps with work
    const int u0 = wj < wa ? cu0 + wj * nunits / wa : cu0 + nunits;
    const int u1 = wj < wa ? cu0 + (wj + 1) * nunits / wa : cu0 + nunits;
    const size_t wpr = (size_t)(p.n_in >> 3);
    float* partials = reinterpret_cast<float*>(smem + partial_offset(p.ng, C::kImgStride));

    uint32_t wv[D][2][C::kWords];
    uint32_t sv[D][4];

    // load cursor: strip ls, tile lq; lp points at this lane's row-g group-row
    int ls = u0 / p.nq, lq = u0 - ls * p.nq;
    const uint32_t* lp = p.w + (size_t)(ls * 16 + g) * wpr + (size_t)(lq * 4 + t) * C::kWords;
    auto issue = [&](uint32_t (&wr)[2][C::kWords], uint32_t (&sr)[4], bool live) {
        const int r0 = ls * 16 + g;
        const int G = lq * 4 + t;
        const bool gok = live && G < p.ng;
        const bool ok0 = gok && r0 < p.n_out, ok1 = gok && r0 + 8 < p.n_out;
        if constexpr (C::kWords == 8) {
            if (ok0) ldg256_stream(lp, wr[0]);
            else
#pragma unroll
                for (int i = 0; i < 8; i++) wr[0][i] = 0u;
            if (ok1) ldg256_stream(lp + 8 * wpr, wr[1]);
            else
#pragma unroll
                for (int i = 0; i < 8; i++) wr[1][i] = 0u;
        } else {
            if (ok0) ldg128_stream(lp, wr[0]);
            else
#pragma unroll
                for (int i = 0; i < 4; i++) wr[0][i] = 0u;
            if (ok1) ldg128_stream(lp + 8 * wpr, wr[1]);
            else
#pragma unroll
                for (int i = 0; i < 4; i++) wr[1][i] = 0u;
        }
        const size_t si = (size_t)r0 * p.n_sg + (G >> p.sg_shift);
        sr[0] = ok0 ? ldg_u16(p.sc + si) : 0u;
        sr[1] = ok0 ? ldg_u16(p.bi + si) : 0u;
        sr[2] = ok1 ? ldg_u16(p.sc + si + (size_t)8 * p.n_sg) : 0u;
        sr[3] = ok1 ? ldg_u16(p.bi + si + (size_t)8 * p.n_sg) : 0u;
        if (live) {
            lp += 4 * C::kWords;
            if (++lq == p.nq) {
                lq = 0;
                ++ls;
                lp = p.w + (size_t)(ls * 16 + g) * wpr + (size_t)t * C::kWords;
            }
        }
    };

    __syncthreads();  // mbarrier initialisation visible to every thread
    if (p.weights_after_wait) pdl_wait();
#pragma unroll
    for (int d = 0; d < D; d++) issue(wv[d], sv[d], u0 + d < u1);

    // x (needs the producer of x).  Short rows: one bulk copy into shared
    // memory (the copy engine, not the load pipeline already holding the
    // weight prefetch); long rows are read from global memory directly.
    pdl_wait();
    bool ok = true;
    if (x_via_smem) {
        const uint32_t x_bytes = (uint32_t)(p.n_in * sizeof(float));
        if (threadIdx.x == 0) {
            mbar_arrive_expect_tx(bar_x, x_bytes);
            bulk_load_g2s(smem_u32(rawx), p.x, x_bytes, bar_x, l2_policy_evict_last());
        }
        ok = mbar_wait(bar_x, 0, kMbarWaitIters);
    }
    const float* xsrc = x_via_smem ? rawx : p.x;
    float norm_r = 1.0f;
    if (p.norm_w) {
        // sum of squares of the whole row: CTA reduction
        __shared__ float red[kGemvWarps];
        float ss = 0.0f;
        if (ok)
            for (int i = threadIdx.x; i < p.n_in; i += kGemvThreads) ss = fmaf(xsrc[i], xsrc[i], ss);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
        __syncthreads();
        float tot = 0.0f;
#pragma unroll
        for (int i = 0; i < kGemvWarps; i++) tot += red[i];
        const float mean = __fdiv_rn(tot, (float)p.n_in);
        norm_r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
    }
    if (ok) build_x_slice<KG>(xsrc, 0, p.ng, img, norm_r, p.norm_w);
    {
        uint4* z = reinterpret_cast<uint4*>(smem + zero_block_offset(p.ng, C::kImgStride));
        if (threadIdx.x < 4) z[threadIdx.x] = make_uint4(0, 0, 0, 0);
    }
    if (!__syncthreads_and(ok)) {  // uniform: every thread leaves together
        if (threadIdx.x == 0 && p.status) atomicOr(p.status, 1);
        return;
    }

    // B operand: lanes g == 2t read digits d2 (n-tile 0) and d0 (n-tile 1) of
    // their lane-group, lanes g == 2t+1 read d1 (n-tile 0); every other slot
    // reads the shared zero block (a broadcast), so no lane branches.
    const int role = (g >> 1) == t ? (g & 1) + 1 : 0;  // 1: d2+d0, 2: d1, 0: none
    const unsigned char* zero_blk = smem + zero_block_offset(p.ng, C::kImgStride);
    const int off0 = role == 1 ? 0 : KG;      // d2 or d1
    const int off1 = 2 * KG;                  // d0

    int cs = u0 / p.nq, cq = u0 - cs * p.nq;
    float acc0 = 0.0f, acc1 = 0.0f;
    for (int ub = u0; ub < u1; ub += D) {
#pragma unroll
        for (int d = 0; d < D; d++) {
            const int u = ub + d;
            if (u >= u1) break;
            const int G = cq * 4 + t;
            const bool gok = G < p.ng;
            const unsigned char* gb = img + (size_t)(gok ? G : p.ng - 1) * C::kImgStride;
            const uint4* src0 = reinterpret_cast<const uint4*>(role ? gb + off0 : zero_blk);
            const uint4* src1 = reinterpret_cast<const uint4*>(role == 1 ? gb + off1 : zero_blk);
            int c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
            uint4 q0 = make_uint4(0, 0, 0, 0), q1 = q0;
#pragma unroll
            for (int ks = 0; ks < C::kKSteps; ks++) {
                if ((ks & 1) == 0) {
                    q0 = src0[ks >> 1];
                    q1 = src1[ks >> 1];
                }
                const uint32_t b00 = (ks & 1) ? q0.z : q0.x, b01 = (ks & 1) ? q0.w : q0.y;
                const uint32_t b10 = (ks & 1) ? q1.z : q1.x, b11 = (ks & 1) ? q1.w : q1.y;
                uint32_t a0, a1, a2, a3;
                unpack_u8(wv[d][0][ks], a0, a2);
                unpack_u8(wv[d][1][ks], a1, a3);
                mma_u8s8_16832(c0, a0, a1, a2, a3, b00, b01);
                mma_u8s8_16832(c1, a0, a1, a2, a3, b10, b11);
            }
            if (gok) {
                const float2 m = *reinterpret_cast<const float2*>(gb + C::kMetaOff);
                const float dot0 = fmaf((float)c0[0], 65536.0f, fmaf((float)c0[1], 256.0f, (float)c1[0]));
                const float dot1 = fmaf((float)c0[2], 65536.0f, fmaf((float)c0[3], 256.0f, (float)c1[2]));
                acc0 = fmaf(h2f(sv[d][0]) * m.x, dot0, acc0);
                acc0 = fmaf(h2f(sv[d][1]), m.y, acc0);
                acc1 = fmaf(h2f(sv[d][2]) * m.x, dot1, acc1);
                acc1 = fmaf(h2f(sv[d][3]), m.y, acc1);
            }
            // refill this stage with the tile D ahead
            issue(wv[d], sv[d], u + D < u1);
            if (++cq == p.nq) {
                const bool head = cs * p.nq < u0;  // started before this warp's range
                flush_strip(p, cs, !head, partials + (wj * 2 + (head ? 0 : 1)) * 16, acc0, acc1, lane);
                acc0 = acc1 = 0.0f;
                cq = 0;
                ++cs;
            }
        }
    }
    if (cq != 0) {  // range ends inside a strip: slot 0 if it also began in it
        const int slot = cs * p.nq <= u0 ? 0 : 1;
        flush_strip(p, cs, false, partials + (wj * 2 + slot) * 16, acc0, acc1, lane);
    }
    // split strips: the warp holding a strip's last piece sums the pieces in
    // warp order
    __syncthreads();
    if (u0 < u1) {
        const int sf = u0 / p.nq;  // first strip of this warp
        const int first_unit = sf * p.nq, last_unit = first_unit + p.nq - 1;
        auto warp_of = [&](int u) {  // warp whose (nonempty) range holds unit u
            return (int)(((long long)(u - cu0 + 1) * wa - 1) / nunits);
        };
        const int wf = warp_of(first_unit), wl = warp_of(last_unit);
        if (wf != wl && wl == wj && t == 0) {
            float y0 = 0.0f, y1 = 0.0f;
            for (int k = wf; k <= wl; k++) {
                const int k_first_strip = (cu0 + (int)((long long)k * nunits / wa)) / p.nq;
                const float* sl = partials + (k * 2 + (k_first_strip == sf ? 0 : 1)) * 16;
                y0 += sl[g];
                y1 += sl[g + 8];
            }
            store_pair(p, sf, g, y0, y1);
        }
    }
}

// ---- streaming GEMV: the weights through a TMA ring ------------------------
// The register-prefetch kernel above can hold only a few tiles of weights in
// flight per warp, and it cannot request more until x has arrived and its
// image has been built.  At each kernel boundary the DRAM therefore idles
// while x is fetched and converted.  This kernel decouples the two:
// * one producer thread streams the CTA's strips through a ring of shared-
//   memory stages with TMA (cp.async.bulk.tensor, 128-byte swizzle; the
//   packed words as a 3D view so one copy brings a whole stage).  It
//   issues the first stages before griddepcontrol.wait, and since a CTA takes
//   under half an SM, the next kernel's CTA fills its ring while this one
//   drains;
// * a stage is one 16-row strip x 8 k-chunks of 256 values (16 KB of packed
//   weights plus its scales and biases).  Consumer warp w takes k-chunk w of
//   every stage.  It therefore needs the x image only of its own k-chunks: it
//   builds them itself, one chunk at a time, just before use (no CTA-wide
//   image phase).  Stages run k-block-major, strip-minor, so one chunk image
//   serves every strip of the CTA;
// * per stage a warp adds its tile's per-row sums into its own shared-memory
//   slot; at the end the 8 warps' slots are summed in warp order
//   (deterministic, no atomics, no global scratch) and stored through the
//   same epilogue as the kernel above.
// Arithmetic per group is the kernel above's: exact digit dots on the
// integer tensor cores, fp32 scale, bias and sums.

struct StreamLayout {
    int ring, ns_max, nkb;  // nkb: k-blocks per strip = chunk images per warp
    __host__ __device__ size_t img_off() const { return (size_t)ring * kStrStageBytes; }
    __host__ __device__ size_t zero_off() const {
        return img_off() + (size_t)kStrConsumers * nkb * kStrImgBytes;
    }
    __host__ __device__ size_t part_off() const { return zero_off() + 64; }
    __host__ __device__ size_t red_off() const {
        return part_off() + (size_t)kStrConsumers * ns_max * 16 * sizeof(float);
    }
    __host__ __device__ size_t bar_off() const { return red_off() + kStrConsumers * sizeof(float); }
    // full[ring], empty[ring], images built
    __host__ __device__ size_t bytes() const { return bar_off() + (size_t)(2 * ring + 1) * 8 + 1024; }
};

// Stages a CTA requests before the dependency wait.  The rest of the ring
// follows once the consumers have built their x images: the x loads then
// meet fewer weight copies in flight (they wait behind them in the memory
// system), which measured faster than filling the whole ring up front.
constexpr int kStrEarlyStages = 3;


__global__ void __launch_bounds__(kStrThreads, 1)
gemv_stream_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s,
                   const __grid_constant__ CUtensorMap tm_b, const GemvM1Params p, const StreamLayout L) {
    extern __shared__ unsigned char smem_raw[];
    // stages need 1024-byte alignment (the 128-byte swizzle repeats every 8 rows)
    const uint32_t raw_u = smem_u32(smem_raw);
    unsigned char* base = smem_raw + (((raw_u + 1023u) & ~1023u) - raw_u);
    const uint32_t base_u = smem_u32(base);
    const int R = L.ring;
    float* partials = reinterpret_cast<float*>(base + L.part_off());
    float* red = reinterpret_cast<float*>(base + L.red_off());
    const uint32_t bars = base_u + (uint32_t)L.bar_off();
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (R + s); };
    const uint32_t images_bar = bars + 8u * (2 * R);  // every consumer warp's x images are built

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int s0, ns;
    str_strips((int)blockIdx.x, p.n_strips, (int)gridDim.x, s0, ns);
    const int nk = (p.ng + 3) >> 2;              // k-chunks of 4 lane-groups
    const int nkb = (nk + kStrKc - 1) / kStrKc;  // stages per strip
    const int n_stages = nkb * ns;
    const int sb_cols = kStrSBCols >> p.sg_shift;  // scale groups per stage
    const uint32_t sb_bytes = 16u * sb_cols * 2u;

    // ---- producer (warp 16, one thread): it sets up the barriers and issues
    // the first stages before the CTA-wide barrier, so the first copies leave
    // as early as possible; it issues every copy, stages in order
    const bool producer = warp == kStrConsumers && lane == 0;
    int p_issued = 0, p_slot = 0, p_use = 0, p_kb = 0, p_jj = 0;
    uint64_t pol = 0;
    auto issue_stage = [&]() {
        const int strip = s0 + p_jj;
        const int kc0 = p_kb * kStrKc;
        const uint32_t dst = base_u + (uint32_t)p_slot * kStrStageBytes;
        // one copy of the stage's k-chunks x 16 rows (chunks past the row end read as zeros)
        mbar_arrive_expect_tx(full_bar(p_slot), (uint32_t)kStrWBytes + 2u * sb_bytes);
        tma_load_3d(dst, &tm_w, 0, strip * 16, kc0, full_bar(p_slot), pol);
        const int gx = (kc0 * 4) >> p.sg_shift;
        tma_load_2d(dst + kStrWBytes, &tm_s, gx, strip * 16, full_bar(p_slot), pol);
        tma_load_2d(dst + kStrWBytes + kStrSBBytes, &tm_b, gx, strip * 16, full_bar(p_slot), pol);
        p_issued++;
        if (++p_slot == R) {
            p_slot = 0;
            p_use++;
        }
        if (++p_jj == ns) {
            p_jj = 0;
            p_kb++;
        }
    };
    if (producer) {
        prefetch_tensormap(&tm_w);
        prefetch_tensormap(&tm_s);
        prefetch_tensormap(&tm_b);
        for (int s = 0; s < R; s++) {
            mbar_init_nofence(full_bar(s), 1);
            mbar_init_nofence(empty_bar(s), kStrConsumers);
        }
        mbar_init_nofence(images_bar, kStrConsumers);
        mbar_init_fence();
        pol = l2_policy_evict_first();  // weights are read once
        if (p.weights_after_wait) pdl_wait();
        const int first = min(min(R, kStrEarlyStages), n_stages);
        for (int i = 0; i < first; i++) issue_stage();
    }
    if (threadIdx.x < 4) reinterpret_cast<uint4*>(base + L.zero_off())[threadIdx.x] = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < kStrConsumers * L.ns_max * 16; i += kStrThreads) partials[i] = 0.0f;
    __syncthreads();  // barriers initialised, zero block and partial slots cleared
    pdl_launch_dependents();

    if (warp == kStrConsumers) {
        if (producer) {
            bool ok = true;
            if (p_issued < n_stages) {
                pdl_wait();  // the waits below depend on the consumers
                ok = mbar_wait_nap(images_bar, 0, kStrWaitNs, 64);
            }
            while (ok && p_issued < n_stages) {
                if (!mbar_wait_nap(empty_bar(p_slot), (p_use - 1) & 1, kStrWaitNs, 64)) {
                    ok = false;
                    break;
                }
                issue_stage();
            }
            if (!ok && p.status) atomicOr(p.status, 1);
            // every issued copy lands before the CTA may exit; the last use of
            // each slot is its final phase, so its parity cannot alias
            for (int k = max(0, p_issued - R); k < p_issued; k++)
                if (!mbar_wait_nap(full_bar(k % R), (k / R) & 1, kStrWaitNs, 64) && p.status) atomicOr(p.status, 1);
        }
        return;
    }

    // ---- consumers (warps 0-15; threadIdx.x in [0, 512))
    pdl_wait();  // x, norm_w, residual and the outputs follow the previous kernel
    const int epi_pos = str_epi_prefetch(p, ns, s0, warp, lane);
    // this warp's chunk images, one per k-block, built up front: the builds
    // overlap the ring filling, and the stage loop is tiles only
    unsigned char* img_w = base + L.img_off() + (size_t)warp * L.nkb * kStrImgBytes;
    str_prologue<5, 2>(p, red, img_w, nkb, nk, warp, lane);
    if (lane == 0) mbar_arrive(images_bar);
    str_epi_prefetch_late(p, ns, s0, warp, lane, epi_pos);
    bool ok = true;
    int slot = 0;
    uint32_t phase = 0;
    StrAcc acc = {0.0f, 0.0f, 0.0f, 0.0f};
    str_consume<true>(p, base, full_bar(0), empty_bar(0), R, slot, phase, ok, ns, nkb, nk, img_w, base + L.zero_off(),
                partials, L.ns_max, warp, lane, acc);
    if (!ok && lane == 0 && p.status) atomicOr(p.status, 1);
    str_finish(p, partials, ns, L.ns_max, s0, ok, acc, warp, lane);
}

// ---- block dequantisation ------------------------------------------------
// One thread per packed word; out rows are relative to row0.
__global__ void dequant_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ sc,
                               const uint16_t* __restrict__ bi, float* __restrict__ out, int row0,
                               int rows, int n_in, int gs) {
    pdl_launch_dependents();
    pdl_wait();
    const int wpr = n_in >> 3, n_sg = n_in / gs;
    const long long total = (long long)rows * wpr;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int rr = (int)(i / wpr), k = (int)(i - (long long)rr * wpr);
        const int r = row0 + rr;
        const uint32_t q = w[(size_t)r * wpr + k];
        const int si = (k * 8) / gs;
        const float s = h2f(sc[(size_t)r * n_sg + si]);
        const float b = h2f(bi[(size_t)r * n_sg + si]);
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; j++) o[j] = __fadd_rn(__fmul_rn((float)((q >> (4 * j)) & 0xFu), s), b);
        float4* dst = reinterpret_cast<float4*>(out + (size_t)rr * n_in + (size_t)k * 8);
        dst[0] = make_float4(o[0], o[1], o[2], o[3]);
        dst[1] = make_float4(o[4], o[5], o[6], o[7]);
    }
}

// ---- host side -------------------------------------------------------------
struct GemvPlan {
    int kg, sg_shift, ng, n_sg, n_strips, nq, grid, cluster;  // cluster: always 1 here
    size_t smem;
};

// Device status word: bit 0 = a bounded wait in a kernel ran out, bit 1 = a
// token id outside the embedding table (the row was written as zeros).
__device__ int g_hq4_status = 0;

static int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    return n;
}

// Device address of g_hq4_status, looked up once per device.
int* status_word() {
    static PerDeviceOnce once;
    static int* addr[kMaxDevices] = {nullptr};
    const cudaError_t e = once.run([&](int d) {
        int* a = nullptr;
        const cudaError_t r = cudaGetSymbolAddress(reinterpret_cast<void**>(&a), g_hq4_status);
        if (r != cudaSuccess) {
            (void)cudaGetLastError();
            return r;
        }
        addr[d] = a;
        return cudaSuccess;
    });
    int dev = 0;
    if (e != cudaSuccess || cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    return addr[dev];
}

static int log2_exact(int v) {
    int s = 0;
    while ((1 << s) < v) s++;
    return (1 << s) == v ? s : -1;
}

// Returns 0 and fills the plan, or HQ4_ERR_SHAPE.
static int plan_gemv(int n_out, int n_in, int gs, GemvPlan& pl) {
    if (n_out <= 0 || n_in <= 0 || gs <= 0 || n_in % gs) return HQ4_ERR_SHAPE;
    if (gs == 32) {
        pl.kg = 32;
        pl.sg_shift = 0;
    } else if (gs % 64 == 0 && log2_exact(gs / 64) >= 0) {
        pl.kg = 64;
        pl.sg_shift = log2_exact(gs / 64);
    } else {
        return HQ4_ERR_SHAPE;
    }
    pl.ng = n_in / pl.kg;
    pl.n_sg = n_in / gs;
    pl.n_strips = (n_out + 15) / 16;
    pl.nq = (pl.ng + 3) / 4;
    if ((long long)pl.n_strips * pl.nq > (1LL << 30)) return HQ4_ERR_SHAPE;
    const int stride = pl.kg == 64 ? M1<64>::kImgStride : M1<32>::kImgStride;
    // whole strips per CTA; enough of them that each warp gets a unit
    const int min_strips = (kGemvWarps + pl.nq - 1) / pl.nq;
    pl.cluster = 1;
    const size_t rawx = (size_t)n_in * sizeof(float) <= (size_t)kRawXMax ? (size_t)n_in * sizeof(float) : 0;
    pl.smem = rawx_offset(pl.ng, stride) + rawx;
    if (pl.smem > 220 * 1024) return HQ4_ERR_SHAPE;  // x image must fit one CTA
    const int ctas_per_sm = pl.smem <= 110 * 1024 ? 2 : 1;
    const int max_grid = sm_count() * ctas_per_sm;
    pl.grid = std::max(1, std::min(max_grid, pl.n_strips / min_strips));
    return HQ4_OK;
}

// HQ4_OK when the current device is an sm_100 part (checked once per device).
static int check_device() {
    static PerDeviceOnce once;
    static bool is_sm100[kMaxDevices] = {false};
    const cudaError_t e = once.run([&](int d) {
        int major = 0;
        const cudaError_t r = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d);
        if (r != cudaSuccess) return r;
        is_sm100[d] = major == 10;
        return cudaSuccess;
    });
    int dev = 0;
    if (e != cudaSuccess || cudaGetDevice(&dev) != cudaSuccess) return HQ4_ERR_DEVICE;
    return is_sm100[dev] ? HQ4_OK : HQ4_ERR_DEVICE;
}

template <int KG>
static int launch_m1(const GemvPlan& pl, const GemvM1Params& prm, cudaStream_t st) {
    auto kern = gemv_m1_kernel<KG>;
    static PerDeviceOnce attr_once;
    if (smem_opt_in(attr_once, kern, 220 * 1024) != cudaSuccess) return HQ4_ERR_LAUNCH;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(pl.grid);
    lc.blockDim = dim3(kGemvThreads);
    lc.dynamicSmemBytes = pl.smem;
    lc.stream = st;
    lc.attrs = attr;
    lc.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&lc, kern, prm);
    return e == cudaSuccess ? HQ4_OK : HQ4_ERR_LAUNCH;
}

// ---- streaming kernel: tensor maps, plan, launch
// One CTA per SM: the ring takes what the SM's shared memory leaves.
constexpr size_t kStrSmemTarget = 220 * 1024;
constexpr int kStrMaxRing = 5;

struct StreamKey {
    const void* w;
    const void* s;
    const void* b;
    int n_out, n_in, sg_cols, dev;
    bool operator==(const StreamKey& o) const {
        return w == o.w && s == o.s && b == o.b && n_out == o.n_out && n_in == o.n_in && sg_cols == o.sg_cols &&
               dev == o.dev;
    }
};
struct StreamKeyHash {
    size_t operator()(const StreamKey& k) const {
        size_t h = std::hash<const void*>()(k.w);
        h = h * 1000003u ^ std::hash<const void*>()(k.s);
        h = h * 1000003u ^ std::hash<const void*>()(k.b);
        h = h * 1000003u ^ (size_t)k.n_out * 31u ^ (size_t)k.n_in * 131u ^ (size_t)k.sg_cols ^ ((size_t)k.dev << 40);
        return h;
    }
};
struct StreamMaps {
    CUtensorMap tw, ts, tb;
};

// The three maps of a weight matrix (packed words: 16 rows x 8 k-chunks of
// 32 words, 128-byte swizzle; scales and biases: sg_cols x 16-row boxes), cached by
// (pointers, shape, device).  False if the driver cannot encode them.
static bool stream_maps(const GemvM1Params& p, int n_sg, int sg_cols, StreamMaps* out) {
    static std::mutex mu;
    static std::unordered_map<StreamKey, StreamMaps, StreamKeyHash> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    const StreamKey key{p.w, p.sc, p.bi, p.n_out, p.n_in, sg_cols, dev};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return true;
    }
    StreamMaps m;
    if (!make_map_chunks(&m.tw, p.w, p.n_out, p.n_in / 8, 16, kStrKc) ||
        !make_map_2d_sw(&m.ts, p.sc, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, p.n_out, n_sg, sg_cols, 16, sb_swizzle(sg_cols)) ||
        !make_map_2d_sw(&m.tb, p.bi, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, p.n_out, n_sg, sg_cols, 16, sb_swizzle(sg_cols)))
        return false;
    if (cache.size() >= 4096) cache.clear();
    cache.emplace(key, m);
    *out = m;
    return true;
}

// Launch the streaming kernel when the shape suits it (lane-groups of 64,
// scale groups of 64..256 whose rows are whole 16-byte units, 16-byte aligned
// scales and biases); *used says whether it was launched.
static int launch_stream(const GemvPlan& pl, const GemvM1Params& prm, cudaStream_t st, bool* used) {
    *used = false;
    if (pl.kg != 64 || pl.sg_shift > 2 || pl.n_sg % 8 || (((uintptr_t)prm.sc | (uintptr_t)prm.bi) & 15))
        return HQ4_OK;
    const int grid = std::min(pl.n_strips, sm_count());
    StreamLayout L;
    L.ns_max = (pl.n_strips + grid - 1) / grid;
    L.nkb = (pl.ng / 4 + kStrKc - 1) / kStrKc;
    L.ring = kStrMaxRing;
    while (L.ring > 3 && L.bytes() > kStrSmemTarget) L.ring--;
    if (L.bytes() > kStrSmemTarget) return HQ4_OK;  // rows too long for the chunk images: register kernel
    StreamMaps m;
    if (!stream_maps(prm, pl.n_sg, kStrSBCols >> pl.sg_shift, &m)) return HQ4_OK;
    static PerDeviceOnce attr_once;
    if (smem_opt_in(attr_once, gemv_stream_kernel, 220 * 1024) != cudaSuccess) return HQ4_ERR_LAUNCH;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(grid);
    lc.blockDim = dim3(kStrThreads);
    lc.dynamicSmemBytes = L.bytes();
    lc.stream = st;
    lc.attrs = attr;
    lc.numAttrs = 1;
    *used = true;
    const cudaError_t e = cudaLaunchKernelEx(&lc, gemv_stream_kernel, m.tw, m.ts, m.tb, prm, L);
    return e == cudaSuccess ? HQ4_OK : HQ4_ERR_LAUNCH;
}

// Fill the shape/plan part of the parameters and launch.  `prm` carries the
// pointers and the epilogue/prologue options.
static void fill_shape(GemvM1Params& prm, const GemvPlan& pl) {
    prm.ng = pl.ng;
    prm.sg_shift = pl.sg_shift;
    prm.n_sg = pl.n_sg;
    prm.n_strips = pl.n_strips;
    prm.nq = pl.nq;
    prm.status = status_word();
}

GemvM1Params gemv_params(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                         const float* x, float* out, int n_out, int n_in);

// The W4A16 GEMM entry point's batch-1 case (x fp32 or bf16): the streaming
// kernel when the shape and pointers suit it; *used says whether it ran.
int gemv_stream_m1(const uint32_t* w, const uint16_t* sc, const uint16_t* bi, const void* x, bool x_bf16,
                   float* out, int n_out, int n_in, int gs, const float* row_add, const float* residual,
                   cudaStream_t st, bool* used) {
    *used = false;
    GemvPlan pl;
    if (plan_gemv(n_out, n_in, gs, pl)) return HQ4_OK;
    GemvM1Params prm = gemv_params(w, sc, bi, static_cast<const float*>(x), out, n_out, n_in);
    prm.row_add = row_add;
    prm.residual = residual;
    prm.x_bf16 = x_bf16 ? 1 : 0;
    fill_shape(prm, pl);
    return launch_stream(pl, prm, st, used);
}

// Whether gemv_stream_m1 takes a shape at group size 64 with 16-byte aligned
// scales and biases (host only; for the launch plan).
bool gemv_stream_fits_gs64(int n_out, int n_in) {
    GemvPlan pl;
    if (n_out <= 0 || n_in <= 0 || plan_gemv(n_out, n_in, 64, pl) || pl.kg != 64 || pl.n_sg % 8) return false;
    const int grid = std::min(pl.n_strips, sm_count());
    StreamLayout L;
    L.ns_max = (pl.n_strips + grid - 1) / grid;
    L.nkb = (pl.ng / 4 + kStrKc - 1) / kStrKc;
    L.ring = 3;
    return L.bytes() <= kStrSmemTarget;
}

int gemv_launch(GemvM1Params prm, int gs, cudaStream_t st) {
    GemvPlan pl;
    int rc = plan_gemv(prm.n_out, prm.n_in, gs, pl);
    if (rc) return rc;
    if (((uintptr_t)prm.w & 31) || ((uintptr_t)prm.x & 15) || ((uintptr_t)prm.out & 3))
        return HQ4_ERR_ALIGN;
    if (prm.norm_w && ((uintptr_t)prm.norm_w & 15)) return HQ4_ERR_ALIGN;
    fill_shape(prm, pl);
    bool streamed = false;
    rc = launch_stream(pl, prm, st, &streamed);
    if (streamed || rc) return rc;
    return pl.kg == 64 ? launch_m1<64>(pl, prm, st) : launch_m1<32>(pl, prm, st);
}

GemvM1Params gemv_params(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                         const float* x, float* out, int n_out, int n_in) {
    GemvM1Params prm = {};
    prm.w = w;
    prm.sc = scales;
    prm.bi = biases;
    prm.x = x;
    prm.out = out;
    prm.n_out = n_out;
    prm.n_in = n_in;
    prm.mode = kEpiPlain;
    return prm;
}

int gemv_m1(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, const float* x,
            float* out, int n_out, int n_in, int gs, const float* row_add, const float* residual,
            cudaStream_t st) {
    GemvM1Params prm = gemv_params(w, scales, biases, x, out, n_out, n_in);
    prm.row_add = row_add;
    prm.residual = residual;
    return gemv_launch(prm, gs, st);
}

int gemv_launch_stage(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                      const float* x, float* out, int n_out, int n_in, int gs, const float* row_add,
                      const float* residual, const float* norm_w, float eps, int mode, int q_strips,
                      int k_strips, int head_dim, int max_ctx, int tok, const int* pos,
                      const float* rope_cos, const float* rope_sin, float* q_out, float* k_cache,
                      float* v_cache, cudaStream_t st) {
    GemvM1Params prm = gemv_params(w, scales, biases, x, out, n_out, n_in);
    prm.row_add = row_add;
    prm.residual = residual;
    prm.norm_w = norm_w;
    prm.eps = eps;
    prm.mode = mode;
    prm.q_strips = q_strips;
    prm.k_strips = k_strips;
    prm.head_dim = head_dim;
    prm.max_ctx = max_ctx;
    prm.tok = tok;
    prm.pos = pos;
    prm.rope_cos = rope_cos;
    prm.rope_sin = rope_sin;
    prm.q_out = q_out;
    prm.k_cache = k_cache;
    prm.v_cache = v_cache;
    return gemv_launch(prm, gs, st);
}

int check_device_cap() { return check_device(); }

// Two or more fp32 tokens through the multi-token streaming kernel (passes
// of up to 4 tokens); *used is false when the shape or pointers do not suit
// it.
static int gemv_tokens_mt(const uint32_t* w, const uint16_t* sc, const uint16_t* bi, const float* x, float* out,
                          int n_out, int n_in, int gs, int m, const float* row_add, const float* residual,
                          int weights_after_wait, cudaStream_t st, bool* used) {
    *used = false;
    if (m < 2) return HQ4_OK;
    MtParams mp = {};
    mp.w = w;
    mp.sc = sc;
    mp.bi = bi;
    mp.x = x;
    mp.x_stride = n_in;
    mp.out = out;
    mp.out_stride = n_out;
    mp.n_out = n_out;
    mp.n_in = n_in;
    mp.row_add = row_add;
    mp.residual = residual;
    mp.mode = kEpiPlain;
    mp.weights_after_wait = weights_after_wait;
    return gemv_mt_tokens(mp, gs, m, st, used);
}

}  // namespace hq4

using namespace hq4;

extern "C" int hq4_version(void) { return (0 << 16) | 2; }

extern "C" int hq4_device_status(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_hq4_status, sizeof(int)) != cudaSuccess) return HQ4_ERR_LAUNCH;
    if (clear) {
        const int z = 0;
        cudaMemcpyToSymbol(g_hq4_status, &z, sizeof(int));
    }
    return v;
}


extern "C" int hq4_gemv(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                        const float* x, float* out, int n_out, int n_in, int gs, int m,
                        void* stream) {
    if (int rc = check_device()) return rc;
    if (m <= 0) return HQ4_ERR_SHAPE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    bool used = false;
    if (int rc = gemv_tokens_mt(w, scales, biases, x, out, n_out, n_in, gs, m, nullptr, nullptr, 0, st, &used))
        return rc;
    if (used) return HQ4_OK;
    for (int i = 0; i < m; i++) {
        int rc = gemv_m1(w, scales, biases, x + (size_t)i * n_in, out + (size_t)i * n_out, n_out,
                         n_in, gs, nullptr, nullptr, st);
        if (rc) return rc;
    }
    return HQ4_OK;
}

extern "C" int hq4_gemv_fused(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                              const float* x, float* out, int n_out, int n_in, int gs, int m,
                              const float* row_add, const float* residual, void* stream) {
    if (int rc = check_device()) return rc;
    if (m <= 0) return HQ4_ERR_SHAPE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    bool used = false;
    if (int rc = gemv_tokens_mt(w, scales, biases, x, out, n_out, n_in, gs, m, row_add, residual, 0, st, &used))
        return rc;
    if (used) return HQ4_OK;
    for (int i = 0; i < m; i++) {
        int rc = gemv_m1(w, scales, biases, x + (size_t)i * n_in, out + (size_t)i * n_out, n_out,
                         n_in, gs, row_add, residual ? residual + (size_t)i * n_out : nullptr, st);
        if (rc) return rc;
    }
    return HQ4_OK;
}

extern "C" int hq4_gemv_ex(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, const float* x,
                           float* out, int n_out, int n_in, int gs, int m, const float* row_add,
                           const float* residual, int flags, void* stream) {
    if (int rc = check_device()) return rc;
    if (m <= 0 || (flags & ~HQ4_GEMV_WEIGHTS_AFTER_WAIT)) return HQ4_ERR_SHAPE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    bool used = false;
    if (int rc = gemv_tokens_mt(w, scales, biases, x, out, n_out, n_in, gs, m, row_add, residual,
                                (flags & HQ4_GEMV_WEIGHTS_AFTER_WAIT) ? 1 : 0, st, &used))
        return rc;
    if (used) return HQ4_OK;
    for (int i = 0; i < m; i++) {
        GemvM1Params prm = gemv_params(w, scales, biases, x + (size_t)i * n_in, out + (size_t)i * n_out, n_out, n_in);
        prm.row_add = row_add;
        prm.residual = residual ? residual + (size_t)i * n_out : nullptr;
        prm.weights_after_wait = (flags & HQ4_GEMV_WEIGHTS_AFTER_WAIT) ? 1 : 0;
        if (int rc = gemv_launch(prm, gs, st)) return rc;
    }
    return HQ4_OK;
}

// x rows from pinned, device-mapped host memory into the device staging
// buffer, one float4 per thread.  It triggers its dependents at once, so the
// GEMV launched after it (PDL) starts its CTAs and streams its first weight
// stages while x crosses the host link; the GEMV reads x only after this
// kernel completes (its dependency wait).
__global__ void __launch_bounds__(256) host_x_kernel(const float4* __restrict__ src, float4* __restrict__ dst,
                                                     int n4) {
    pdl_launch_dependents();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n4) dst[i] = src[i];
}

extern "C" int hq4_gemv_host(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                             const float* row_add, const float* x_host, float* out_host, int n_out, int n_in,
                             int gs, int m, float* x_dev, float* out_dev, void* stream) {
    if (int rc = check_device()) return rc;
    if (m <= 0 || n_out <= 0 || n_in <= 0 || !x_host || !out_host || !x_dev || !out_dev) return HQ4_ERR_SHAPE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t in_bytes = (size_t)m * n_in * sizeof(float), out_bytes = (size_t)m * n_out * sizeof(float);
    // Pinned, device-mapped host output: the GEMV's epilogue stores straight
    // into it (the products cross the bus once, from the kernel), which saves
    // the separate device-to-host copy and its latency.  Other host memory
    // takes the copy.
    float* out_direct = nullptr;
    cudaPointerAttributes pa;
    if (cudaPointerGetAttributes(&pa, out_host) == cudaSuccess && pa.type == cudaMemoryTypeHost && pa.devicePointer &&
        ((uintptr_t)pa.devicePointer & 3) == 0)
        out_direct = static_cast<float*>(pa.devicePointer);
    else
        (void)cudaGetLastError();  // an unregistered pointer is not an error here
    // A pinned, device-mapped x is fetched by a small kernel instead of a copy,
    // so the GEMV's weight stream starts while x is in flight (a copy would
    // have to finish before the GEMV could start).  Other host memory is copied.
    const float4* x_direct = nullptr;
    if ((in_bytes & 15) == 0 && ((uintptr_t)x_dev & 15) == 0 && cudaPointerGetAttributes(&pa, x_host) == cudaSuccess &&
        pa.type == cudaMemoryTypeHost && pa.devicePointer && ((uintptr_t)pa.devicePointer & 15) == 0)
        x_direct = static_cast<const float4*>(pa.devicePointer);
    else
        (void)cudaGetLastError();
    if (x_direct) {
        const int n4 = (int)(in_bytes / 16);
        host_x_kernel<<<(n4 + 255) / 256, 256, 0, st>>>(x_direct, reinterpret_cast<float4*>(x_dev), n4);
        if (cudaGetLastError() != cudaSuccess) return HQ4_ERR_LAUNCH;
    } else if (cudaMemcpyAsync(x_dev, x_host, in_bytes, cudaMemcpyHostToDevice, st) != cudaSuccess) {
        return HQ4_ERR_LAUNCH;
    }
    if (int rc = hq4_gemv_fused(w, scales, biases, x_dev, out_direct ? out_direct : out_dev, n_out, n_in, gs, m,
                                row_add, nullptr, stream))
        return rc;
    if (!out_direct && cudaMemcpyAsync(out_host, out_dev, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return HQ4_ERR_LAUNCH;
    return cudaStreamSynchronize(st) == cudaSuccess ? HQ4_OK : HQ4_ERR_LAUNCH;
}

extern "C" int hq4_dequant(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                           float* out, int row0, int row1, int n_in, int gs, void* stream) {
    if (int rc = check_device()) return rc;
    if (n_in <= 0 || gs <= 0 || n_in % gs || gs % 8 || row0 < 0) return HQ4_ERR_SHAPE;
    const int rows = row1 - row0;
    if (rows <= 0) return HQ4_OK;
    if (((uintptr_t)out & 15) || ((uintptr_t)w & 3)) return HQ4_ERR_ALIGN;
    const long long total = (long long)rows * (n_in / 8);
    const int threads = 256;
    const long long want = (total + threads - 1) / threads;
    const int grid = (int)std::min<long long>(want, (long long)sm_count() * 16);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(grid);
    lc.blockDim = dim3(threads);
    lc.stream = static_cast<cudaStream_t>(stream);
    lc.attrs = attr;
    lc.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&lc, dequant_kernel, w, scales, biases, out, row0, rows, n_in, gs);
    return e == cudaSuccess ? HQ4_OK : HQ4_ERR_LAUNCH;
}
