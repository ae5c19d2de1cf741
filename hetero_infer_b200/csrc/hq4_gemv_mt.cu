// Multi-token streaming W4A16 product (a few tokens per pass over the weights):
//   out[j][r] = sum_k x[j][k] * (q[r][k] * scale[r][k/gs] + bias[r][k/gs])
// for microbatched decode and prompt chunks.  The reference computes the
// same product in QLinear (hetero/cpu_model.py:118-136): one q4gemv call per
// token (kernel/q4gemv.c:232-301), dequantisation plus a BLAS matmul for a
// prompt.
//
// The weight stream is the one-token streaming GEMV's (hq4_gemv.cu): one
// producer thread brings 16-row strips x 16 k-chunks of 256 values (32 KB of
// packed words plus the strip's scales and biases) through a ring of shared-
// memory stages with TMA, and consumer warp w takes k-chunk w of every stage.
// The arithmetic is that kernel's exact digit product, laid out so that the
// tokens share each weight fragment:
// * x of a (64-value group, token) is a 22-bit fixed-point integer (the
//   group's exponent E, v = rint(x 2^(22-E))) written as three balanced s8
//   digits d2, d1, d0, one MMA column per digit;
// * in an m16n8k32 integer MMA all 32 k-slots belong to one group (words 2t
//   and 2t+1 of the group for lane t: even nibbles of a word in one register,
//   odd ones in the other, 3 instructions per word), so the 8 columns are 8
//   (token, digit) pairs and a group is 2 MMAs per 8 columns: 16 MMAs per
//   16 x 256 tile serve 4 tokens (2 column tiles), 24 serve 8 (3 tiles);
// * lane t of the accumulator holds columns 2t, 2t+1 of every tile: its
//   tokens are t, t+4 and their digits sit in its own columns, so a token's
//   dot (d2 2^16 + d1 2^8 + d0, exact integers, two fp32 roundings) and its
//   scale and bias (s 2^(E-22) dot + b sum(x)) stay lane-local.
// The digits of bf16 x are exact; fp32 x carries 22 bits below its group's
// maximum, as in the one-token kernel.  Every sum runs in a fixed order
// (deterministic).
//
// x is converted once per CTA, before the stage loop.  For passes of up to
// 4 tokens a CTA's k-range is at most 16 chunks (K is split over a cluster
// where it is longer), so warp w owns chunk w and keeps its digit registers
// (the MMAs' B operands) and each group's (2^(E-22), sum(x)) in registers for
// the whole pass; the two lanes of a token's columns split its values.  For
// 8-token passes the digits of the CTA's k-range wait in a shared-memory
// image.
//
// Stages run strip-major (a strip's k-blocks back to back), so a warp keeps
// its share of a strip in registers.  At the strip's end each warp parks its
// 16-row x token sums in shared memory; every 32/T strips all consumer
// threads add the parked sums over the 16 warps in warp order (between two
// named barriers, no per-stage synchronisation) and apply the epilogue of the
// one-token kernel: plain with row add and residual, SiLU(gate) * up, or
// q|k|v with RoPE and the cache writes.  With K split over a cluster each
// CTA parks its per-strip sums, and after a cluster barrier they are added
// over the ranks in rank order through distributed shared memory
// (deterministic, no atomics, no global scratch).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "hq4.h"
#include "hq4_common.cuh"
#include "hq4_gemv_dev.cuh"
#include "hq4_host.cuh"
#include "hq4_mt.cuh"
#include "hq4_tmap.cuh"

namespace hq4 {

int* status_word();
int check_device_cap();

// Column tiles (8 MMA columns each) per pass and the tokens they carry: lane
// t holds 2 CT columns, 3 per token, so 4 * floor(2 CT / 3) tokens.
__host__ __device__ constexpr int mt_tokens(int ct) { return 4 * ((2 * ct) / 3); }
// Image bytes of one k-chunk: per column tile 4 groups x 32 lanes x 16 B of B
// fragments, then per (group, token) the fp32 pair (2^(E-22), sum of x).
__host__ __device__ constexpr int mt_img_bytes(int ct) { return ct * 2048 + 4 * kMtMaxTok * 8; }
constexpr int kMtEarlyStages = 3;          // stages issued before the x images are built
// Per-warp strip sums wait in shared memory for a batch of 32 / T strips (32
// KB) before the 16 warps add them up together.
constexpr int kMtPartFloats = 8192;
__host__ __device__ constexpr int mt_batch(int tok) { return kMtPartFloats / (kStrConsumers * 16 * tok); }
constexpr size_t kMtSmemTarget = 220 * 1024;
constexpr int kMtMaxRing = 5;

// Passes of up to 4 tokens (2 column tiles) keep each warp's x digits in
// registers (one k-chunk per warp: the CTA's k-range is at most 16 chunks);
// 8-token passes keep a shared-memory image of the CTA's k-range.
__host__ __device__ constexpr bool mt_reg(int ct) { return ct == 2; }

struct MtLayout {
    int ring, ns_max, nch_max, ct, ks;
    __host__ __device__ int tok() const { return mt_tokens(ct); }
    __host__ __device__ size_t img_off() const { return (size_t)ring * kStrStageBytes; }
    __host__ __device__ size_t part_off() const {
        return img_off() + (mt_reg(ct) ? 0 : (size_t)nch_max * mt_img_bytes(ct));
    }
    __host__ __device__ size_t res_off() const { return part_off() + (size_t)kMtPartFloats * 4; }
    __host__ __device__ size_t red_off() const {
        return res_off() + (ks > 1 ? (size_t)ns_max * 16 * tok() * 4 : 0);
    }
    __host__ __device__ size_t nf_off() const { return red_off() + (size_t)kMtMaxTok * kStrConsumers * 4; }
    __host__ __device__ size_t bar_off() const { return nf_off() + (size_t)kMtMaxTok * 4; }
    // full[ring], empty[ring], images built
    __host__ __device__ size_t bytes() const { return bar_off() + (size_t)(2 * ring + 1) * 8 + 1024; }
};

// RMSNorm factors 1/sqrt(mean(x_j^2) + eps) of the pass's tokens into nf[]:
// thread i sums squares of x values 4i..4i+3 (mod 2048) in k order, the warp's
// xor tree, then the warps in order.  Named barrier 1 over the consumers.
__device__ __forceinline__ void mt_norm_factors(const MtParams& p, float* red, float* nf, int warp, int lane) {
    const int tid = warp * 32 + lane;
    for (int j = 0; j < p.m; j++) {
        const float* xr = static_cast<const float*>(p.x) + (size_t)j * p.x_stride;
        float ss = 0.0f;
        for (int k = tid * 4; k < p.n_in; k += kStrConsumers * 32 * 4) {
            const float4 v = *reinterpret_cast<const float4*>(xr + k);
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) red[j * kStrConsumers + warp] = ss;
    }
    asm volatile("bar.sync 1, 512;" ::: "memory");
    if (tid < p.m) {
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < kStrConsumers; w++) tot += red[tid * kStrConsumers + w];
        const float mean = __fdiv_rn(tot, (float)p.n_in);
        nf[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
    }
    asm volatile("bar.sync 1, 512;" ::: "memory");
}

// x values 16t..16t+15 of each of the 4 groups of the chunk whose first
// value is kbase - 16t, for token j (zeros when !valid), RMSNorm applied
// when p.norm_w: every value requested before any is used (one round trip
// to memory, which under the weight stream is the prologue's cost).
__device__ __forceinline__ void mt_load_x(const MtParams& p, int j, bool valid, int kbase, const float* nf,
                                          float (&v)[4][16]) {
    if (!valid) {
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
            for (int i = 0; i < 16; i++) v[u][i] = 0.0f;
        return;
    }
    if (p.x_bf16) {  // bf16 widens to fp32 exactly
        uint4 r[4][2];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.x) +
                                                              (size_t)j * p.x_stride + kbase + 64 * u);
            r[u][0] = src[0];
            r[u][1] = src[1];
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const uint32_t wv[8] = {r[u][0].x, r[u][0].y, r[u][0].z, r[u][0].w,
                                    r[u][1].x, r[u][1].y, r[u][1].z, r[u][1].w};
#pragma unroll
            for (int i = 0; i < 8; i++) {
                v[u][2 * i] = __uint_as_float(wv[i] << 16);
                v[u][2 * i + 1] = __uint_as_float(wv[i] & 0xFFFF0000u);
            }
        }
        return;
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.x) + (size_t)j * p.x_stride +
                                                            kbase + 64 * u);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float4 q = src[i];
            v[u][4 * i] = q.x;
            v[u][4 * i + 1] = q.y;
            v[u][4 * i + 2] = q.z;
            v[u][4 * i + 3] = q.w;
        }
    }
    if (p.norm_w) {
        const float r = nf[j];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const float4* nw = reinterpret_cast<const float4*>(p.norm_w + kbase + 64 * u);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float4 q = nw[i];
                v[u][4 * i] = __fmul_rn(__fmul_rn(v[u][4 * i], r), q.x);
                v[u][4 * i + 1] = __fmul_rn(__fmul_rn(v[u][4 * i + 1], r), q.y);
                v[u][4 * i + 2] = __fmul_rn(__fmul_rn(v[u][4 * i + 2], r), q.z);
                v[u][4 * i + 3] = __fmul_rn(__fmul_rn(v[u][4 * i + 3], r), q.w);
            }
        }
    }
}

// One group's exponent E and sum over the four lanes of a column (two
// shuffles each) and its 16 values' digit words (d2 d1 d0 in bytes 2 1 0).
__device__ __forceinline__ void mt_group(const float (&v)[16], int& E, float& sum, uint32_t (&dw)[16]) {
    float amax = 0.0f;
    sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
        amax = fmaxf(amax, fabsf(v[i]));
        sum += v[i];
    }
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    E = group_exponent(amax);
    const float up = exp2i(kXBits - E);
#pragma unroll
    for (int i = 0; i < 16; i++) dw[i] = digits3(v[i], up);
}

// The two MMAs' B registers of digit di (0: d2, 1: d1, 2: d0): even k to
// b0, odd k to b1, values 0-7 for the first MMA, 8-15 for the second.
__device__ __forceinline__ uint4 mt_frag(const uint32_t (&dw)[16], int di) {
    // byte b of two words into bytes 0, 1 (prmt selector nibbles b, b + 4)
    const uint32_t b = 2 - di, sel = b | ((b + 4) << 4);
    auto word = [&](int i) {  // bytes b of dw[i], dw[i+2], dw[i+4], dw[i+6]
        return prmt(prmt(dw[i], dw[i + 2], sel), prmt(dw[i + 4], dw[i + 6], sel), 0x5410);
    };
    return make_uint4(word(0), word(1), word(8), word(9));
}

// The digit columns of this warp's k-chunks (local chunk lc = warp + 16 i of
// the CTA's range starting at c0) into the shared-memory image.  Lane (g, t)
// supplies B column g of every column tile ct: the column's owner in the
// accumulator is lane-group g/2, its flat index f = 2 ct + g%2 among that
// lane-group's columns, token g/2 + 4 (f / 3), digit f % 3 (d2, d1, d0).  A
// lane therefore serves one token at 2 column tiles and two at 3.
template <int CT>
__device__ __forceinline__ void mt_build(const MtParams& p, unsigned char* img, int c0, int nch, const float* nf,
                                         int warp, int lane) {
    constexpr int T = mt_tokens(CT), NSG = T / 4;
    const int g = lane >> 2, t = lane & 3, h = g & 1;
    for (int lc = warp; lc < nch; lc += kStrConsumers) {
        unsigned char* cimg = img + (size_t)lc * mt_img_bytes(CT);
        const int kbase = (c0 + lc) * 256 + 16 * t;
#pragma unroll
        for (int sg = 0; sg < NSG; sg++) {
            const int j = (g >> 1) + 4 * sg;
            float v[4][16];
            mt_load_x(p, j, j < p.m, kbase, nf, v);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                int E;
                float sum;
                uint32_t dw[16];
                mt_group(v[u], E, sum, dw);
#pragma unroll
                for (int ct = 0; ct < CT; ct++) {
                    const int f = 2 * ct + h;
                    if (f / 3 == sg)
                        *reinterpret_cast<uint4*>(cimg + ct * 2048 + u * 512 + lane * 16) = mt_frag(dw, f % 3);
                }
                // (2^(E-22), sum) of (group u, token j), from the lane of its d2 column
                if (t == 0 && h == ((3 * sg) & 1))
                    *reinterpret_cast<float2*>(cimg + CT * 2048 + (u * kMtMaxTok + j) * 8) =
                        make_float2(exp2i(E - kXBits), sum);
            }
        }
        // columns past the last token slot multiply zeros
#pragma unroll
        for (int ct = 0; ct < CT; ct++) {
            if ((2 * ct + h) / 3 < NSG) continue;
#pragma unroll
            for (int u = 0; u < 4; u++)
                *reinterpret_cast<uint4*>(cimg + ct * 2048 + u * 512 + lane * 16) = make_uint4(0, 0, 0, 0);
        }
    }
}

// The same columns in registers, for a CTA whose k-range is at most 16
// chunks (warp w's chunk is w): B[ct][u] the lane's B registers, M[sg][u]
// the (2^(E-22), sum) of group u of token t + 4 sg -- the token this lane
// accumulates, whose values lane 8t converted.  The two lanes of a token's
// columns (g and g^1, lanes l and l^4) split its 16 values: lane g%2 = h
// loads and converts values 8h..8h+7 of each group, the group's exponent
// and sum take one more shuffle level, and the partners swap digit words.
template <int CT>
__device__ __forceinline__ void mt_build_reg(const MtParams& p, int c0, int nch, const float* nf, int warp, int lane,
                                             uint4 (&B)[CT][4], float2 (&M)[mt_tokens(CT) / 4][4]) {
    constexpr int NSG = mt_tokens(CT) / 4;
    const int g = lane >> 2, t = lane & 3, h = g & 1;
    const bool has = warp < nch;
    const int kbase = (c0 + warp) * 256 + 16 * t + 8 * h;
#pragma unroll
    for (int ct = 0; ct < CT; ct++)
#pragma unroll
        for (int u = 0; u < 4; u++) B[ct][u] = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int sg = 0; sg < NSG; sg++) {
        const int j = (g >> 1) + 4 * sg;
        const bool valid = has && j < p.m;
        float v[4][8];
        if (!valid) {
#pragma unroll
            for (int u = 0; u < 4; u++)
#pragma unroll
                for (int i = 0; i < 8; i++) v[u][i] = 0.0f;
        } else if (p.x_bf16) {  // bf16 widens to fp32 exactly
            uint4 r[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                r[u] = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.x) + (size_t)j * p.x_stride +
                                                       kbase + 64 * u);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint32_t wv[4] = {r[u].x, r[u].y, r[u].z, r[u].w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    v[u][2 * i] = __uint_as_float(wv[i] << 16);
                    v[u][2 * i + 1] = __uint_as_float(wv[i] & 0xFFFF0000u);
                }
            }
        } else {
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.x) +
                                                                    (size_t)j * p.x_stride + kbase + 64 * u);
                const float4 a = src[0], b = src[1];
                v[u][0] = a.x; v[u][1] = a.y; v[u][2] = a.z; v[u][3] = a.w;
                v[u][4] = b.x; v[u][5] = b.y; v[u][6] = b.z; v[u][7] = b.w;
            }
            if (p.norm_w) {
                const float r = nf[j];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const float4* nw = reinterpret_cast<const float4*>(p.norm_w + kbase + 64 * u);
                    const float4 a = nw[0], b = nw[1];
                    const float wn[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
                    for (int i = 0; i < 8; i++) v[u][i] = __fmul_rn(__fmul_rn(v[u][i], r), wn[i]);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            float amax = 0.0f, sum = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                amax = fmaxf(amax, fabsf(v[u][i]));
                sum += v[u][i];
            }
#pragma unroll
            for (int o = 1; o <= 4; o <<= 1) {
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                sum += __shfl_xor_sync(0xffffffffu, sum, o);
            }
            const int E = group_exponent(amax);
            const float up = exp2i(kXBits - E);
            uint32_t dw[16];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const uint32_t own = digits3(v[u][i], up);
                const uint32_t other = __shfl_xor_sync(0xffffffffu, own, 4);
                dw[i] = h ? other : own;
                dw[8 + i] = h ? own : other;
            }
#pragma unroll
            for (int ct = 0; ct < CT; ct++) {
                const int f = 2 * ct + h;
                if (f / 3 == sg) B[ct][u] = mt_frag(dw, f % 3);
            }
            const float mx = __shfl_sync(0xffffffffu, exp2i(E - kXBits), 8 * t);
            const float ms = __shfl_sync(0xffffffffu, sum, 8 * t);
            M[sg][u] = make_float2(mx, ms);
        }
    }
}

// Scale-tile byte offset of (row, scale group gi) inside a stage (the tile
// carries the swizzle of its row width, as the one-token kernel's).
__device__ __forceinline__ int mt_sb_off(int row, int gi, int sb_row, int sb_mask) {
    const int o = row * sb_row + gi * 2;
    return o ^ (((o >> 7) & sb_mask) << 4);
}

// Per-lane constants of the tile arithmetic: the scale-tile offsets of this
// warp's 4 groups in rows g and g+8 (at one scale per group the four are 8
// consecutive bytes inside one swizzle unit: one 8-byte load per row).
struct MtLane {
    int so[2][4];
    bool vec;
};
__device__ __forceinline__ MtLane mt_lane(int warp, int lane, int sg_shift, int sb_row, int sb_mask) {
    MtLane L;
    const int g = lane >> 2;
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int gi = (warp * 4 + u) >> sg_shift;
        L.so[0][u] = mt_sb_off(g, gi, sb_row, sb_mask);
        L.so[1][u] = mt_sb_off(g + 8, gi, sb_row, sb_mask);
    }
    L.vec = sg_shift == 0;
    return L;
}

// One stage tile of this warp (16 rows x k-chunk `warp`) against its x
// digits (registers B, M when REG, else the chunk image `cimg`), accumulated
// into acc[sigma] = rows (g, g+8) of token t + 4 sigma.
template <int CT, bool REG>
__device__ __forceinline__ void mt_tile(const unsigned char* st, const unsigned char* cimg, const uint4 (&Br)[CT][4],
                                        const float2 (&Mr)[mt_tokens(CT) / 4][4], int warp, int lane,
                                        const MtLane& L, float (&acc)[mt_tokens(CT) / 4][2]) {
    constexpr int NS = mt_tokens(CT) / 4;
    const int g = lane >> 2, t = lane & 3;
    const unsigned char* wt = st + warp * kStrTileBytes;
    const unsigned char* ss = st + kStrWBytes;
    const unsigned char* sbi = st + kStrWBytes + kStrSBBytes;
    uint32_t sc[2][4], bc[2][4];  // fp16 bits of the 4 groups' scales and biases, rows g and g+8
    if (L.vec) {
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const uint2 a = *reinterpret_cast<const uint2*>(ss + L.so[r][0]);
            const uint2 b = *reinterpret_cast<const uint2*>(sbi + L.so[r][0]);
            sc[r][0] = a.x & 0xFFFFu, sc[r][1] = a.x >> 16, sc[r][2] = a.y & 0xFFFFu, sc[r][3] = a.y >> 16;
            bc[r][0] = b.x & 0xFFFFu, bc[r][1] = b.x >> 16, bc[r][2] = b.y & 0xFFFFu, bc[r][3] = b.y >> 16;
        }
    } else {
#pragma unroll
        for (int r = 0; r < 2; r++)
#pragma unroll
            for (int u = 0; u < 4; u++) {
                sc[r][u] = *reinterpret_cast<const uint16_t*>(ss + L.so[r][u]);
                bc[r][u] = *reinterpret_cast<const uint16_t*>(sbi + L.so[r][u]);
            }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const float s0 = h2f(sc[0][u]), s1 = h2f(sc[1][u]);
        const float b0 = h2f(bc[0][u]), b1 = h2f(bc[1][u]);
        // words 2t, 2t+1 of group u in rows g and g+8 (128-byte swizzle)
        const int c16 = 2 * u + (t >> 1);
        const int wo = ((c16 ^ g) << 4) + (t & 1) * 8;
        const uint2 w0 = *reinterpret_cast<const uint2*>(wt + g * 128 + wo);
        const uint2 w1 = *reinterpret_cast<const uint2*>(wt + (g + 8) * 128 + wo);
        uint32_t e0, o0, e1, o1, e2, o2, e3, o3;
        unpack_u8(w0.x, e0, o0);
        unpack_u8(w1.x, e1, o1);
        unpack_u8(w0.y, e2, o2);
        unpack_u8(w1.y, e3, o3);
        int c[CT][4];
#pragma unroll
        for (int ct = 0; ct < CT; ct++) {
            const uint4 B = REG ? Br[ct][u] : *reinterpret_cast<const uint4*>(cimg + ct * 2048 + u * 512 + lane * 16);
            mma_u8s8_16832_first(c[ct], e0, e1, o0, o1, B.x, B.y);
            mma_u8s8_16832(c[ct], e2, e3, o2, o3, B.z, B.w);
        }
#pragma unroll
        for (int sg = 0; sg < NS; sg++) {
            // columns 3 sg (d2), 3 sg + 1 (d1), 3 sg + 2 (d0) of this lane's flat list
            const int f2 = 3 * sg, f1 = 3 * sg + 1, f0 = 3 * sg + 2;
            const float2 meta =
                REG ? Mr[sg][u] : *reinterpret_cast<const float2*>(cimg + CT * 2048 + (u * kMtMaxTok + t + 4 * sg) * 8);
            // dot = d2 2^16 + d1 2^8 + d0: the low two digits combined exactly in
            // 32 bits (|d1 sum| * 2^8 < 2^25), then one fp32 rounding
            const int lo0 = c[f1 >> 1][f1 & 1] * 256 + c[f0 >> 1][f0 & 1];
            const int lo1 = c[f1 >> 1][2 + (f1 & 1)] * 256 + c[f0 >> 1][2 + (f0 & 1)];
            const float dot0 = fmaf((float)c[f2 >> 1][f2 & 1], 65536.0f, (float)lo0);
            const float dot1 = fmaf((float)c[f2 >> 1][2 + (f2 & 1)], 65536.0f, (float)lo1);
            acc[sg][0] = fmaf(s0 * meta.x, dot0, fmaf(b0, meta.y, acc[sg][0]));
            acc[sg][1] = fmaf(s1 * meta.x, dot1, fmaf(b1, meta.y, acc[sg][1]));
        }
    }
}

// Store rows (g, g+8) of strip s for token j of the pass, as the one-token
// kernel's store_pair_in does for its token.
__device__ __forceinline__ void mt_store(const MtParams& p, int s, int g, int j, float y0, float y1) {
    if (p.mode == kEpiPlain) {
        const int r[2] = {s * 16 + g, s * 16 + g + 8};
        const float yv[2] = {y0, y1};
#pragma unroll
        for (int q = 0; q < 2; q++) {
            if (r[q] >= p.n_out) continue;
            const size_t o = (size_t)j * p.out_stride + r[q];
            float y = yv[q];
            if (p.row_add) y += p.row_add[r[q]];
            if (p.residual) y += p.residual[o];
            p.out[o] = y;
        }
        return;
    }
    if (p.mode == kEpiSiluMul) {
        // strip s holds gate rows 8s..8s+7 (g) and the matching up rows (g+8)
        const int r = s * 8 + g;
        if (r < p.n_out / 2) p.out[(size_t)j * p.out_stride + r] = __fmul_rn(silu_ref(y0), y1);
        return;
    }
    // kEpiQkvRope
    if (p.row_add) {
        y0 = __fadd_rn(y0, p.row_add[s * 16 + g]);
        y1 = __fadd_rn(y1, p.row_add[s * 16 + g + 8]);
    }
    const int half = p.head_dim >> 1;
    const int spp = half >> 3;  // strips per head (8 rotation pairs per strip)
    const int pos = *p.pos + p.tok0 + j;
    if (pos < 0 || pos >= p.max_ctx) return;  // outside the cache: write nothing
    if (s < p.q_strips + p.k_strips) {
        const bool is_q = s < p.q_strips;
        const int sl = is_q ? s : s - p.q_strips;
        const int head = sl / spp, jj = (sl % spp) * 8 + g;
        const float c = p.rope_cos[(size_t)pos * half + jj], sn = p.rope_sin[(size_t)pos * half + jj];
        // hetero/cpu_model.py:200-203: (x1*cos - x2*sin, x1*sin + x2*cos)
        const float o1 = __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, sn));
        const float o2 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, c));
        float* dst = is_q ? p.q_out + (size_t)j * p.q_stride + (size_t)head * p.head_dim
                          : p.k_cache + ((size_t)head * p.max_ctx + pos) * p.head_dim;
        dst[jj] = o1;
        dst[jj + half] = o2;
    } else {
        const int r0 = (s - p.q_strips - p.k_strips) * 16 + g;  // natural v row order
        const int r1 = r0 + 8;
        const int head0 = r0 / p.head_dim, head1 = r1 / p.head_dim;
        p.v_cache[((size_t)head0 * p.max_ctx + pos) * p.head_dim + (r0 % p.head_dim)] = y0;
        p.v_cache[((size_t)head1 * p.max_ctx + pos) * p.head_dim + (r1 % p.head_dim)] = y1;
    }
}

// Sums of rows (g, g+8) of strip s for token `lane` -> the epilogue.
__device__ __forceinline__ void mt_emit(const MtParams& p, int s, int g, int lane, int tok, float y0, float y1,
                                        bool store) {
    if (store && lane < tok && lane < p.m) mt_store(p, s, g, lane, y0, y1);
}

template <int CT>
__global__ void __launch_bounds__(kStrThreads, 1)
    gemv_mt_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w1,
                   const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_b,
                   const MtParams p, const MtLayout L) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw_u = smem_u32(smem_raw);
    unsigned char* base = smem_raw + (((raw_u + 1023u) & ~1023u) - raw_u);
    const uint32_t base_u = smem_u32(base);
    const int R = L.ring;
    unsigned char* img = base + L.img_off();
    float* part = reinterpret_cast<float*>(base + L.part_off());
    float* res = reinterpret_cast<float*>(base + L.res_off());
    float* red = reinterpret_cast<float*>(base + L.red_off());
    float* nf = reinterpret_cast<float*>(base + L.nf_off());
    const uint32_t bars = base_u + (uint32_t)L.bar_off();
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (R + s); };
    const uint32_t images_bar = bars + 8u * (2 * R);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ks = p.ks;
    const int rank = (int)blockIdx.y;  // cluster rank: the cluster is 1 x ks x 1
    const int cl = (int)blockIdx.x;
    const int s0 = (int)((long long)cl * p.n_strips / p.n_clusters);
    const int s1 = (int)((long long)(cl + 1) * p.n_strips / p.n_clusters);
    const int ns = s1 - s0;
    const int align = 2 << p.sg_shift;
    const int c0 = mt_chunk_start(rank, ks, p.n_chunks, align), c1 = mt_chunk_start(rank + 1, ks, p.n_chunks, align);
    const int nch = c1 - c0;
    const int nkb = (nch + kStrKc - 1) / kStrKc;
    const int n_stages = ns * nkb;
    const int sg_cols = kStrSBCols >> p.sg_shift;
    const uint32_t sb_bytes = 16u * sg_cols * 2u;
    const int sb_row = sg_cols * 2, sb_mask = (sb_row >> 4) - 1;

    // ---- producer (warp 16, one thread): stages strip-major
    const bool producer = warp == kStrConsumers && lane == 0;
    int p_issued = 0, p_slot = 0, p_use = 0, p_kb = 0, p_j = 0;
    uint64_t pol = 0;
    auto issue_stage = [&]() {
        const int strip = s0 + p_j;
        const int cbase = c0 + p_kb * kStrKc;
        const int nval = min(kStrKc, nch - p_kb * kStrKc);
        // a whole box unless it would reach into the next rank's chunks (a
        // box past the row end reads zeros and costs no traffic)
        const bool whole = nval == kStrKc || c1 == p.n_chunks;
        const uint32_t dst = base_u + (uint32_t)p_slot * kStrStageBytes;
        mbar_arrive_expect_tx(full_bar(p_slot),
                              (uint32_t)(whole ? kStrWBytes : nval * kStrTileBytes) + 2u * sb_bytes);
        if (whole) {
            tma_load_3d(dst, &tm_w, 0, strip * 16, cbase, full_bar(p_slot), pol);
        } else {
            for (int i = 0; i < nval; i++)
                tma_load_3d(dst + (uint32_t)(i * kStrTileBytes), &tm_w1, 0, strip * 16, cbase + i, full_bar(p_slot),
                            pol);
        }
        const int gx = (cbase * 4) >> p.sg_shift;
        tma_load_2d(dst + kStrWBytes, &tm_s, gx, strip * 16, full_bar(p_slot), pol);
        tma_load_2d(dst + kStrWBytes + kStrSBBytes, &tm_b, gx, strip * 16, full_bar(p_slot), pol);
        p_issued++;
        if (++p_slot == R) {
            p_slot = 0;
            p_use++;
        }
        if (++p_kb == nkb) {
            p_kb = 0;
            p_j++;
        }
    };
    if (producer) {
        prefetch_tensormap(&tm_w);
        prefetch_tensormap(&tm_w1);
        prefetch_tensormap(&tm_s);
        prefetch_tensormap(&tm_b);
        for (int s = 0; s < R; s++) {
            mbar_init_nofence(full_bar(s), 1);
            mbar_init_nofence(empty_bar(s), kStrConsumers);
        }
        mbar_init_nofence(images_bar, kStrConsumers);
        mbar_init_fence();
    }
    __syncthreads();  // barriers initialised
    pdl_launch_dependents();
    // the first stages leave after the CTA barrier: the consumers start on
    // their x digits meanwhile instead of waiting for the copies' issue
    if (producer) {
        pol = l2_policy_evict_first();  // weights are read once
        if (p.weights_after_wait) pdl_wait();
        const int first = min(min(R, kMtEarlyStages), n_stages);
        for (int i = 0; i < first; i++) issue_stage();
    }

    bool ok = true;
    if (warp == kStrConsumers) {
        if (producer) {
            if (p_issued < n_stages) {
                pdl_wait();
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
            // every issued copy lands before the CTA may exit
            for (int k = max(0, p_issued - R); k < p_issued; k++)
                if (!mbar_wait_nap(full_bar(k % R), (k / R) & 1, kStrWaitNs, 64) && p.status) atomicOr(p.status, 1);
        }
        __syncwarp();
    } else {
        // ---- consumers (warps 0-15)
        constexpr int T = mt_tokens(CT), NS = T / 4;
        constexpr bool kReg = mt_reg(CT);
        pdl_wait();  // x, norm weights, residual and the outputs follow the previous kernel
        if (!p.x_bf16 && p.norm_w) mt_norm_factors(p, red, nf, warp, lane);
        uint4 Breg[CT][4];
        float2 Mreg[NS][4];
        if (kReg)
            mt_build_reg<CT>(p, c0, nch, nf, warp, lane, Breg, Mreg);
        else
            mt_build<CT>(p, img, c0, nch, nf, warp, lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(images_bar);
        const MtLane ML = mt_lane(warp, lane, p.sg_shift, sb_row, sb_mask);
        int slot = 0;
        uint32_t phase = 0;
        const int g = lane >> 2, t = lane & 3;
        constexpr int NB = mt_batch(T);
        // a batch of strips' per-warp sums [strip % NB][warp][16 rows][T] is
        // added over the 16 warps in warp order by all consumer threads, one
        // (strip, row pair, token) each; named barrier 1 before (every warp
        // has parked its sums) and after (the slots may be reused)
        auto flush = [&](int si_last, int nb) {
            asm volatile("bar.sync 1, 512;" ::: "memory");
            const int tid = warp * 32 + lane;
            for (int u = tid; u < nb * 8 * T; u += kStrConsumers * 32) {
                const int bi = u / (8 * T), gg = (u / T) % 8, j = u % T;
                const float* src = part + (size_t)bi * kStrConsumers * 16 * T + gg * T + j;
                float y0 = 0.0f, y1 = 0.0f;
#pragma unroll
                for (int w = 0; w < kStrConsumers; w++) {
                    y0 += src[(size_t)w * 16 * T];
                    y1 += src[(size_t)w * 16 * T + 8 * T];
                }
                const int si = si_last - (nb - 1) + bi;
                if (ks == 1) {
                    if (ok && j < p.m) mt_store(p, s0 + si, gg, j, y0, y1);
                } else {
                    res[((size_t)si * 16 + gg) * T + j] = y0;
                    res[((size_t)si * 16 + gg + 8) * T + j] = y1;
                }
            }
            asm volatile("bar.sync 1, 512;" ::: "memory");
        };
        for (int si = 0; si < ns; si++) {
            float acc[NS][2];
#pragma unroll
            for (int sg = 0; sg < NS; sg++) acc[sg][0] = acc[sg][1] = 0.0f;
            for (int kb = 0; kb < nkb; kb++) {
                if (ok && !mbar_wait_tries(full_bar(slot), phase, kStrTryHintNs, kStrTries)) ok = false;
                const int lc = kb * kStrKc + warp;
                if (ok && lc < nch)
                    mt_tile<CT, kReg>(base + (size_t)slot * kStrStageBytes, img + (size_t)lc * mt_img_bytes(CT),
                                      Breg, Mreg, warp, lane, ML, acc);
                __syncwarp();
                // a slot whose copy never arrived is not handed back
                if (ok && lane == 0) mbar_arrive(empty_bar(slot));
                if (++slot == R) {
                    slot = 0;
                    phase ^= 1u;
                }
            }
            // park the strip's sums; every NB strips (and at the end) the batch is added up
            float* dst = part + ((size_t)(si % NB) * kStrConsumers + warp) * 16 * T;
#pragma unroll
            for (int sg = 0; sg < NS; sg++) {
                dst[g * T + t + 4 * sg] = acc[sg][0];
                dst[(g + 8) * T + t + 4 * sg] = acc[sg][1];
            }
            if (si % NB == NB - 1 || si == ns - 1) flush(si, si % NB + 1);
        }
        if (!ok && lane == 0 && p.status) atomicOr(p.status, 1);
    }

    // ---- split K: the cluster's ranks' strip sums, added in rank order
    if (ks > 1) {
        constexpr int T = mt_tokens(CT);
        __syncwarp();
        cluster_sync();  // every rank's strip sums are parked
        if (warp < kStrConsumers) {
            const uint32_t res_u = smem_u32(res);
            for (int u = rank + ks * warp; u < ns * 8; u += ks * kStrConsumers) {
                const int si = u >> 3, gg = u & 7;
                float y0 = 0.0f, y1 = 0.0f;
                if (lane < T) {
                    const uint32_t a0 = res_u + (uint32_t)((((size_t)si * 16 + gg) * T + lane) * 4);
                    const uint32_t a1 = res_u + (uint32_t)((((size_t)si * 16 + gg + 8) * T + lane) * 4);
                    for (int q = 0; q < ks; q++) {
                        y0 += ld_cluster_f32(map_to_rank(a0, (uint32_t)q));
                        y1 += ld_cluster_f32(map_to_rank(a1, (uint32_t)q));
                    }
                }
                mt_emit(p, s0 + si, gg, lane, T, y0, y1, true);
            }
        }
        __syncwarp();
        cluster_sync();  // no rank leaves while others read its sums
    }
}

// ---- host side -------------------------------------------------------------
struct MtKey {
    const void* w;
    const void* s;
    const void* b;
    int n_out, n_in, sg_cols, dev;
    bool operator==(const MtKey& o) const {
        return w == o.w && s == o.s && b == o.b && n_out == o.n_out && n_in == o.n_in && sg_cols == o.sg_cols &&
               dev == o.dev;
    }
};
struct MtKeyHash {
    size_t operator()(const MtKey& k) const {
        size_t h = std::hash<const void*>()(k.w);
        h = h * 1000003u ^ std::hash<const void*>()(k.s);
        h = h * 1000003u ^ std::hash<const void*>()(k.b);
        h = h * 1000003u ^ (size_t)k.n_out * 31u ^ (size_t)k.n_in * 131u ^ (size_t)k.sg_cols ^ ((size_t)k.dev << 40);
        return h;
    }
};
struct MtMaps {
    CUtensorMap tw, tw1, ts, tb;
};

// Packed words as (32 words, rows, chunks) with 16-row boxes of 16 chunks
// (a stage) and of 1 chunk (a stage cut at a rank's range end); scales and
// biases as sg_cols x 16-row boxes.  Cached by (pointers, shape, device).
static bool mt_maps(const MtParams& p, int sg_cols, MtMaps* out) {
    static std::mutex mu;
    static std::unordered_map<MtKey, MtMaps, MtKeyHash> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    const MtKey key{p.w, p.sc, p.bi, p.n_out, p.n_in, sg_cols, dev};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return true;
    }
    MtMaps m;
    if (!make_map_chunks(&m.tw, p.w, p.n_out, p.n_in / 8, 16, kStrKc) ||
        !make_map_chunks(&m.tw1, p.w, p.n_out, p.n_in / 8, 16, 1) ||
        !make_map_2d_sw(&m.ts, p.sc, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, p.n_out, p.n_sg, sg_cols, 16,
                        sb_swizzle(sg_cols)) ||
        !make_map_2d_sw(&m.tb, p.bi, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, p.n_out, p.n_sg, sg_cols, 16,
                        sb_swizzle(sg_cols)))
        return false;
    if (cache.size() >= 4096) cache.clear();
    cache.emplace(key, m);
    *out = m;
    return true;
}

static int sm_count_mt() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    return n;
}

// Column tiles for a pass of m tokens: 2 (4 tokens) or 3 (8 tokens).
static int mt_ct(int m) { return m <= mt_tokens(2) ? 2 : 3; }
static const void* mt_kernel_of(int ct) {
    return ct == 2 ? (const void*)gemv_mt_kernel<2> : (const void*)gemv_mt_kernel<3>;
}

struct MtPlan {
    int ct, ks, n_clusters;
    MtLayout L;
};

// The K split and ring for a pass of m tokens: the split (1..8 ranks) with the
// fewest weight chunks on the busiest CTA (strips per cluster x chunks per
// rank), among those whose image fits beside a ring of at least 3 stages and
// whose clusters the device holds at once; the smaller split on a tie.
// False if none fits.
static bool mt_plan(int n_out, int n_in, int m, int sg_shift, MtPlan& pl) {
    static SplitPicker caps;
    const int align = 2 << sg_shift;
    const int n_strips = (n_out + 15) / 16, n_chunks = n_in / 256;
    const int sms = sm_count_mt();
    pl.ct = mt_ct(m);
    const void* kern = mt_kernel_of(pl.ct);
    long long best = -1;
    for (int ks = 1; ks <= 8 && ks <= n_chunks; ks++) {
        MtLayout L;
        L.ct = pl.ct;
        L.ks = ks;
        L.nch_max = 0;
        for (int r = 0; r < ks; r++)
            L.nch_max = std::max(L.nch_max, mt_chunk_start(r + 1, ks, n_chunks, align) -
                                                mt_chunk_start(r, ks, n_chunks, align));
        int n_clusters = std::min(n_strips, sms / ks);
        if (n_clusters <= 0) break;
        L.ns_max = (n_strips + n_clusters - 1) / n_clusters;
        L.ring = kMtMaxRing;
        while (L.ring > 3 && L.bytes() > kMtSmemTarget) L.ring--;
        if (L.bytes() > kMtSmemTarget) continue;
        if (mt_reg(pl.ct) && L.nch_max > kStrKc) continue;  // one chunk per warp
        if (ks > 1) {
            const int cap = caps.capacity(kern, kStrThreads, L.bytes(), (int)kMtSmemTarget, ks);
            if (cap <= 0) continue;
            if (cap < n_clusters) {
                n_clusters = cap;
                L.ns_max = (n_strips + n_clusters - 1) / n_clusters;
                L.ring = kMtMaxRing;
                while (L.ring > 3 && L.bytes() > kMtSmemTarget) L.ring--;
                if (L.bytes() > kMtSmemTarget) continue;
            }
        }
        const long long cost = (long long)L.ns_max * L.nch_max;
        if (best < 0 || cost < best) {
            best = cost;
            pl.ks = ks;
            pl.n_clusters = n_clusters;
            pl.L = L;
        }
    }
    return best >= 0;
}

template <int CT>
static int mt_launch_t(const MtMaps& m, const MtParams& prm, const MtPlan& pl, cudaStream_t st) {
    static PerDeviceOnce attr_once;
    if (smem_opt_in(attr_once, gemv_mt_kernel<CT>, (int)kMtSmemTarget) != cudaSuccess) return HQ4_ERR_LAUNCH;
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
    lc.gridDim = dim3((unsigned)pl.n_clusters, (unsigned)pl.ks, 1);
    lc.blockDim = dim3(kStrThreads);
    lc.dynamicSmemBytes = pl.L.bytes();
    lc.stream = st;
    lc.attrs = attr;
    lc.numAttrs = na;
    return cudaLaunchKernelEx(&lc, gemv_mt_kernel<CT>, m.tw, m.tw1, m.ts, m.tb, prm, pl.L) == cudaSuccess
               ? HQ4_OK
               : HQ4_ERR_LAUNCH;
}

static bool mt_shape_ok(int n_out, int n_in, int gs, int* sg_shift) {
    if (n_out <= 0 || n_in <= 0 || n_in % 256 || gs < 64 || gs % 64) return false;
    int s = 0;
    while ((64 << s) < gs) s++;
    if ((64 << s) != gs || s > 2 || (n_in / gs) % 8) return false;
    *sg_shift = s;
    return true;
}

int gemv_mt_pass(MtParams prm, int gs, cudaStream_t st, bool* used) {
    *used = false;
    int sgs = 0;
    if (prm.m <= 0 || prm.m > kMtMaxTok || !mt_shape_ok(prm.n_out, prm.n_in, gs, &sgs)) return HQ4_OK;
    if (prm.x_bf16 && prm.norm_w) return HQ4_OK;  // the norm prologue takes fp32 x
    if ((((uintptr_t)prm.sc | (uintptr_t)prm.bi) & 15) || ((uintptr_t)prm.w & 15) || ((uintptr_t)prm.x & 15) ||
        (prm.norm_w && ((uintptr_t)prm.norm_w & 15)) || (prm.x_stride % 8))
        return HQ4_OK;
    MtPlan pl;
    if (!mt_plan(prm.n_out, prm.n_in, prm.m, sgs, pl)) return HQ4_OK;
    prm.n_chunks = prm.n_in / 256;
    prm.sg_shift = sgs;
    prm.n_sg = prm.n_in / gs;
    prm.n_strips = (prm.n_out + 15) / 16;
    prm.ks = pl.ks;
    prm.n_clusters = pl.n_clusters;
    prm.status = status_word();
    MtMaps m;
    if (!mt_maps(prm, kStrSBCols >> sgs, &m)) return HQ4_OK;
    *used = true;
    return pl.ct == 2 ? mt_launch_t<2>(m, prm, pl, st) : mt_launch_t<3>(m, prm, pl, st);
}

bool gemv_mt_fits(int n_out, int n_in, int gs, int m) {
    int sgs = 0;
    MtPlan pl;
    return m > 0 && m <= kMtMaxTok && mt_shape_ok(n_out, n_in, gs, &sgs) && mt_plan(n_out, n_in, m, sgs, pl);
}

// Passes of 4 tokens (the register path): a prompt's passes read the
// weights more often than 8-token passes would, but each runs faster
// (measured 16.7 against 17.8 ms time to first token on the 7B-shape model).
int gemv_mt_tokens(MtParams prm, int gs, int m_total, cudaStream_t st, bool* used) {
    *used = false;
    constexpr int per = mt_tokens(2);
    if (m_total <= 0 || !gemv_mt_fits(prm.n_out, prm.n_in, gs, std::min(m_total, per))) return HQ4_OK;
    const size_t xe = prm.x_bf16 ? 2 : 4;  // bytes per x element
    for (int t0 = 0; t0 < m_total; t0 += per) {
        MtParams q = prm;
        q.m = std::min(per, m_total - t0);
        q.x = static_cast<const unsigned char*>(prm.x) + (size_t)t0 * prm.x_stride * xe;
        q.out = prm.out ? prm.out + (size_t)t0 * prm.out_stride : nullptr;
        q.residual = prm.residual ? prm.residual + (size_t)t0 * prm.out_stride : nullptr;
        q.q_out = prm.q_out ? prm.q_out + (size_t)t0 * prm.q_stride : nullptr;
        q.tok0 = prm.tok0 + t0;
        bool u = false;
        const int rc = gemv_mt_pass(q, gs, st, &u);
        if (rc) return rc;
        if (!u) return t0 == 0 ? HQ4_OK : HQ4_ERR_LAUNCH;  // the shape fits every pass once it fits one
        *used = true;
    }
    return HQ4_OK;
}

}  // namespace hq4
