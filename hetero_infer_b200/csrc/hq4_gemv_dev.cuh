// Device-side pieces of the one-token GEMV shared by the streaming kernel
// (hq4_gemv.cu) and the persistent decode kernel (hq4_decode.cu): the launch
// parameters, the epilogues, and the streaming kernel's consumer steps (x
// image build, stage loop, strip totals).  Both kernels therefore compute
// every output with the same instructions in the same order.
#pragma once
#include "hq4_common.cuh"

namespace hq4 {

template <int KG>
struct M1 {
    static constexpr int kWords = KG / 8;        // packed words per group-row
    static constexpr int kKSteps = KG / 8;       // one word per row per k32 step
    static constexpr int kDigitBytes = KG;       // one s8 digit per value
    static constexpr int kBRegs = KG / 4;        // B registers per (group, digit)
    static constexpr int kImgStride = 3 * KG + 16;  // bytes per group: d2|d1|d0|(2^(E-22), xsum)|pad
    static constexpr int kMetaOff = 3 * KG;
};

struct GemvM1Params {
    const uint32_t* w;
    const uint16_t* sc;
    const uint16_t* bi;
    const float* x;
    float* out;
    int n_out, n_in;
    int ng;        // lane-groups per row (n_in / KG)
    int sg_shift;  // scale index = lane-group >> sg_shift
    int n_sg;      // scale groups per row (n_in / gs)
    int n_strips, nq;
    const float* row_add;   // optional: out[r] += row_add[r]
    const float* residual;  // optional: out[r] += residual[r]
    int* status;            // device status word; bit 0 set when a bounded wait ran out
    // optional RMSNorm of x before the product: x <- x * rsqrt(mean(x^2)+eps) * norm_w
    const float* norm_w;
    float eps;
    // epilogue mode
    int mode;               // kEpiPlain, kEpiSiluMul or kEpiQkvRope
    int x_bf16;             // streaming kernel only: x is bf16 (no RMSNorm then)
    int weights_after_wait; // read the weights only after the dependency wait (they may
                            // have been written by the preceding kernel)
    // kEpiQkvRope: q|k|v rows of one decoder layer, q and k rows permuted so
    // strip rows g and g+8 are the rotation pair (d, d + head_dim/2)
    int q_strips, k_strips, head_dim, max_ctx;
    int tok;                // token index inside this call (position = *pos + tok)
    const int* pos;         // device position of token 0
    const float* rope_cos;  // [max_ctx][head_dim/2]
    const float* rope_sin;
    float* q_out;           // [n_heads][head_dim], rotated
    float* k_cache;         // [n_kv][max_ctx][head_dim]
    float* v_cache;
};

enum : int { kEpiPlain = 0, kEpiSiluMul = 1, kEpiQkvRope = 2 };

// Inputs of a strip's store that do not depend on the product: the row add
// and residual of rows g and g+8, and for q|k|v the position and the RoPE
// rotation.  Loaded ahead (before the stage loop) so their latency hides
// behind the weight stream; applied by store_pair_in.
struct EpiIn {
    float a0, a1;  // row_add[r0], row_add[r1] (kEpiPlain, kEpiQkvRope)
    float r0, r1;  // residual[r0], residual[r1] (kEpiPlain)
    float c, sn;   // cos, sin of the rotation pair (kEpiQkvRope, q and k strips)
    int pos;       // *pos + tok (kEpiQkvRope)
};

__device__ __forceinline__ EpiIn epi_load(const GemvM1Params& p, int s, int g) {
    EpiIn e = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0};
    if (p.mode == kEpiPlain) {
        const int r0 = s * 16 + g, r1 = r0 + 8;
        if (p.row_add) {
            if (r0 < p.n_out) e.a0 = p.row_add[r0];
            if (r1 < p.n_out) e.a1 = p.row_add[r1];
        }
        if (p.residual) {
            if (r0 < p.n_out) e.r0 = p.residual[r0];
            if (r1 < p.n_out) e.r1 = p.residual[r1];
        }
    } else if (p.mode == kEpiQkvRope) {
        if (p.row_add) {
            e.a0 = p.row_add[s * 16 + g];
            e.a1 = p.row_add[s * 16 + g + 8];
        }
        e.pos = *p.pos + p.tok;
        if (e.pos >= 0 && e.pos < p.max_ctx && s < p.q_strips + p.k_strips) {
            const int half = p.head_dim >> 1;
            const int spp = half >> 3;  // strips per head (8 rotation pairs per strip)
            const int sl = s < p.q_strips ? s : s - p.q_strips;
            const int j = (sl % spp) * 8 + g;
            e.c = p.rope_cos[(size_t)e.pos * half + j];
            e.sn = p.rope_sin[(size_t)e.pos * half + j];
        }
    }
    return e;
}

__device__ __forceinline__ void store_row_in(const GemvM1Params& p, int r, float y, float add, float res) {
    if (r >= p.n_out) return;
    if (p.row_add) y += add;
    if (p.residual) y += res;
    p.out[r] = y;
}

// silu as the reference's NumPy stage writes it: x / (1 + exp(-x))
// (hetero/cpu_model.py:169-170), every operation rounded separately.
__device__ __forceinline__ float silu_ref(float x) {
    return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
}

// Store the finished pair of rows (g, g+8) of strip s according to the mode,
// with the inputs e = epi_load(p, s, g).
__device__ __forceinline__ void store_pair_in(const GemvM1Params& p, int s, int g, float y0, float y1,
                                              const EpiIn& e) {
    if (p.mode == kEpiPlain) {
        store_row_in(p, s * 16 + g, y0, e.a0, e.r0);
        store_row_in(p, s * 16 + g + 8, y1, e.a1, e.r1);
        return;
    }
    if (p.mode == kEpiSiluMul) {
        // strip s holds gate rows 8s..8s+7 (g) and the matching up rows (g+8)
        const int r = s * 8 + g;
        if (r < p.n_out / 2) p.out[r] = __fmul_rn(silu_ref(y0), y1);
        return;
    }
    // kEpiQkvRope
    if (p.row_add) {
        y0 = __fadd_rn(y0, e.a0);
        y1 = __fadd_rn(y1, e.a1);
    }
    const int half = p.head_dim >> 1;
    const int spp = half >> 3;  // strips per head (8 rotation pairs per strip)
    const int pos = e.pos;
    if (pos < 0 || pos >= p.max_ctx) return;  // outside the cache: write nothing
    if (s < p.q_strips + p.k_strips) {
        const bool is_q = s < p.q_strips;
        const int sl = is_q ? s : s - p.q_strips;
        const int head = sl / spp, j = (sl % spp) * 8 + g;
        const float c = e.c, sn = e.sn;
        // hetero/cpu_model.py:200-203: (x1*cos - x2*sin, x1*sin + x2*cos)
        const float o1 = __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, sn));
        const float o2 = __fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, c));
        float* dst = is_q ? p.q_out + (size_t)head * p.head_dim
                          : p.k_cache + ((size_t)head * p.max_ctx + pos) * p.head_dim;
        dst[j] = o1;
        dst[j + half] = o2;
    } else {
        const int r0 = (s - p.q_strips - p.k_strips) * 16 + g;  // natural v row order
        const int r1 = r0 + 8;
        const int head0 = r0 / p.head_dim, head1 = r1 / p.head_dim;
        p.v_cache[((size_t)head0 * p.max_ctx + pos) * p.head_dim + (r0 % p.head_dim)] = y0;
        p.v_cache[((size_t)head1 * p.max_ctx + pos) * p.head_dim + (r1 % p.head_dim)] = y1;
    }
}

__device__ __forceinline__ void store_pair(const GemvM1Params& p, int s, int g, float y0, float y1) {
    store_pair_in(p, s, g, y0, y1, epi_load(p, s, g));
}


// Strips [s0, s0 + ns) of CTA b when n strips are split over G CTAs: every
// CTA takes n / G, and the first n % G take one more.  A launch's CTAs start
// in index order as the previous kernel's CTAs leave their SMs (the last ones
// also behind a short kernel such as attention), so the extra strips go to
// the CTAs that start first.
__host__ __device__ __forceinline__ void str_strips(int b, int n, int G, int& s0, int& ns) {
    const int q = n / G, extra = n - q * G;
    s0 = b * q + (b < extra ? b : extra);
    ns = q + (b < extra ? 1 : 0);
}

constexpr int kStrConsumers = 16;
constexpr int kStrThreads = (kStrConsumers + 1) * kWarp;  // + one producer warp
constexpr int kStrKc = kStrConsumers;                      // k-chunks per stage (one per consumer warp)
constexpr int kStrTileBytes = 16 * 128;                    // 16 rows x 32 packed words
constexpr int kStrWBytes = kStrKc * kStrTileBytes;         // 32 KB
constexpr int kStrSBCols = kStrKc * 4;                     // scale groups per stage at gs 64
constexpr int kStrSBBytes = 16 * kStrSBCols * 2;           // 16 rows x up to 64 scale groups
constexpr int kStrStageBytes = kStrWBytes + 2 * kStrSBBytes;  // 36 KB (a multiple of 1024)
constexpr int kStrImgBytes = 4 * M1<64>::kImgStride;       // one k-chunk: 4 lane-groups
constexpr uint64_t kStrWaitNs = 1000000000ull;             // bounded waits: 1 s
constexpr uint32_t kStrTryHintNs = 10000;                  // consumer waits: 10 us per try_wait,
constexpr int kStrTries = 100000;                          // at most 1 s in all

// AND of v over the 512 consumer threads (named barrier 1; every consumer
// thread must arrive).
__device__ __forceinline__ bool consumers_and(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.and.pred p, 1, 512, q;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(r) : "r"((uint32_t)v) : "memory");
    return r != 0;
}

__device__ __forceinline__ uint4 lds128(const unsigned char* p) {
    return *reinterpret_cast<const uint4*>(p);
}

// ---- streaming consumer steps (512 consumer threads, warps 0-15) ----------

// Lane (bq = lane/8, bp = lane%8) holds values [8 bp, 8 bp + 8) of lane-group
// bq of a k-chunk.  x of chunk kc (zeros past the row end).
__device__ __forceinline__ void str_load_x(const GemvM1Params& p, int kc, int nk, int lane, float (&dst)[8]) {
    const int G = kc * 4 + (lane >> 3);
    if (kc < nk && G < p.ng && p.x_bf16) {  // bf16 widens to fp32 exactly
        const uint4 r = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.x) +
                                                        (size_t)kc * 256 + lane * 8);
        const uint32_t w4[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            dst[2 * i] = __uint_as_float(w4[i] << 16);
            dst[2 * i + 1] = __uint_as_float(w4[i] & 0xFFFF0000u);
        }
    } else if (kc < nk && G < p.ng) {
        const float4* src = reinterpret_cast<const float4*>(p.x + (size_t)kc * 256 + lane * 8);
        const float4 a = src[0], b = src[1];
        dst[0] = a.x; dst[1] = a.y; dst[2] = a.z; dst[3] = a.w;
        dst[4] = b.x; dst[5] = b.y; dst[6] = b.z; dst[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) dst[i] = 0.0f;
    }
}
// RMSNorm weights of chunk kc (ones past the row end).
__device__ __forceinline__ void str_load_nw(const GemvM1Params& p, int kc, int nk, int lane, float (&dst)[8]) {
    if (kc < nk && kc * 4 + (lane >> 3) < p.ng) {
        const float4* nw = reinterpret_cast<const float4*>(p.norm_w + (size_t)kc * 256 + lane * 8);
        const float4 c = nw[0], d = nw[1];
        dst[0] = c.x; dst[1] = c.y; dst[2] = c.z; dst[3] = c.w;
        dst[4] = d.x; dst[5] = d.y; dst[6] = d.z; dst[7] = d.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) dst[i] = 1.0f;
    }
}

// Digit image of chunk kc (k-block kb of this warp) from its x values
// (normalised first when `norm`).  Image format: per lane-group the digit
// blocks d2, d1, d0 of 64 bytes (four 16-byte units, one per word pair),
// then (2^(E-22), xsum).
__device__ __forceinline__ void str_build_chunk(const GemvM1Params& p, unsigned char* img_w, int kb, int kc,
                                                int lane, const float (&xin)[8], const float (&n8)[8], bool norm,
                                                float norm_r) {
    using C = M1<64>;
    const int bq = lane >> 3, bp = lane & 7;
    float xv[8];
#pragma unroll
    for (int i = 0; i < 8; i++) xv[i] = xin[i];
    if (norm && kc * 4 + bq < p.ng) {
#pragma unroll
        for (int i = 0; i < 8; i++) xv[i] = __fmul_rn(__fmul_rn(xv[i], norm_r), n8[i]);
    }
    float amax = 0.0f, s = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        amax = fmaxf(amax, fabsf(xv[i]));
        s += xv[i];
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        s += __shfl_xor_sync(0xffffffffu, s, o);
    }
    const int E = group_exponent(amax);
    const float up = exp2i(kXBits - E);
    uint32_t r[8];
#pragma unroll
    for (int k = 0; k < 8; k++) r[k] = digits3(xv[k], up);
    const uint32_t e01 = prmt(prmt(r[0], r[2], 0x5140), prmt(r[4], r[6], 0x5140), 0x5410);
    const uint32_t e11 = prmt(prmt(r[0], r[2], 0x5140), prmt(r[4], r[6], 0x5140), 0x7632);
    const uint32_t e21 = prmt(prmt(r[0], r[2], 0x0062), prmt(r[4], r[6], 0x0062), 0x5410);
    const uint32_t o01 = prmt(prmt(r[1], r[3], 0x5140), prmt(r[5], r[7], 0x5140), 0x5410);
    const uint32_t o11 = prmt(prmt(r[1], r[3], 0x5140), prmt(r[5], r[7], 0x5140), 0x7632);
    const uint32_t o21 = prmt(prmt(r[1], r[3], 0x0062), prmt(r[5], r[7], 0x0062), 0x5410);
    unsigned char* gb = img_w + (size_t)kb * kStrImgBytes + bq * C::kImgStride;
    // Each 16-byte unit of a digit block holds words 2i and 2i+1 of the
    // group as (even digits of 2i, even of 2i+1, odd of 2i, odd of 2i+1): the
    // B register pairs of the even-nibble and the odd-nibble MMA.  Neighbour
    // lanes (words 2i, 2i+1) swap halves so each stores 8 contiguous bytes.
    const bool odd_w = bp & 1;
    unsigned char* u = gb + (bp >> 1) * 16 + (odd_w ? 8 : 0);
    const uint32_t x2 = __shfl_xor_sync(0xffffffffu, odd_w ? e21 : o21, 1);
    const uint32_t x1 = __shfl_xor_sync(0xffffffffu, odd_w ? e11 : o11, 1);
    const uint32_t x0 = __shfl_xor_sync(0xffffffffu, odd_w ? e01 : o01, 1);
    *reinterpret_cast<uint2*>(u + 0 * 64) = odd_w ? make_uint2(x2, o21) : make_uint2(e21, x2);
    *reinterpret_cast<uint2*>(u + 1 * 64) = odd_w ? make_uint2(x1, o11) : make_uint2(e11, x1);
    *reinterpret_cast<uint2*>(u + 2 * 64) = odd_w ? make_uint2(x0, o01) : make_uint2(e01, x0);
    if (bp == 0) *reinterpret_cast<float2*>(gb + C::kMetaOff) = make_float2(exp2i(E - kXBits), s);
}

// RMSNorm factor 1/sqrt(mean(x^2)+eps) from the per-warp sums of squares:
// the 16 consumer warps' sums, parked in red[], added in warp order.  Uses
// named barrier 1 over the 512 consumer threads.
__device__ __forceinline__ float str_norm_combine(const GemvM1Params& p, float* red, float ss, int warp, int lane) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    asm volatile("bar.sync 1, 512;" ::: "memory");
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < kStrConsumers; i++) tot += red[i];
    const float mean = __fdiv_rn(tot, (float)p.n_in);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
}

// The GEMV prologue of a warp: its chunk images (k-chunk kb*16 + warp for
// kb < nkb) and, when p.norm_w is set, the RMSNorm of x applied first.  The
// x values a warp converts are the ones it sums for the norm, so the whole
// prologue costs one round trip to memory: every chunk's x (and norm
// weights) is requested before the first is used.  Sum of squares: each
// lane's 8 values per chunk in chunk order, the warp's xor tree, the warps
// in order (str_norm_combine).  Rows longer than the chunks a pass holds in
// registers (kProKb without the norm, kProKbNorm with it; a kernel with less
// register room takes smaller passes, the arithmetic is the same) take
// further passes.
template <int kProKb, int kProKbNorm>
__device__ __forceinline__ void str_prologue(const GemvM1Params& p, float* red, unsigned char* img_w, int nkb,
                                             int nk, int warp, int lane) {
    if (p.norm_w) {
        constexpr int U = kProKbNorm;
        float xr[U][8], nw[U][8];
        float ss = 0.0f;
        for (int kb0 = 0; kb0 < nkb; kb0 += U) {
#pragma unroll
            for (int u = 0; u < U; u++)
                if (kb0 + u < nkb) {
                    str_load_x(p, (kb0 + u) * kStrKc + warp, nk, lane, xr[u]);
                    str_load_nw(p, (kb0 + u) * kStrKc + warp, nk, lane, nw[u]);
                }
#pragma unroll
            for (int u = 0; u < U; u++)
                if (kb0 + u < nkb)
#pragma unroll
                    for (int i = 0; i < 8; i++) ss = fmaf(xr[u][i], xr[u][i], ss);
        }
        const float norm_r = str_norm_combine(p, red, ss, warp, lane);
        for (int kb0 = 0; kb0 < nkb; kb0 += U) {
            if (nkb > U) {  // the registers hold the last pass: reload this one
#pragma unroll
                for (int u = 0; u < U; u++)
                    if (kb0 + u < nkb) {
                        str_load_x(p, (kb0 + u) * kStrKc + warp, nk, lane, xr[u]);
                        str_load_nw(p, (kb0 + u) * kStrKc + warp, nk, lane, nw[u]);
                    }
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int kc = (kb0 + u) * kStrKc + warp;
                if (kb0 + u < nkb && kc < nk) str_build_chunk(p, img_w, kb0 + u, kc, lane, xr[u], nw[u], true, norm_r);
            }
        }
    } else {
        constexpr int U = kProKb;
        for (int kb0 = 0; kb0 < nkb; kb0 += U) {
            float xr[U][8];
#pragma unroll
            for (int u = 0; u < U; u++)
                if (kb0 + u < nkb) str_load_x(p, (kb0 + u) * kStrKc + warp, nk, lane, xr[u]);
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int kc = (kb0 + u) * kStrKc + warp;
                if (kb0 + u < nkb && kc < nk) str_build_chunk(p, img_w, kb0 + u, kc, lane, xr[u], xr[u], false, 1.0f);
            }
        }
    }
    __syncwarp();
}

// Lane sums of the (at most two) strips a CTA keeps in registers.
struct StrAcc {
    float r00, r01, r10, r11;
};

// Per-lane constants of the stage arithmetic (lane g = lane/4 owns rows g and
// g+8 of a tile, t = lane%4 its lane-group): which digit blocks of the x
// image feed its B registers, and where its scale and bias sit in a stage's
// swizzled scale/bias tiles.
struct StrLane {
    int g, t, role, off0, sbo0, sbo1;
};

__device__ __forceinline__ StrLane str_lane(const GemvM1Params& p, int warp, int lane) {
    StrLane L;
    L.g = lane >> 2;
    L.t = lane & 3;
    L.role = (L.g >> 1) == L.t ? (L.g & 1) + 1 : 0;  // 1: d2+d0, 2: d1, 0: none
    L.off0 = L.role == 1 ? 0 : 64;
    // scale/bias tiles carry the swizzle of their row width (128, 64 or 32 B)
    const int sb_cols = kStrSBCols >> p.sg_shift;
    const int sb_row = sb_cols * 2;
    const int sb_mask = (sb_row >> 4) - 1;  // 16-byte units per row - 1: 128 B: 7, 64 B: 3, 32 B: 1
    const int lg = (warp * 4 + L.t) >> p.sg_shift;  // scale group inside the stage
    auto sb_off = [&](int row) {
        const int o = row * sb_row + lg * 2;
        return o ^ (((o >> 7) & sb_mask) << 4);
    };
    L.sbo0 = sb_off(L.g);
    L.sbo1 = sb_off(L.g + 8);
    return L;
}

// The x side of a warp's tiles for one k-chunk: the lane's B fragments of
// the three digit blocks (zero where its column belongs to another lane-group
// or digit) and the group's (2^(E-22), xsum).  Loaded once per k-block and
// kept in registers across every strip of that k-block.
struct StrB {
    uint4 q0[4], q1[4];  // c0 columns (d2 | d1) and c1 columns (d0 | 0), word pairs 0..3
    float2 meta;
};

__device__ __forceinline__ void str_load_b(const StrLane& L, const unsigned char* img,
                                           const unsigned char* zero_blk, StrB& B) {
    using C = M1<64>;
    const unsigned char* gb = img + L.t * C::kImgStride;
    const uint4* src0 = reinterpret_cast<const uint4*>(L.role ? gb + L.off0 : zero_blk);
    const uint4* src1 = reinterpret_cast<const uint4*>(L.role == 1 ? gb + 128 : zero_blk);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        B.q0[i] = src0[i];
        B.q1[i] = src1[i];
    }
    B.meta = *reinterpret_cast<const float2*>(gb + C::kMetaOff);
}

// One stage's tile for this warp (k-chunk `warp` of the stage, x fragments B
// of that chunk): the lane's shares of rows g and g+8, zero when its
// lane-group lies past the row end (gok false).  Exact digit dots on the
// integer tensor cores, then scale * dot * 2^(E-22) + bias * xsum in fp32.
//
// A packed word gives two A registers with one mask each: the even nibbles
// (w & 0x0F0F0F0F) and the odd nibbles left in place, i.e. 16 x their value
// (w & 0xF0F0F0F0).  One MMA takes the even nibbles of words ks and ks+1
// against their x digits, another the odd ones; the odd chain's sums are
// exact multiples of 16 (|sum| < 2^20), so (odd >> 4) + even is the exact
// integer column dot, identical to unpacking both nibbles to 0..15.
__device__ __forceinline__ void str_tile(const StrLane& L, const unsigned char* st, const StrB& B, bool gok,
                                         int warp, float& a0f, float& a1f) {
    const int g = L.g, t = L.t;
    const unsigned char* wt = st + warp * kStrTileBytes;
    // rows g and g+8; 16-byte chunks 2t and 2t+1 of the row, swizzled
    const int c0 = ((2 * t) ^ g) << 4, c1 = ((2 * t + 1) ^ g) << 4;
    const uint4 ra = lds128(wt + g * 128 + c0), rb = lds128(wt + g * 128 + c1);
    const uint4 rc = lds128(wt + (g + 8) * 128 + c0), rd = lds128(wt + (g + 8) * 128 + c1);
    const uint32_t w0[8] = {ra.x, ra.y, ra.z, ra.w, rb.x, rb.y, rb.z, rb.w};
    const uint32_t w1[8] = {rc.x, rc.y, rc.z, rc.w, rd.x, rd.y, rd.z, rd.w};
    constexpr uint32_t kLo = 0x0F0F0F0Fu, kHi = 0xF0F0F0F0u;
    int c0l[4], c1l[4], c0h[4], c1h[4];
#pragma unroll
    for (int ks = 0; ks < M1<64>::kKSteps; ks += 2) {
        const uint4 q0 = B.q0[ks >> 1], q1 = B.q1[ks >> 1];
        const uint32_t l0 = w0[ks] & kLo, l1 = w1[ks] & kLo, l2 = w0[ks + 1] & kLo, l3 = w1[ks + 1] & kLo;
        const uint32_t h0 = w0[ks] & kHi, h1 = w1[ks] & kHi, h2 = w0[ks + 1] & kHi, h3 = w1[ks + 1] & kHi;
        if (ks == 0) {
            mma_u8s8_16832_first(c0l, l0, l1, l2, l3, q0.x, q0.y);
            mma_u8s8_16832_first(c1l, l0, l1, l2, l3, q1.x, q1.y);
            mma_u8s8_16832_first(c0h, h0, h1, h2, h3, q0.z, q0.w);
            mma_u8s8_16832_first(c1h, h0, h1, h2, h3, q1.z, q1.w);
        } else {
            mma_u8s8_16832(c0l, l0, l1, l2, l3, q0.x, q0.y);
            mma_u8s8_16832(c1l, l0, l1, l2, l3, q1.x, q1.y);
            mma_u8s8_16832(c0h, h0, h1, h2, h3, q0.z, q0.w);
            mma_u8s8_16832(c1h, h0, h1, h2, h3, q1.z, q1.w);
        }
    }
    const unsigned char* ss = st + kStrWBytes;
    const unsigned char* sbi = st + kStrWBytes + kStrSBBytes;
    a0f = 0.0f;
    a1f = 0.0f;
    if (gok) {
        // column dots (d2, d1, d0) of rows g and g+8
        const int d2a = c0l[0] + (c0h[0] >> 4), d1a = c0l[1] + (c0h[1] >> 4), d0a = c1l[0] + (c1h[0] >> 4);
        const int d2b = c0l[2] + (c0h[2] >> 4), d1b = c0l[3] + (c0h[3] >> 4), d0b = c1l[2] + (c1h[2] >> 4);
        const float dot0 = fmaf((float)d2a, 65536.0f, fmaf((float)d1a, 256.0f, (float)d0a));
        const float dot1 = fmaf((float)d2b, 65536.0f, fmaf((float)d1b, 256.0f, (float)d0b));
        const float s0 = h2f(*reinterpret_cast<const uint16_t*>(ss + L.sbo0));
        const float b0 = h2f(*reinterpret_cast<const uint16_t*>(sbi + L.sbo0));
        const float s1 = h2f(*reinterpret_cast<const uint16_t*>(ss + L.sbo1));
        const float b1 = h2f(*reinterpret_cast<const uint16_t*>(sbi + L.sbo1));
        a0f = fmaf(s0 * B.meta.x, dot0, 0.0f);
        a0f = fmaf(b0, B.meta.y, a0f);
        a1f = fmaf(s1 * B.meta.x, dot1, 0.0f);
        a1f = fmaf(b1, B.meta.y, a1f);
    }
}

// The stage loop of one GEMV: ns strips x nkb k-blocks through the ring
// (stages k-block-major, strip-minor), starting at ring position (slot,
// phase), which it advances.  `stages` is the ring's first stage, `full` /
// `empty` the barrier addresses of slot 0 (8 bytes apart).  A wait that
// runs out clears ok; a slot whose copy never arrived is not handed back.
// kHoistB keeps the x fragments of a k-block in registers across its strips
// (34 registers); without it they are reloaded per tile, for kernels with
// less register room.
template <bool kHoistB>
__device__ __forceinline__ void str_consume(const GemvM1Params& p, const unsigned char* stages, uint32_t full,
                                            uint32_t empty, int R, int& slot, uint32_t& phase, bool& ok, int ns,
                                            int nkb, int nk, const unsigned char* img_w,
                                            const unsigned char* zero_blk, float* partials, int ns_max, int warp,
                                            int lane, StrAcc& acc) {
    const StrLane L = str_lane(p, warp, lane);
    const int g = L.g, t = L.t;
    // CTAs with one or two strips keep each strip's lane sums in registers
    // across k-blocks; more strips go through the shared-memory slots per stage
    const bool regacc = ns <= 2;
    for (int kb = 0; kb < nkb; kb++) {
        const int kc = kb * kStrKc + warp;
        const bool active = kc < nk;
        const bool gok = kc * 4 + t < p.ng;
        const unsigned char* img = img_w + (size_t)kb * kStrImgBytes;
        StrB B;
        if (kHoistB && active) str_load_b(L, img, zero_blk, B);
        for (int j = 0; j < ns; j++) {
            if (ok && !mbar_wait_tries(full + 8u * slot, phase, kStrTryHintNs, kStrTries)) ok = false;
            if (ok && active) {
                float a0f, a1f;
                if (!kHoistB) str_load_b(L, img, zero_blk, B);
                str_tile(L, stages + (size_t)slot * kStrStageBytes, B, gok, warp, a0f, a1f);
                if (regacc) {
                    if (j == 0) {
                        acc.r00 += a0f;
                        acc.r01 += a1f;
                    } else {
                        acc.r10 += a0f;
                        acc.r11 += a1f;
                    }
                } else {
                    // sums over the 4 lanes t of rows g and g+8 in three steps:
                    // even t keeps row g, odd t row g+8, each taking its partner's
                    // share of that row, then the pair two lanes away; lane t=0
                    // ends with row g, t=1 with row g+8 (the additions of the
                    // plain xor tree, in the same order)
                    const bool odd = t & 1;
                    float keep = odd ? a1f : a0f;
                    keep += __shfl_xor_sync(0xffffffffu, odd ? a0f : a1f, 1);
                    keep += __shfl_xor_sync(0xffffffffu, keep, 2);
                    if (t < 2) partials[((size_t)warp * ns_max + j) * 16 + g + 8 * t] += keep;
                }
            }
            __syncwarp();
            // a slot whose copy never arrived is not handed back: the producer
            // then stops instead of reusing it under a copy still in flight
            if (ok && lane == 0) mbar_arrive(empty + 8u * slot);
            if (++slot == R) {
                slot = 0;
                phase ^= 1u;
            }
        }
    }
}

__device__ __forceinline__ void prefetch_l1(const void* ptr) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(ptr));
}

// Bring the inputs of this lane's first store in str_finish (strip s0 + warp,
// lanes t == 0) into L1 before the stage loop, so the store does not wait on
// L2 at the end: the row add and residual lines now, the RoPE lines once the
// position has arrived (str_epi_prefetch_late, after the prologue).  Returns
// the position for q|k|v (its load is in flight meanwhile).
__device__ __forceinline__ int str_epi_prefetch(const GemvM1Params& p, int ns, int s0, int warp, int lane) {
    if (warp >= ns || (lane & 3)) return 0;
    const int r0 = (s0 + warp) * 16 + (lane >> 2);
    if (p.row_add) prefetch_l1(p.row_add + r0);
    if (p.mode == kEpiPlain) {
        if (p.residual) prefetch_l1(p.residual + r0);
        if (p.row_add && r0 + 8 < p.n_out) prefetch_l1(p.row_add + r0 + 8);
        if (p.residual && r0 + 8 < p.n_out) prefetch_l1(p.residual + r0 + 8);
        return 0;
    }
    if (p.mode == kEpiQkvRope) return *p.pos + p.tok;
    return 0;
}
__device__ __forceinline__ void str_epi_prefetch_late(const GemvM1Params& p, int ns, int s0, int warp, int lane,
                                                      int pos) {
    if (p.mode != kEpiQkvRope || warp >= ns || (lane & 3)) return;
    const int s = s0 + warp;
    if (pos < 0 || pos >= p.max_ctx || s >= p.q_strips + p.k_strips) return;
    const int half = p.head_dim >> 1, spp = half >> 3;
    const int sl = s < p.q_strips ? s : s - p.q_strips;
    const int j = (sl % spp) * 8 + (lane >> 2);
    prefetch_l1(p.rope_cos + (size_t)pos * half + j);
    prefetch_l1(p.rope_sin + (size_t)pos * half + j);
}

// Strip totals: register sums parked in the warp's slots, then per strip the
// 16 warps' slots summed in a fixed order (lane t adds warps 4t..4t+3, then a
// fixed xor tree) and stored through the epilogue.  Deterministic, no
// atomics.  Named barrier 1 over the 512 consumer threads; nothing is stored
// when any warp of the CTA saw a wait run out.
__device__ __forceinline__ void str_finish(const GemvM1Params& p, float* partials, int ns, int ns_max, int s0,
                                           bool ok, const StrAcc& acc, int warp, int lane) {
    const int g = lane >> 2, t = lane & 3;
    if (ns <= 2) {
#pragma unroll
        for (int j = 0; j < 2; j++) {
            float a0f = j == 0 ? acc.r00 : acc.r10, a1f = j == 0 ? acc.r01 : acc.r11;
            a0f += __shfl_xor_sync(0xffffffffu, a0f, 1);
            a0f += __shfl_xor_sync(0xffffffffu, a0f, 2);
            a1f += __shfl_xor_sync(0xffffffffu, a1f, 1);
            a1f += __shfl_xor_sync(0xffffffffu, a1f, 2);
            if (j < ns && t == 0) {
                float* slotp = partials + ((size_t)warp * ns_max + j) * 16;
                slotp[g] = a0f;
                slotp[g + 8] = a1f;
            }
        }
    }
    asm volatile("bar.sync 1, 512;" ::: "memory");
    if (!__any_sync(0xffffffffu, !ok)) {
        for (int j = warp; j < ns; j += kStrConsumers) {
            float y0 = 0.0f, y1 = 0.0f;
#pragma unroll
            for (int k = 0; k < kStrConsumers / 4; k++) {
                const float* sl = partials + ((size_t)(t * (kStrConsumers / 4) + k) * ns_max + j) * 16;
                y0 += sl[g];
                y1 += sl[g + 8];
            }
            y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
            y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
            y1 += __shfl_xor_sync(0xffffffffu, y1, 1);
            y1 += __shfl_xor_sync(0xffffffffu, y1, 2);
            if (t == 0) store_pair(p, s0 + j, g, y0, y1);
        }
    }
}

}  // namespace hq4
