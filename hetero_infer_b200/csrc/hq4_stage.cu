// The non-GEMV kernels of the qwen2 stage forward (hetero/cpu_model.py:164-368)
// and the C entry points that expose the stage's fused GEMV modes.
//
//  * embedding:  fp16 table row gather -> fp32 hidden state
//  * attention:  grouped-query SDPA over the KV cache, one CTA per
//                (query head, query token); causal when several tokens
//                (hetero/cpu_model.py:233-252)
//  * argmax:     greedy sampling, first index wins ties (numpy argmax,
//                hetero/backends.py:106-109)
//  * position:   the device-side token position the decode step reads, so a
//                whole step can be replayed as one CUDA graph
#include <algorithm>
#include <cfloat>

#include "hq4_attn.cuh"
#include "hq4_host.cuh"
#include "hq4_common.cuh"
#include "hq4_mt.cuh"
#include "hq4.h"

namespace hq4 {

// from hq4_gemv.cu
struct GemvM1Params;
int gemv_launch_stage(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                      const float* x, float* out, int n_out, int n_in, int gs, const float* row_add,
                      const float* residual, const float* norm_w, float eps, int mode, int q_strips,
                      int k_strips, int head_dim, int max_ctx, int tok, const int* pos,
                      const float* rope_cos, const float* rope_sin, float* q_out, float* k_cache,
                      float* v_cache, cudaStream_t st);
int check_device_cap();
int* status_word();

static cudaLaunchAttribute pdl_attr() {
    cudaLaunchAttribute a;
    a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a.val.programmaticStreamSerializationAllowed = 1;
    return a;
}

template <typename Kern, typename... Args>
static int launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchAttribute attr[1] = {pdl_attr()};
    cudaLaunchConfig_t lc = {};
    lc.gridDim = grid;
    lc.blockDim = block;
    lc.dynamicSmemBytes = smem;
    lc.stream = st;
    lc.attrs = attr;
    lc.numAttrs = 1;
    return cudaLaunchKernelEx(&lc, kern, args...) == cudaSuccess ? HQ4_OK : HQ4_ERR_LAUNCH;
}

// ---- embedding ---------------------------------------------------------------
// An id outside [0, vocab) reads nothing: its row is written as zeros and
// status bit 1 is set (the reference's table indexing raises there).
__global__ void embed_kernel(const __half* __restrict__ table, const int* __restrict__ ids, int n,
                             int hidden, int vocab, float* __restrict__ out, int* status) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.y;
    if (t >= n) return;
    const int id = ids[t];
    const bool ok = id >= 0 && id < vocab;
    if (!ok && blockIdx.x == 0 && threadIdx.x == 0 && status) atomicOr(status, 2);
    const __half* row = table + (size_t)(ok ? id : 0) * hidden;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x)
        out[(size_t)t * hidden + i] = ok ? __half2float(row[i]) : 0.0f;
}

// ---- attention ---------------------------------------------------------------
// CTA (head h, query token i): position p = *pos + i attends to keys [0, p],
// in the reference's order of operations (hetero/cpu_model.py:233-252):
// s = (q . k) * scale, s -= max, e = exp(s), e /= sum(e), out = sum_s e_s v_s.
// Decode is latency-bound (a few hundred keys, 28 heads), so every key's score
// is its own thread: a 4-chain fp32 dot over float4 rows of the K cache, with
// q broadcast from shared memory.  The value pass gives each thread a float4
// column of V and one of 8 key residues; the 8 partial sums are added in a
// fixed order (deterministic).  attention_row (hq4_attn.cuh) is the same
// arithmetic for the persistent decode kernel.
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(
    const float* __restrict__ q, const float* __restrict__ k_cache, const float* __restrict__ v_cache,
    float* __restrict__ out, int n_heads, int n_kv, int head_dim, int max_ctx, const int* __restrict__ pos,
    float scale) {
    extern __shared__ float sc[];  // [max positions]
    __shared__ float4 qs[64];      // head_dim <= 256
    __shared__ float red[kAttnThreads / 32];
    __shared__ float4 part[kAttnParts][64];
    pdl_launch_dependents();
    pdl_wait();
    const int h = blockIdx.x, i = blockIdx.y;
    const int kh = h / (n_heads / n_kv);
    const int p = *pos + i;
    if (p < 0 || p >= max_ctx) return;  // outside the cache: write nothing
    const int n = p + 1;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = kAttnThreads / 32;
    const int d4n = head_dim >> 2;  // float4 columns
    const float4* qh = reinterpret_cast<const float4*>(q + ((size_t)i * n_heads + h) * head_dim);
    const float4* kbase = reinterpret_cast<const float4*>(k_cache + (size_t)kh * max_ctx * head_dim);
    const float4* vbase = reinterpret_cast<const float4*>(v_cache + (size_t)kh * max_ctx * head_dim);
    for (int j = threadIdx.x; j < d4n; j += kAttnThreads) qs[j] = qh[j];
    __syncthreads();

    float mx = -FLT_MAX;
    for (int s = threadIdx.x; s < n; s += kAttnThreads) {
        const float4* kr = kbase + (size_t)s * d4n;
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        for (int j0 = 0; j0 < d4n; j0 += 8) {  // d4n is a multiple of 8: 8 loads in flight
            float4 kv[8];
#pragma unroll
            for (int u = 0; u < 8; u++) kv[u] = __ldg(kr + j0 + u);
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const float4 qv = qs[j0 + u];
                a0 = fmaf(qv.x, kv[u].x, a0);
                a1 = fmaf(qv.y, kv[u].y, a1);
                a2 = fmaf(qv.z, kv[u].z, a2);
                a3 = fmaf(qv.w, kv[u].w, a3);
            }
        }
        const float d = __fmul_rn(__fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3)), scale);
        sc[s] = d;
        mx = fmaxf(mx, d);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
    for (int j = 1; j < nw; j++) mx = fmaxf(mx, red[j]);
    __syncthreads();
    float sum = 0.0f;
    for (int s = threadIdx.x; s < n; s += kAttnThreads) {
        const float e = expf(__fsub_rn(sc[s], mx));
        sc[s] = e;
        sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    float tot = 0.0f;
    for (int j = 0; j < nw; j++) tot += red[j];
    for (int s = threadIdx.x; s < n; s += kAttnThreads) sc[s] = __fdiv_rn(sc[s], tot);
    __syncthreads();

    // out[d] = sum_s e_s v_s[d]: thread (column c, residue r) sums keys r, r+8, ...
    for (int c0 = 0; c0 < d4n; c0 += kAttnThreads / kAttnParts) {
        const int c = c0 + threadIdx.x % (kAttnThreads / kAttnParts);
        const int r = threadIdx.x / (kAttnThreads / kAttnParts);
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (c < d4n) {
            int s = r;
            for (; s + 3 * kAttnParts < n; s += 4 * kAttnParts) {  // four keys' loads in flight
                float4 v[4];
#pragma unroll
                for (int u = 0; u < 4; u++) v[u] = __ldg(vbase + (size_t)(s + u * kAttnParts) * d4n + c);
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const float e = sc[s + u * kAttnParts];
                    acc.x = fmaf(e, v[u].x, acc.x);
                    acc.y = fmaf(e, v[u].y, acc.y);
                    acc.z = fmaf(e, v[u].z, acc.z);
                    acc.w = fmaf(e, v[u].w, acc.w);
                }
            }
            for (; s < n; s += kAttnParts) {
                const float e = sc[s];
                const float4 v = __ldg(vbase + (size_t)s * d4n + c);
                acc.x = fmaf(e, v.x, acc.x);
                acc.y = fmaf(e, v.y, acc.y);
                acc.z = fmaf(e, v.z, acc.z);
                acc.w = fmaf(e, v.w, acc.w);
            }
            part[r][c - c0] = acc;
        }
        __syncthreads();
        if (r == 0 && c < d4n) {
            float4 o4 = part[0][c - c0];
#pragma unroll
            for (int k = 1; k < kAttnParts; k++) {
                const float4 t4 = part[k][c - c0];
                o4.x += t4.x;
                o4.y += t4.y;
                o4.z += t4.z;
                o4.w += t4.w;
            }
            reinterpret_cast<float4*>(out + ((size_t)i * n_heads + h) * head_dim)[c] = o4;
        }
        __syncthreads();
    }
}

// ---- int8 activation codec (hetero/transport.py:198-225) ----------------------
// The pipeline hand-off at half the bytes of fp16: per row an fp32 scale
// amax/127 (1 for an all-zero row) and int8 q = clip(rint(x / scale), +-127);
// decoded as fp16(q * scale).  Every step is one IEEE fp32 operation in the
// reference's order (max of |x|, division, round-half-even, clip; multiply,
// round to fp16), so both directions are bit-identical to the NumPy codec.
// Payload layout as the reference's bytes: [rows] fp32 scales, then
// [rows][cols] int8.  (Non-finite inputs are outside the codec's contract.)
constexpr int kCodecThreads = 256;

// kWire: each value is first rounded to fp16 and widened back, as the
// reference's engine encodes the fp16 wire array (NumpyBackend.to_wire,
// hetero/backends.py:100-101, then transport.encode, hetero/engine.py:97).
template <bool kWire>
__device__ __forceinline__ float codec_in(const float* xr, int i) {
    const float v = xr[i];
    return kWire ? __half2float(__float2half_rn(v)) : v;
}

template <bool kWire>
__global__ void __launch_bounds__(kCodecThreads) act_encode_i8_kernel(const float* __restrict__ x, int rows, int cols,
                                                                     unsigned char* __restrict__ payload) {
    __shared__ float red[kCodecThreads / 32];
    __shared__ float s_scale;
    pdl_launch_dependents();
    pdl_wait();
    const int r = blockIdx.x;
    const float* xr = x + (size_t)r * cols;
    float amax = 0.0f;
    for (int i = threadIdx.x; i < cols; i += kCodecThreads) amax = fmaxf(amax, fabsf(codec_in<kWire>(xr, i)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = red[0];
        for (int j = 1; j < kCodecThreads / 32; j++) m = fmaxf(m, red[j]);
        float sc = __fdiv_rn(m, 127.0f);
        if (sc == 0.0f) sc = 1.0f;
        s_scale = sc;
        reinterpret_cast<float*>(payload)[r] = sc;
    }
    __syncthreads();
    const float sc = s_scale;
    signed char* q = reinterpret_cast<signed char*>(payload + (size_t)rows * 4 + (size_t)r * cols);
    for (int i = threadIdx.x; i < cols; i += kCodecThreads) {
        const float v = fminf(fmaxf(rintf(__fdiv_rn(codec_in<kWire>(xr, i), sc)), -127.0f), 127.0f);
        q[i] = (signed char)(int)v;
    }
}

__global__ void __launch_bounds__(kCodecThreads) act_decode_i8_kernel(const unsigned char* __restrict__ payload,
                                                                     int rows, int cols, __half* __restrict__ out16,
                                                                     float* __restrict__ out32) {
    pdl_launch_dependents();
    pdl_wait();
    const float* scales = reinterpret_cast<const float*>(payload);
    const signed char* q = reinterpret_cast<const signed char*>(payload + (size_t)rows * 4);
    const size_t n = (size_t)rows * cols;
    for (size_t i = (size_t)blockIdx.x * kCodecThreads + threadIdx.x; i < n; i += (size_t)gridDim.x * kCodecThreads) {
        const __half h = __float2half_rn(__fmul_rn((float)q[i], scales[i / cols]));
        if (out16) out16[i] = h;
        if (out32) out32[i] = __half2float(h);
    }
}

// ---- argmax --------------------------------------------------------------------
// numpy argmax order (hetero/backends.py:106-109 calls z.argmax()): a NaN is
// above every number and the first NaN wins; otherwise the largest value,
// lowest index among equals (-inf included, so the result is always in
// [0, n)).  Writes the index to idx_out and, when given, to history[*pos]
// (the generated-token record).
constexpr int kArgmaxThreads = 1024;
constexpr int kArgmaxCluster = 8;  // CTAs (SMs) that split the vector

__device__ __forceinline__ bool argmax_before(float v, int i, float bv, int bi) {
    const bool vn = v != v, bn = bv != bv;
    if (vn || bn) return vn && (!bn || i < bi);
    return v > bv || (v == bv && i < bi);
}

// Numpy-order best of x[lo..hi) over the CTA; the result is valid in thread 0.
// (-inf, INT_MAX) loses to every element, so a thread that saw one element
// holds an index in [lo, hi).
__device__ __forceinline__ void cta_argmax(const float* __restrict__ x, int lo, int hi, float& best, int& bidx) {
    __shared__ float bv[kArgmaxThreads / 32];
    __shared__ int bi[kArgmaxThreads / 32];
    best = -INFINITY;
    bidx = 0x7fffffff;
    for (int i = lo + threadIdx.x; i < hi; i += kArgmaxThreads) {
        const float v = x[i];
        if (argmax_before(v, i, best, bidx)) {
            best = v;
            bidx = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
        if (argmax_before(ov, oi, best, bidx)) {
            best = ov;
            bidx = oi;
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        bv[warp] = best;
        bi[warp] = bidx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        best = bv[0];
        bidx = bi[0];
        for (int j = 1; j < kArgmaxThreads / 32; j++)
            if (argmax_before(bv[j], bi[j], best, bidx)) {
                best = bv[j];
                bidx = bi[j];
            }
    }
}

// Argmax over a thread-block cluster: CTA r of the cluster takes the r-th
// slice of x, then rank 0 combines the slices' pairs read over DSMEM (the
// pair order is total -- value, then lowest index, NaN first -- so the
// combination order does not change the result).  Outputs: either
// (idx_out [, val_out] [, history[*pos]]) or, with `pair`, the shard pair
// (value bits, offset + index) for a cross-rank all-gather.
__global__ void __launch_bounds__(kArgmaxThreads) argmax_cluster_kernel(
    const float* __restrict__ x, int n, int* __restrict__ idx_out, int* __restrict__ history, int hist_len,
    const int* __restrict__ pos, float* __restrict__ val_out, int* __restrict__ pair, int offset) {
    __shared__ float cbest;
    __shared__ int cidx;
    pdl_launch_dependents();
    pdl_wait();
    const int rank = (int)cluster_ctarank(), nr = (int)cluster_nctarank();
    const int chunk = (n + nr - 1) / nr;
    const int lo = min(n, rank * chunk), hi = min(n, lo + chunk);
    float best;
    int bidx;
    cta_argmax(x, lo, hi, best, bidx);
    if (threadIdx.x == 0) {
        cbest = best;
        cidx = bidx;
    }
    cluster_sync();  // every slice's pair written and visible across the cluster
    if (rank == 0 && threadIdx.x == 0) {
        for (int r = 1; r < nr; r++) {
            float v;
            int i;
            asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(map_to_rank(smem_u32(&cbest), r)) : "memory");
            asm volatile("ld.shared::cluster.b32 %0, [%1];" : "=r"(i) : "r"(map_to_rank(smem_u32(&cidx), r)) : "memory");
            if (argmax_before(v, i, best, bidx)) {
                best = v;
                bidx = i;
            }
        }
        if (pair) {
            pair[0] = __float_as_int(best);
            pair[1] = offset + bidx;
        } else {
            *idx_out = bidx;
            if (val_out) *val_out = best;
            if (history) {
                const int at = *pos;
                if (at >= 0 && at < hist_len) history[at] = bidx;
            }
        }
    }
    cluster_sync();  // the other CTAs' shared memory stays alive until rank 0 has read it
}

// The global greedy token from `world` shard pairs (value bits, global
// index): numpy argmax over the whole vocabulary (first NaN, else the largest
// value, lowest index among equals).  Optionally also recorded in
// history[slot].
__global__ void pick_token_kernel(const int* __restrict__ pairs, int world, int* __restrict__ tok,
                                  int* __restrict__ history, int slot, int* __restrict__ count, int hist_len) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x != 0) return;
    float best = -INFINITY;
    int bidx = 0x7fffffff;
    for (int w = 0; w < world; w++) {
        const float v = __int_as_float(pairs[2 * w]);
        const int i = pairs[2 * w + 1];
        if (argmax_before(v, i, best, bidx)) {
            best = v;
            bidx = i;
        }
    }
    *tok = bidx;
    if (count) {  // the slot is the device counter, which advances (a full history drops the token)
        const int s = *count;
        if (history && s >= 0 && s < hist_len) history[s] = bidx;
        *count = s + 1;
    } else if (history) {
        history[slot] = bidx;
    }
}

__global__ void advance_kernel(int* pos, int delta) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) *pos += delta;
}

}  // namespace hq4

using namespace hq4;

extern "C" int hq4_embed_f16(const uint16_t* table, const int* ids, int n_tokens, int hidden,
                             int vocab, float* out, void* stream) {
    if (int rc = check_device_cap()) return rc;
    if (n_tokens <= 0 || hidden <= 0 || vocab <= 0) return HQ4_ERR_SHAPE;
    int* status = status_word();
    if (!status) return HQ4_ERR_LAUNCH;
    return launch_pdl(embed_kernel, dim3(std::min(8, (hidden + 255) / 256), n_tokens), dim3(256), 0,
                      static_cast<cudaStream_t>(stream), reinterpret_cast<const __half*>(table), ids,
                      n_tokens, hidden, vocab, out, status);
}

extern "C" int hq4_attention(const float* q, const float* k_cache, const float* v_cache, float* out,
                             int n_heads, int n_kv, int head_dim, int max_ctx, const int* pos,
                             int n_tokens, float scale, void* stream) {
    if (int rc = check_device_cap()) return rc;
    if (n_heads <= 0 || n_kv <= 0 || n_heads % n_kv || head_dim % 32 || head_dim > 256 ||
        n_tokens <= 0 || max_ctx <= 0)
        return HQ4_ERR_SHAPE;
    if (((uintptr_t)q | (uintptr_t)k_cache | (uintptr_t)v_cache | (uintptr_t)out) & 15) return HQ4_ERR_ALIGN;
    const size_t smem = (size_t)max_ctx * sizeof(float);
    if (smem > 200 * 1024) return HQ4_ERR_SHAPE;
    static PerDeviceOnce attr_once;
    if (smem_opt_in(attr_once, attention_kernel, 200 * 1024) != cudaSuccess) return HQ4_ERR_LAUNCH;
    return launch_pdl(attention_kernel, dim3(n_heads, n_tokens), dim3(kAttnThreads), smem,
                      static_cast<cudaStream_t>(stream), q, k_cache, v_cache, out, n_heads, n_kv,
                      head_dim, max_ctx, pos, scale);
}

// ---- temperature / top-p sampling -----------------------------------------
// NumpyBackend.sample (hetero/backends.py:110-120) for temperature > 0, on a
// cluster of 8 CTAs that splits the vocabulary in contiguous slices held in
// shared memory: z = x / T; z -= max; p = exp(z) / sum; with top_p < 1 the
// nucleus -- the elements whose strictly larger elements hold less than
// top_p of the mass -- renormalised; then the draw of rng.choice for the
// caller's uniform variate u: the first index whose cumulative probability,
// divided by the total, exceeds u.  Every reduction runs in a fixed order and
// every CTA combines the 8 slice totals in rank order, so all CTAs agree.
// The nucleus bound is found by bisection on the bit patterns of the
// probabilities (non-negative floats order as their bits).  Sums differ from
// NumPy's only in rounding order; an exact tie in probability at the nucleus
// edge keeps every tied element (NumPy's unstable argsort keeps some).
constexpr int kSampleThreads = 1024;
constexpr int kSampleCluster = 8;

struct SampleShared {
    float red[kSampleThreads / 32];
    float cl[2];  // this CTA's slice total, double-buffered between reductions
    int icl[2];
    float bcast;
    int ibcast;
};

// Sum over the cluster of every thread's v: warp trees, the 32 warp sums in
// order, the 8 CTA sums in rank order.  `k` alternates the exchange buffer.
__device__ __forceinline__ float sample_cluster_sum(SampleShared& sh, float v, int& k) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) sh.red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = 0.0f;
        for (int w = 0; w < kSampleThreads / 32; w++) b += sh.red[w];
        sh.cl[k] = b;
    }
    cluster_sync();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int r = 0; r < kSampleCluster; r++) {
            float x;
            asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(x) : "r"(map_to_rank(smem_u32(&sh.cl[k]), r))
                         : "memory");
            t += x;
        }
        sh.bcast = t;
    }
    __syncthreads();
    k ^= 1;
    return sh.bcast;
}
__device__ __forceinline__ float sample_cluster_max(SampleShared& sh, float v, int& k) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) sh.red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = sh.red[0];
        for (int w = 1; w < kSampleThreads / 32; w++) b = fmaxf(b, sh.red[w]);
        sh.cl[k] = b;
    }
    cluster_sync();
    if (threadIdx.x == 0) {
        float t = -INFINITY;
        for (int r = 0; r < kSampleCluster; r++) {
            float x;
            asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(x) : "r"(map_to_rank(smem_u32(&sh.cl[k]), r))
                         : "memory");
            t = fmaxf(t, x);
        }
        sh.bcast = t;
    }
    __syncthreads();
    k ^= 1;
    return sh.bcast;
}
__device__ __forceinline__ int sample_cluster_min(SampleShared& sh, int v, int& k) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) sh.red[threadIdx.x >> 5] = __int_as_float(v);
    __syncthreads();
    if (threadIdx.x == 0) {
        int b = __float_as_int(sh.red[0]);
        for (int w = 1; w < kSampleThreads / 32; w++) b = min(b, __float_as_int(sh.red[w]));
        sh.icl[k] = b;
    }
    cluster_sync();
    if (threadIdx.x == 0) {
        int t = 0x7fffffff;
        for (int r = 0; r < kSampleCluster; r++) {
            int x;
            asm volatile("ld.shared::cluster.b32 %0, [%1];" : "=r"(x) : "r"(map_to_rank(smem_u32(&sh.icl[k]), r))
                         : "memory");
            t = min(t, x);
        }
        sh.ibcast = t;
    }
    __syncthreads();
    k ^= 1;
    return sh.ibcast;
}

__global__ void __launch_bounds__(kSampleThreads) sample_cluster_kernel(const float* __restrict__ x, int n, float temp,
                                                                       float top_p, double u, int* __restrict__ tok,
                                                                       int* status) {
    extern __shared__ float ps[];  // this CTA's slice of the distribution
    __shared__ SampleShared sh;
    pdl_launch_dependents();
    pdl_wait();
    const int rank = (int)cluster_ctarank();
    const int chunk = (n + kSampleCluster - 1) / kSampleCluster;
    const int lo = min(n, rank * chunk), cnt = min(n, lo + chunk) - lo;
    // thread t owns the contiguous run [t*E, t*E + E) of the slice
    const int E = (chunk + kSampleThreads - 1) / kSampleThreads;
    const int a = min(cnt, (int)threadIdx.x * E), b = min(cnt, a + E);
    int k = 0;
    float mx = -INFINITY;
    for (int i = a; i < b; i++) {
        const float z = __fdiv_rn(x[lo + i], temp);  // z = logits / temperature
        ps[i] = z;
        mx = fmaxf(mx, z);
    }
    mx = sample_cluster_max(sh, mx, k);
    float s = 0.0f;
    for (int i = a; i < b; i++) {
        const float e = expf(__fsub_rn(ps[i], mx));  // z -= z.max(); p = exp(z)
        ps[i] = e;
        s += e;
    }
    const float tot = sample_cluster_sum(sh, s, k);
    for (int i = a; i < b; i++) ps[i] = __fdiv_rn(ps[i], tot);  // p /= p.sum()
    if (top_p < 1.0f) {
        // smallest bit pattern c whose strictly larger probabilities hold less
        // than top_p: the nucleus is every p with bits >= c
        unsigned int lo_c = 0u, hi_c = 0x3F800001u;  // mass above hi_c (> 1.0f) is zero
        while (hi_c - lo_c > 1u) {
            const unsigned int mid = lo_c + ((hi_c - lo_c) >> 1);
            float m = 0.0f;
            for (int i = a; i < b; i++)
                if (__float_as_uint(ps[i]) > mid) m += ps[i];
            if (sample_cluster_sum(sh, m, k) < top_p) hi_c = mid;
            else lo_c = mid;
        }
        float m = 0.0f;
        for (int i = a; i < b; i++) {
            const float v = __float_as_uint(ps[i]) >= hi_c ? ps[i] : 0.0f;
            ps[i] = v;
            m += v;
        }
        const float kept = sample_cluster_sum(sh, m, k);
        for (int i = a; i < b; i++) ps[i] = __fdiv_rn(ps[i], kept);  // p = masked / masked.sum()
    }
    // the draw: cumulative probability in index order -- the thread's run in
    // order, after the runs before it (the CTA's threads, then the slices of
    // lower ranks) -- over its total, the first entry above u
    float run = 0.0f;
    for (int i = a; i < b; i++) run += ps[i];
    // exclusive prefix of the runs: warp scan, then the warps, then the CTAs
    float inc = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, inc, o);
        if ((threadIdx.x & 31) >= o) inc += y;
    }
    if ((threadIdx.x & 31) == 31) sh.red[threadIdx.x >> 5] = inc;
    __syncthreads();
    float before = inc - run;
    for (int w = 0; w < (int)(threadIdx.x >> 5); w++) before += sh.red[w];
    float cta_total = 0.0f;
    for (int w = 0; w < kSampleThreads / 32; w++) cta_total += sh.red[w];
    __syncthreads();
    if (threadIdx.x == 0) sh.cl[k] = cta_total;
    cluster_sync();
    float grand = 0.0f, lower = 0.0f;
    for (int r = 0; r < kSampleCluster; r++) {
        float y;
        asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(y) : "r"(map_to_rank(smem_u32(&sh.cl[k]), r))
                     : "memory");
        if (r < rank) lower += y;
        grand += y;
    }
    k ^= 1;
    int pick = 0x7fffffff;
    float c = lower + before;
    for (int i = a; i < b; i++) {
        c += ps[i];
        if ((double)__fdiv_rn(c, grand) > u) {
            pick = lo + i;
            break;
        }
    }
    pick = sample_cluster_min(sh, pick, k);
    if (rank == 0 && threadIdx.x == 0) {
        if (pick == 0x7fffffff || !(grand > 0.0f) || grand != grand) {
            // no entry above u (u >= 1) or no usable distribution (NaN logits)
            pick = n - 1;
            if (status && !(grand > 0.0f)) atomicOr(status, 8);
        }
        *tok = pick;
    }
    cluster_sync();  // the other CTAs' shared memory stays alive until every remote read is done
}

static int launch_argmax_cluster(cudaStream_t st, const float* x, int n, int* idx_out, int* history, int hist_len,
                                 const int* pos, float* val_out, int* pair, int offset) {
    cudaLaunchAttribute attr[2];
    attr[0] = pdl_attr();
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = kArgmaxCluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(kArgmaxCluster);
    lc.blockDim = dim3(kArgmaxThreads);
    lc.stream = st;
    lc.attrs = attr;
    lc.numAttrs = 2;
    return cudaLaunchKernelEx(&lc, argmax_cluster_kernel, x, n, idx_out, history, hist_len, pos, val_out, pair,
                              offset) == cudaSuccess
               ? HQ4_OK
               : HQ4_ERR_LAUNCH;
}

extern "C" int hq4_act_encode_i8(const float* x, int rows, int cols, void* payload, void* stream) {
    if (int rc = check_device_cap()) return rc;
    if (rows <= 0 || cols <= 0 || !x || !payload) return HQ4_ERR_SHAPE;
    if (((uintptr_t)x & 3) || ((uintptr_t)payload & 3)) return HQ4_ERR_ALIGN;
    return launch_pdl(act_encode_i8_kernel<false>, dim3(rows), dim3(kCodecThreads), 0,
                      static_cast<cudaStream_t>(stream), x, rows, cols, static_cast<unsigned char*>(payload));
}

extern "C" int hq4_act_encode_i8_wire(const float* x, int rows, int cols, void* payload, void* stream) {
    if (int rc = check_device_cap()) return rc;
    if (rows <= 0 || cols <= 0 || !x || !payload) return HQ4_ERR_SHAPE;
    if (((uintptr_t)x & 3) || ((uintptr_t)payload & 3)) return HQ4_ERR_ALIGN;
    return launch_pdl(act_encode_i8_kernel<true>, dim3(rows), dim3(kCodecThreads), 0,
                      static_cast<cudaStream_t>(stream), x, rows, cols, static_cast<unsigned char*>(payload));
}

extern "C" int hq4_act_decode_i8(const void* payload, int rows, int cols, uint16_t* out_f16, float* out_f32,
                                 void* stream) {
    if (int rc = check_device_cap()) return rc;
    if (rows <= 0 || cols <= 0 || !payload || (!out_f16 && !out_f32)) return HQ4_ERR_SHAPE;
    if (((uintptr_t)payload & 3) || ((uintptr_t)out_f16 & 1) || ((uintptr_t)out_f32 & 3)) return HQ4_ERR_ALIGN;
    const long long n = (long long)rows * cols;
    const int grid = (int)std::min<long long>((n + kCodecThreads - 1) / kCodecThreads, 1184);
    return launch_pdl(act_decode_i8_kernel, dim3(grid), dim3(kCodecThreads), 0, static_cast<cudaStream_t>(stream),
                      static_cast<const unsigned char*>(payload), rows, cols, reinterpret_cast<__half*>(out_f16),
                      out_f32);
}

extern "C" int hq4_argmax(const float* x, int n, int* idx_out, int* history, int hist_len,
                          const int* pos, float* val_out, void* stream) {
    if (int rc = check_device_cap()) return rc;
    if (n <= 0) return HQ4_ERR_SHAPE;
    if (history && (!pos || hist_len <= 0)) return HQ4_ERR_SHAPE;
    return launch_argmax_cluster(static_cast<cudaStream_t>(stream), x, n, idx_out, history, hist_len, pos, val_out,
                                 nullptr, 0);
}

extern "C" int hq4_sample(const float* x, int n, float temperature, float top_p, double u, int* tok,
                          void* stream) {
    if (int rc = check_device_cap()) return rc;
    if (n <= 0 || !x || !tok || !(temperature > 0.0f) || !(top_p > 0.0f)) return HQ4_ERR_SHAPE;
    const int chunk = (n + kSampleCluster - 1) / kSampleCluster;
    const size_t smem = (size_t)chunk * sizeof(float);
    if (smem > 200 * 1024) return HQ4_ERR_SHAPE;
    static PerDeviceOnce attr_once;
    if (smem_opt_in(attr_once, sample_cluster_kernel, 200 * 1024) != cudaSuccess) return HQ4_ERR_LAUNCH;
    cudaLaunchAttribute attr[2];
    attr[0] = pdl_attr();
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = kSampleCluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(kSampleCluster);
    lc.blockDim = dim3(kSampleThreads);
    lc.dynamicSmemBytes = smem;
    lc.stream = static_cast<cudaStream_t>(stream);
    lc.attrs = attr;
    lc.numAttrs = 2;
    return cudaLaunchKernelEx(&lc, sample_cluster_kernel, x, n, temperature, top_p, u, tok, status_word()) ==
                   cudaSuccess
               ? HQ4_OK
               : HQ4_ERR_LAUNCH;
}

extern "C" int hq4_argmax_pair(const float* x, int n, int offset, int* pair, void* stream) {
    if (int rc = check_device_cap()) return rc;
    if (n <= 0 || !pair) return HQ4_ERR_SHAPE;
    return launch_argmax_cluster(static_cast<cudaStream_t>(stream), x, n, nullptr, nullptr, 0, nullptr, nullptr, pair,
                                 offset);
}

extern "C" int hq4_pick_token(const int* pairs, int world, int* tok, int* history, int slot, void* stream) {
    if (int rc = check_device_cap()) return rc;
    if (world <= 0 || !tok || (history && slot < 0)) return HQ4_ERR_SHAPE;
    return launch_pdl(pick_token_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), pairs, world, tok,
                      history, slot, (int*)nullptr, 0);
}

extern "C" int hq4_pick_token_next(const int* pairs, int world, int* tok, int* history, int* count, int hist_len,
                                   void* stream) {
    if (int rc = check_device_cap()) return rc;
    if (world <= 0 || !tok || !count || hist_len < 0) return HQ4_ERR_SHAPE;
    return launch_pdl(pick_token_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), pairs, world, tok,
                      history, 0, count, hist_len);
}

extern "C" int hq4_advance_position(int* pos, int delta, void* stream) {
    if (int rc = check_device_cap()) return rc;
    return launch_pdl(advance_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), pos, delta);
}

extern "C" int hq4_gemv_norm(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                             const float* x, float* out, int n_out, int n_in, int gs, int m,
                             const float* norm_w, float eps, int silu_mul, const float* row_add,
                             const float* residual, void* stream) {
    if (int rc = check_device_cap()) return rc;
    if (m <= 0 || (silu_mul && n_out % 16)) return HQ4_ERR_SHAPE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int n_store = silu_mul ? n_out / 2 : n_out;
    if (m >= 2) {  // a prompt: the multi-token kernel, passes of up to 4 tokens
        MtParams mp = {};
        mp.w = w;
        mp.sc = scales;
        mp.bi = biases;
        mp.x = x;
        mp.x_stride = n_in;
        mp.out = out;
        mp.out_stride = n_store;
        mp.n_out = n_out;
        mp.n_in = n_in;
        mp.row_add = silu_mul ? nullptr : row_add;
        mp.residual = silu_mul ? nullptr : residual;
        mp.norm_w = norm_w;
        mp.eps = eps;
        mp.mode = silu_mul ? 1 : 0;  // kEpiSiluMul : kEpiPlain
        bool used = false;
        if (int rc = gemv_mt_tokens(mp, gs, m, st, &used)) return rc;
        if (used) return HQ4_OK;
    }
    for (int i = 0; i < m; i++) {
        int rc = gemv_launch_stage(w, scales, biases, x + (size_t)i * n_in, out + (size_t)i * n_store,
                                   n_out, n_in, gs, silu_mul ? nullptr : row_add,
                                   (residual && !silu_mul) ? residual + (size_t)i * n_out : nullptr, norm_w,
                                   eps, silu_mul ? 1 : 0, 0, 0, 0, 0, 0, nullptr, nullptr, nullptr,
                                   nullptr, nullptr, nullptr, st);
        if (rc) return rc;
    }
    return HQ4_OK;
}

extern "C" int hq4_qkv_rope(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                            const float* x, int n_heads, int n_kv, int head_dim, int n_in, int gs, int m,
                            const float* norm_w, float eps, const float* bias, const int* pos,
                            const float* rope_cos, const float* rope_sin, int max_ctx, float* q_out,
                            float* k_cache, float* v_cache, void* stream) {
    if (int rc = check_device_cap()) return rc;
    if (m <= 0 || head_dim % 16 || n_heads % n_kv) return HQ4_ERR_SHAPE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int half = head_dim / 2;
    const int q_strips = n_heads * half / 8, k_strips = n_kv * half / 8;
    const int n_out = (n_heads + 2 * n_kv) * head_dim;
    if (m >= 2) {  // a prompt: the multi-token kernel, passes of up to 4 tokens
        MtParams mp = {};
        mp.w = w;
        mp.sc = scales;
        mp.bi = biases;
        mp.x = x;
        mp.x_stride = n_in;
        mp.out = q_out;
        mp.out_stride = n_heads * head_dim;
        mp.n_out = n_out;
        mp.n_in = n_in;
        mp.row_add = bias;
        mp.norm_w = norm_w;
        mp.eps = eps;
        mp.mode = 2;  // kEpiQkvRope
        mp.q_strips = q_strips;
        mp.k_strips = k_strips;
        mp.head_dim = head_dim;
        mp.max_ctx = max_ctx;
        mp.pos = pos;
        mp.rope_cos = rope_cos;
        mp.rope_sin = rope_sin;
        mp.q_out = q_out;
        mp.q_stride = n_heads * head_dim;
        mp.k_cache = k_cache;
        mp.v_cache = v_cache;
        bool used = false;
        if (int rc = gemv_mt_tokens(mp, gs, m, st, &used)) return rc;
        if (used) return HQ4_OK;
    }
    for (int i = 0; i < m; i++) {
        int rc = gemv_launch_stage(w, scales, biases, x + (size_t)i * n_in, q_out, n_out, n_in, gs, bias,
                                   nullptr, norm_w, eps, 2, q_strips, k_strips, head_dim, max_ctx, i, pos,
                                   rope_cos, rope_sin, q_out + (size_t)i * n_heads * head_dim, k_cache,
                                   v_cache, st);
        if (rc) return rc;
    }
    return HQ4_OK;
}
