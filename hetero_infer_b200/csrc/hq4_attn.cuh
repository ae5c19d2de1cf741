// Grouped-query attention of one query row over the fp32 KV cache inside the
// persistent decode kernel (hq4_decode.cu).  The arithmetic, thread for
// thread, is attention_kernel's in hq4_stage.cu, so both give the same bits.
//
// Query (head h, token i): position p = *pos + i attends to keys [0, p], in the
// reference's order of operations (hetero/cpu_model.py:233-252):
// s = (q . k) * scale, s -= max, e = exp(s), e /= sum(e), out = sum_s e_s v_s.
// Decode is latency-bound (a few hundred keys, 28 heads), so every key's score
// is its own thread: a 4-chain fp32 dot over float4 rows of the K cache, with
// q broadcast from shared memory.  The value pass gives each thread a float4
// column of V and one of 8 key residues; the 8 partial sums are added in a
// fixed order (deterministic).
#pragma once
#include <cfloat>

#include "hq4_common.cuh"

namespace hq4 {

constexpr int kAttnThreads = 256;
constexpr int kAttnParts = 8;  // key residues in the value pass

// Shared memory: sc [max_ctx] scores, qs [64] the query row (head_dim <= 256),
// red [8] warp partials, part [kAttnParts][64] value-pass partials.
// The decode kernel's 512 consumer threads take part in the barriers (named
// barrier 1); threads 0-255 do the work.  The cache is read with coherent
// loads: it was written earlier in the same launch.
__device__ __forceinline__ void attn_sync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

__device__ __forceinline__ void attention_row(const float* q, const float* k_cache, const float* v_cache, float* out,
                                              int n_heads, int n_kv, int head_dim, int max_ctx, const int* pos,
                                              float scale, int h, int i, float* sc, float4* qs, float* red,
                                              float4* part) {
    const int kh = h / (n_heads / n_kv);
    const int p = *pos + i;
    if (p < 0 || p >= max_ctx) return;  // outside the cache: write nothing (uniform)
    const int n = p + 1;
    const bool worker = threadIdx.x < kAttnThreads;
    const int tid = worker ? (int)threadIdx.x : 0;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = kAttnThreads / 32;
    const int d4n = head_dim >> 2;  // float4 columns
    const float4* qh = reinterpret_cast<const float4*>(q + ((size_t)i * n_heads + h) * head_dim);
    const float4* kbase = reinterpret_cast<const float4*>(k_cache + (size_t)kh * max_ctx * head_dim);
    const float4* vbase = reinterpret_cast<const float4*>(v_cache + (size_t)kh * max_ctx * head_dim);
    if (worker)
        for (int j = tid; j < d4n; j += kAttnThreads) qs[j] = qh[j];
    attn_sync();

    float mx = -FLT_MAX;
    for (int s = worker ? tid : n; s < n; s += kAttnThreads) {
        const float4* kr = kbase + (size_t)s * d4n;
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        for (int j0 = 0; j0 < d4n; j0 += 8) {  // d4n is a multiple of 8: 8 loads in flight
            float4 kv[8];
#pragma unroll
            for (int u = 0; u < 8; u++) kv[u] = *(kr + j0 + u);
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
    if (lane == 0 && worker) red[warp] = mx;
    attn_sync();
    mx = red[0];
    for (int j = 1; j < nw; j++) mx = fmaxf(mx, red[j]);
    attn_sync();
    float sum = 0.0f;
    for (int s = worker ? tid : n; s < n; s += kAttnThreads) {
        const float e = expf(__fsub_rn(sc[s], mx));
        sc[s] = e;
        sum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0 && worker) red[warp] = sum;
    attn_sync();
    float tot = 0.0f;
    for (int j = 0; j < nw; j++) tot += red[j];
    for (int s = worker ? tid : n; s < n; s += kAttnThreads) sc[s] = __fdiv_rn(sc[s], tot);
    attn_sync();

    // out[d] = sum_s e_s v_s[d]: thread (column c, residue r) sums keys r, r+8, ...
    for (int c0 = 0; c0 < d4n; c0 += kAttnThreads / kAttnParts) {
        const int c = c0 + tid % (kAttnThreads / kAttnParts);
        const int r = tid / (kAttnThreads / kAttnParts);
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (worker && c < d4n) {
            int s = r;
            for (; s + 3 * kAttnParts < n; s += 4 * kAttnParts) {  // four keys' loads in flight
                float4 v[4];
#pragma unroll
                for (int u = 0; u < 4; u++) v[u] = *(vbase + (size_t)(s + u * kAttnParts) * d4n + c);
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
                const float4 v = *(vbase + (size_t)s * d4n + c);
                acc.x = fmaf(e, v.x, acc.x);
                acc.y = fmaf(e, v.y, acc.y);
                acc.z = fmaf(e, v.z, acc.z);
                acc.w = fmaf(e, v.w, acc.w);
            }
            part[r * 64 + (c - c0)] = acc;
        }
        attn_sync();
        if (worker && r == 0 && c < d4n) {
            float4 o4 = part[c - c0];
#pragma unroll
            for (int k = 1; k < kAttnParts; k++) {
                const float4 t4 = part[k * 64 + (c - c0)];
                o4.x += t4.x;
                o4.y += t4.y;
                o4.z += t4.z;
                o4.w += t4.w;
            }
            reinterpret_cast<float4*>(out + ((size_t)i * n_heads + h) * head_dim)[c] = o4;
        }
        attn_sync();
    }
}

}  // namespace hq4
