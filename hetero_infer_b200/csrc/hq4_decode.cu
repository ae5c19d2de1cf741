// Persistent decode: every decoder layer of a stage for one token in ONE
// cooperative launch (the device runtime of the qwen2 stage forward,
// hetero/cpu_model.py:280-310 per layer, decode step of
// hetero/coordinator.py:266-292).
//
// Why: one token's layer is five dependent steps (q|k|v GEMV, attention, o
// GEMV, gate|up GEMV, down GEMV).  As separate launches every boundary costs
// ~1.5-2 us in which the HBM stream stops: the next kernel's CTAs cannot start
// until the previous kernel's leave their SMs, and then need a DRAM round trip
// before the first weights arrive.  Here one CTA per SM stays resident for the
// whole step and runs the steps as phases separated by a grid barrier.  The
// weights do not depend on the activations, so the CTA's TMA producer keeps
// streaming the NEXT phases' weights into its shared-memory ring while the
// consumer warps wait at a barrier or run attention: the ring is the slack
// that carries the HBM stream across every phase boundary.
//
// Every output is computed by the same device code as the per-launch kernels
// (hq4_gemv_dev.cuh for the GEMV phases, hq4_attn.cuh for attention, with
// each CTA owning the same strips as the streaming kernel), so a decode step
// here gives the same bits as the five launches per layer.
//
// Roles in a CTA (544 threads): warps 0-15 consume (x images, integer MMA,
// epilogues, attention on threads 0-255); warp 16 lane 0 produces: phase
// descriptors (one bulk copy each, double-buffered) and weight stages (three
// tensor copies each, a ring of R stages).
//
// Grid barrier: a 64-bit arrival counter in a caller-visible workspace.  Each
// CTA adds 1 per barrier and waits until the counter reaches (barriers passed)
// x gridDim.x; waits are bounded by the global timer, and a CTA whose wait ran
// out raises an abort word the others poll, so a failure ends every CTA
// within one bound.  The last CTA to leave the kernel zeroes the words, so
// consecutive launches need no reset.
#include <cstdio>
#include <mutex>
#include <vector>

#include "hq4_attn.cuh"
#include "hq4_common.cuh"
#include "hq4_gemv_dev.cuh"
#include "hq4_tmap.cuh"
#include "hq4.h"

namespace hq4 {

int* status_word();      // hq4_gemv.cu
int check_device_cap();  // hq4_gemv.cu

enum : int { kPhGemv = 0, kPhAttn = 1 };

// One phase of the program, read by the kernel from global memory (one bulk
// copy per phase; the size is a multiple of 16 bytes).
struct alignas(16) DecPhase {
    GemvM1Params p;  // GEMV phase: the streaming kernel's parameters
    int kind;        // kPhGemv or kPhAttn
    int nkb;         // GEMV: k-blocks per strip
    // attention phase
    const float* q;
    const float* k_cache;
    const float* v_cache;
    float* out;
    const int* pos;
    int n_heads, n_kv, head_dim, max_ctx, n_tok;
    float scale;
};

struct DecSync {  // grid barrier words; all zero between launches
    unsigned long long arrive;
    unsigned int exit;
    unsigned int abort;
};

// Dynamic shared memory: [ring R x 36 KB][zero block 64 B][union][red 16 floats]
// [mbarriers: full R, empty R, desc_full 2, desc_empty 2].  The union holds a
// GEMV phase's chunk images and strip slots, or attention's scratch.
struct DecLayout {
    int ring;
    int union_bytes;
    __host__ __device__ size_t zero_off() const { return (size_t)ring * kStrStageBytes; }
    __host__ __device__ size_t uni_off() const { return zero_off() + 64; }
    __host__ __device__ size_t red_off() const { return uni_off() + (size_t)union_bytes; }
    __host__ __device__ size_t bar_off() const { return red_off() + kStrConsumers * sizeof(float); }
    __host__ __device__ size_t bytes() const { return bar_off() + (size_t)(2 * ring + 4) * 8 + 1024; }
};

constexpr uint64_t kDecBarrierNs = 1000000000ull;  // a grid barrier waits at most 1 s
constexpr int kDecMaxRing = 5;                     // stages, as many as shared memory allows

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned int ld_relaxed_u32(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Failure-path test hook, set on the host per plan (hq4_decode_plan_fault):
// CTA skip_cta withholds its arrival at the first grid barrier, which then
// never completes, and every barrier wait is bounded by barrier_ns.
struct DecFault {
    int skip_cta;               // -1: none
    unsigned long long barrier_ns;
};

__global__ void __launch_bounds__(kStrThreads, 1)
decode_kernel(const DecPhase* __restrict__ phases, const CUtensorMap* __restrict__ maps, int n_phases,
              DecSync* sy, int* status, const DecLayout L, const DecFault F) {
    extern __shared__ unsigned char smem_raw[];
    __shared__ DecPhase sd[2];  // descriptors of phases ph (slot ph & 1)
    __shared__ int sflag;
    const uint32_t raw_u = smem_u32(smem_raw);
    unsigned char* base = smem_raw + (((raw_u + 1023u) & ~1023u) - raw_u);
    const uint32_t base_u = smem_u32(base);
    const int R = L.ring;
    unsigned char* uni = base + L.uni_off();
    float* red = reinterpret_cast<float*>(base + L.red_off());
    const uint32_t bars = base_u + (uint32_t)L.bar_off();
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (R + s); };
    auto dfull_bar = [&](int b) { return bars + 8u * (2 * R + b); };
    auto dempty_bar = [&](int b) { return bars + 8u * (2 * R + 2 + b); };
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t G = gridDim.x;

    // ---- producer state (warp 16, lane 0).  Two cursors: dq, the next phase
    // descriptor to copy (slot dq & 1, free once the consumers have left phase
    // dq - 2), and the stage cursor (phase sp, k-block pkb, strip pjj), which
    // runs ahead on the ring and reads the phase shapes from global memory.
    // The descriptor copies are serviced inside every ring wait, so a full
    // ring never holds back the descriptor the consumers wait for.
    const bool producer = warp == kStrConsumers && lane == 0;
    int dq = 0;
    int sp = 0, pkb = 0, pjj = 0, ps0 = 0, pns = 0, pnkb = 0, pshift = 0;
    bool sp_open = false;
    int p_issued = 0, p_slot = 0, p_use = 0;
    uint64_t pol = 0;
    auto desc_ready = [&]() {
        return dq < 2 || mbar_try(dempty_bar(dq & 1), (uint32_t)((dq >> 1) - 1) & 1u);
    };
    auto service_desc = [&]() {
        while (dq < n_phases && desc_ready()) {
            const int b = dq & 1;
            mbar_arrive_expect_tx(dfull_bar(b), (uint32_t)sizeof(DecPhase));
            bulk_load_g2s(smem_u32(&sd[b]), phases + dq, (uint32_t)sizeof(DecPhase), dfull_bar(b),
                          l2_policy_evict_last());
            dq++;
        }
    };
    // Wait for `ready` while servicing descriptors; false after the time bound.
    auto wait_serving = [&](auto ready) -> bool {
        if (ready()) return true;
        const uint64_t t0 = globaltimer_ns();
        for (;;) {
            service_desc();
            __nanosleep(64);
            if (ready()) return true;
            if (globaltimer_ns() - t0 > kStrWaitNs) return false;
        }
    };
    // Issue descriptors and stages in program order; with may_wait false it
    // returns at the first slot that is not free yet.  False when a wait ran out.
    auto produce = [&](bool may_wait) -> bool {
        service_desc();
        while (sp < n_phases) {
            if (!sp_open) {
                const DecPhase& d = phases[sp];
                pns = 0;
                if (d.kind == kPhGemv) {
                    const int n = d.p.n_strips;
                    str_strips((int)blockIdx.x, n, (int)G, ps0, pns);
                    pnkb = d.nkb;
                    pshift = d.p.sg_shift;
                    if (pns > 0) {
                        prefetch_tensormap(maps + 3 * sp);
                        prefetch_tensormap(maps + 3 * sp + 1);
                        prefetch_tensormap(maps + 3 * sp + 2);
                    }
                }
                pkb = pjj = 0;
                sp_open = true;
            }
            while (pns > 0 && pkb < pnkb) {
                if (p_issued >= R) {  // slot p_slot's previous stage released by all 16 warps
                    const uint32_t bar = empty_bar(p_slot), par = (uint32_t)(p_use - 1) & 1u;
                    auto ready = [&]() { return mbar_try(bar, par); };
                    if (!may_wait) {
                        if (!ready()) {
                            service_desc();
                            return true;
                        }
                    } else if (!wait_serving(ready)) {
                        return false;
                    }
                }
                const CUtensorMap* tm = maps + 3 * sp;
                const int strip = ps0 + pjj, kc0 = pkb * kStrKc;
                const uint32_t sb_bytes = 16u * (uint32_t)(kStrSBCols >> pshift) * 2u;
                const uint32_t dst = base_u + (uint32_t)p_slot * kStrStageBytes;
                mbar_arrive_expect_tx(full_bar(p_slot), (uint32_t)kStrWBytes + 2u * sb_bytes);
                tma_load_3d(dst, tm, 0, strip * 16, kc0, full_bar(p_slot), pol);
                const int gx = (kc0 * 4) >> pshift;
                tma_load_2d(dst + kStrWBytes, tm + 1, gx, strip * 16, full_bar(p_slot), pol);
                tma_load_2d(dst + kStrWBytes + kStrSBBytes, tm + 2, gx, strip * 16, full_bar(p_slot), pol);
                p_issued++;
                if (++p_slot == R) {
                    p_slot = 0;
                    p_use++;
                }
                if (++pjj == pns) {
                    pjj = 0;
                    pkb++;
                }
            }
            sp++;
            sp_open = false;
            service_desc();
        }
        // every stage issued: the remaining descriptors, in order
        while (dq < n_phases) {
            if (!may_wait) {
                service_desc();
                return true;
            }
            if (!wait_serving([&]() { return dq >= n_phases || desc_ready(); })) return false;
            service_desc();
        }
        return true;
    };

    if (producer) {
        for (int s = 0; s < R; s++) {
            mbar_init_nofence(full_bar(s), 1);
            mbar_init_nofence(empty_bar(s), kStrConsumers);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init_nofence(dfull_bar(b), 1);
            mbar_init_nofence(dempty_bar(b), 1);
        }
        mbar_init_fence();
        pol = l2_policy_evict_first();  // weights are read once
        produce(false);                 // first descriptors and stages, before the CTA barrier
    }
    if (threadIdx.x < 4) reinterpret_cast<uint4*>(base + L.zero_off())[threadIdx.x] = make_uint4(0, 0, 0, 0);
    __syncthreads();  // barriers initialised, zero block written

    if (warp == kStrConsumers) {
        if (producer) {
            const bool ok = produce(true);
            if (!ok) {
                if (status) atomicOr(status, 1);
                atomicExch(&sy->abort, 1u);
            }
            // every issued copy lands before the CTA may exit; the last use of
            // each slot is its final phase, so its parity cannot alias
            for (int k = max(0, p_issued - R); k < p_issued; k++)
                if (!mbar_wait_nap(full_bar(k % R), (k / R) & 1, kStrWaitNs, 64) && status) atomicOr(status, 1);
            for (int k = max(0, dq - 2); k < dq; k++)
                if (!mbar_wait_nap(dfull_bar(k & 1), (k >> 1) & 1, kStrWaitNs, 64) && status) atomicOr(status, 1);
        }
    } else {
        // ---- consumers (warps 0-15; threadIdx.x in [0, 512))
        const unsigned char* zero_blk = base + L.zero_off();
        bool ok = true;
        int slot = 0;
        uint32_t phase = 0;
        for (int ph = 0; ph < n_phases; ph++) {
            const int b = ph & 1;
            if (ph > 0) {
                // grid barrier: the previous phase's outputs are visible everywhere
                ok = consumers_and(ok);
                if (threadIdx.x == 0) {
                    bool good = ok;
                    mbar_arrive(dempty_bar(b ^ 1));  // phase ph - 1's descriptor is no longer read
                    if (good) {
                        // the CTA's writes (ordered before this thread by the
                        // named barrier) are published by the release; the
                        // acquire below orders the next phase's reads
                        const unsigned long long target = (unsigned long long)ph * G;  // ph barriers
                        if (!(ph == 1 && (int)blockIdx.x == F.skip_cta)) red_release_add_u64(&sy->arrive, 1ull);
                        uint64_t t0 = 0;
                        for (uint32_t n = 1;; n++) {
                            if (ld_acquire_u64(&sy->arrive) >= target) break;
                            if (ld_relaxed_u32(&sy->abort)) {
                                good = false;
                                break;
                            }
                            if ((n & 15) == 0) {
                                const uint64_t now = globaltimer_ns();
                                if (t0 == 0) {
                                    t0 = now;
                                } else if (now - t0 > F.barrier_ns) {
                                    good = false;
                                    break;
                                }
                            }
                        }
                    }
                    if (!good) {
                        atomicExch(&sy->abort, 1u);
                        if (status) atomicOr(status, 1);
                    }
                    sflag = good ? 1 : 0;
                }
                asm volatile("bar.sync 1, 512;" ::: "memory");
                ok = sflag != 0;
                if (!ok) break;
            }
            if (!mbar_wait_tries(dfull_bar(b), (uint32_t)(ph >> 1) & 1u, kStrTryHintNs, kStrTries)) ok = false;
            if (!consumers_and(ok)) {
                if (threadIdx.x == 0) {
                    atomicExch(&sy->abort, 1u);
                    if (status) atomicOr(status, 1);
                }
                ok = false;
                break;
            }
            const DecPhase& d = sd[b];
            if (ph == n_phases - 1) pdl_launch_dependents();  // the next kernel may start its prologue
            if (d.kind == kPhAttn) {
                float* sc = reinterpret_cast<float*>(uni);
                float4* qs = reinterpret_cast<float4*>(uni + (((size_t)d.max_ctx * 4 + 15) & ~(size_t)15));
                float4* part = qs + 64;
                for (int r = blockIdx.x; r < d.n_heads * d.n_tok; r += (int)G)
                    attention_row(d.q, d.k_cache, d.v_cache, d.out, d.n_heads, d.n_kv, d.head_dim, d.max_ctx,
                                  d.pos, d.scale, r % d.n_heads, r / d.n_heads, sc, qs, red, part);
                continue;
            }
            const GemvM1Params& p = d.p;
            const int n = p.n_strips;
            int s0, ns;
            str_strips((int)blockIdx.x, n, (int)G, s0, ns);
            if (ns == 0) continue;
            const int ns_max = (int)((n + G - 1) / G);
            const int nk = (p.ng + 3) >> 2, nkb = d.nkb;
            unsigned char* img_w = uni + (size_t)warp * nkb * kStrImgBytes;
            float* partials = reinterpret_cast<float*>(uni + (size_t)kStrConsumers * nkb * kStrImgBytes);
            const int epi_pos = str_epi_prefetch(p, ns, s0, warp, lane);
            for (int i = threadIdx.x; i < kStrConsumers * ns_max * 16; i += kStrConsumers * kWarp) partials[i] = 0.0f;
            str_prologue<3, 1>(p, red, img_w, nkb, nk, warp, lane);  // the kernel's register room
            str_epi_prefetch_late(p, ns, s0, warp, lane, epi_pos);
            asm volatile("bar.sync 1, 512;" ::: "memory");  // slots cleared before any warp adds into them
            StrAcc acc = {0.0f, 0.0f, 0.0f, 0.0f};
            str_consume<false>(p, base, full_bar(0), empty_bar(0), R, slot, phase, ok, ns, nkb, nk, img_w, zero_blk,
                        partials, ns_max, warp, lane, acc);
            if (!ok && lane == 0 && status) atomicOr(status, 1);
            str_finish(p, partials, ns, ns_max, s0, ok, acc, warp, lane);
        }
        if (!ok && threadIdx.x == 0) atomicExch(&sy->abort, 1u);
    }

    // ---- leave: the last CTA out resets the barrier words for the next launch
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned int t = atomicAdd(&sy->exit, 1u);
        if (t == G - 1) {  // every CTA has passed every barrier
            atomicExch(&sy->arrive, 0ull);
            atomicExch(&sy->abort, 0u);
            __threadfence();
            atomicExch(&sy->exit, 0u);
        }
    }
}

// ---- host: the decode plan -------------------------------------------------
struct DecodePlan {
    int dev = -1;
    int n_phases = 0;
    int grid = 0;
    DecLayout L = {0, 0};
    DecPhase* d_phases = nullptr;
    CUtensorMap* d_maps = nullptr;
    DecSync* d_sync = nullptr;
    DecFault fault = {-1, kDecBarrierNs};
};

static size_t dec_smem_limit() {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) v = 227 * 1024;
    return (size_t)v - sizeof(DecPhase) * 2 - 64;  // the kernel's static shared memory
}

static int gemv_phase(DecPhase& ph, CUtensorMap* maps, const uint32_t* w, const uint16_t* sc, const uint16_t* bi,
                      int n_out, int n_in, int gs) {
    if (n_out <= 0 || n_in <= 0 || n_in % gs || gs < 64 || gs > 256 || (gs & (gs - 1))) return HQ4_ERR_SHAPE;
    const int n_sg = n_in / gs;
    if (n_in % 256 || n_sg % 8) return HQ4_ERR_SHAPE;  // whole k-chunks; 16-byte scale rows
    if (((uintptr_t)w & 31) || (((uintptr_t)sc | (uintptr_t)bi) & 15)) return HQ4_ERR_ALIGN;
    GemvM1Params& p = ph.p;
    p.w = w;
    p.sc = sc;
    p.bi = bi;
    p.n_out = n_out;
    p.n_in = n_in;
    p.ng = n_in / 64;
    p.sg_shift = gs == 64 ? 0 : gs == 128 ? 1 : 2;
    p.n_sg = n_sg;
    p.n_strips = (n_out + 15) / 16;
    p.nq = (p.ng + 3) / 4;
    p.status = status_word();
    ph.kind = kPhGemv;
    ph.nkb = ((p.ng + 3) / 4 + kStrKc - 1) / kStrKc;
    const int sg_cols = kStrSBCols >> p.sg_shift;
    if (!make_map_chunks(&maps[0], w, n_out, n_in / 8, 16, kStrKc) ||
        !make_map_2d_sw(&maps[1], sc, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, n_out, n_sg, sg_cols, 16,
                        sb_swizzle(sg_cols)) ||
        !make_map_2d_sw(&maps[2], bi, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, n_out, n_sg, sg_cols, 16,
                        sb_swizzle(sg_cols)))
        return HQ4_ERR_LAUNCH;
    return HQ4_OK;
}

static void free_plan(DecodePlan* pl) {
    if (!pl) return;
    int cur = 0;
    cudaGetDevice(&cur);
    if (pl->dev >= 0) cudaSetDevice(pl->dev);
    cudaFree(pl->d_phases);
    cudaFree(pl->d_maps);
    cudaFree(pl->d_sync);
    cudaSetDevice(cur);
    delete pl;
}

}  // namespace hq4

using namespace hq4;

extern "C" int hq4_decode_plan_create(const hq4_decode_layer* layers, int n_layers, int hidden, int n_heads,
                                      int n_kv, int head_dim, int intermediate, int gs, float eps, float attn_scale,
                                      const float* rope_cos, const float* rope_sin, int max_ctx, float* h,
                                      const int* pos, float* q_buf, float* attn_buf, float* mlp_buf, void** plan) {
    if (!plan) return HQ4_ERR_SHAPE;
    *plan = nullptr;
    if (int rc = check_device_cap()) return rc;
    if (!layers || n_layers <= 0 || hidden <= 0 || n_heads <= 0 || n_kv <= 0 || n_heads % n_kv ||
        head_dim % 32 || head_dim > 256 || intermediate <= 0 || max_ctx <= 0 || !h || !pos || !q_buf ||
        !attn_buf || !mlp_buf || !rope_cos || !rope_sin)
        return HQ4_ERR_SHAPE;
    if (((uintptr_t)h | (uintptr_t)q_buf | (uintptr_t)attn_buf | (uintptr_t)mlp_buf) & 15) return HQ4_ERR_ALIGN;
    const int nq = n_heads * head_dim, nkv = n_kv * head_dim;
    const int n_phases = 5 * n_layers;
    std::vector<DecPhase> ph(n_phases);
    std::vector<CUtensorMap> maps((size_t)3 * n_phases);
    memset(ph.data(), 0, sizeof(DecPhase) * ph.size());
    memset(maps.data(), 0, sizeof(CUtensorMap) * maps.size());
    int union_bytes = 0;
    int G = 0;
    {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&G, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || G <= 0)
            return HQ4_ERR_LAUNCH;
    }
    auto gemv_union = [&](const DecPhase& d) {
        const int ns_max = (d.p.n_strips + G - 1) / G;
        return kStrConsumers * d.nkb * kStrImgBytes + kStrConsumers * ns_max * 16 * (int)sizeof(float);
    };
    for (int l = 0; l < n_layers; l++) {
        const hq4_decode_layer& y = layers[l];
        if (!y.input_norm || !y.post_norm || !y.k_cache || !y.v_cache ||
            (((uintptr_t)y.input_norm | (uintptr_t)y.post_norm | (uintptr_t)y.k_cache | (uintptr_t)y.v_cache) & 15))
            return HQ4_ERR_ALIGN;
        DecPhase* P = &ph[5 * l];
        CUtensorMap* M = &maps[(size_t)15 * l];
        int rc;
        // q|k|v: RMSNorm prologue, bias + RoPE + cache append epilogue
        if ((rc = gemv_phase(P[0], M + 0, y.qkv_w, y.qkv_s, y.qkv_b, nq + 2 * nkv, hidden, gs))) return rc;
        GemvM1Params& a = P[0].p;
        a.x = h;
        a.out = q_buf;
        a.row_add = y.qkv_bias;
        a.norm_w = y.input_norm;
        a.eps = eps;
        a.mode = kEpiQkvRope;
        a.q_strips = nq / 16;
        a.k_strips = nkv / 16;
        a.head_dim = head_dim;
        a.max_ctx = max_ctx;
        a.tok = 0;
        a.pos = pos;
        a.rope_cos = rope_cos;
        a.rope_sin = rope_sin;
        a.q_out = q_buf;
        a.k_cache = y.k_cache;
        a.v_cache = y.v_cache;
        // attention
        DecPhase& t = P[1];
        t.kind = kPhAttn;
        t.q = q_buf;
        t.k_cache = y.k_cache;
        t.v_cache = y.v_cache;
        t.out = attn_buf;
        t.pos = pos;
        t.n_heads = n_heads;
        t.n_kv = n_kv;
        t.head_dim = head_dim;
        t.max_ctx = max_ctx;
        t.n_tok = 1;
        t.scale = attn_scale;
        // o + residual
        if ((rc = gemv_phase(P[2], M + 6, y.o_w, y.o_s, y.o_b, hidden, nq, gs))) return rc;
        P[2].p.x = attn_buf;
        P[2].p.out = h;
        P[2].p.residual = h;
        P[2].p.mode = kEpiPlain;
        // gate|up (interleaved): RMSNorm prologue, silu(gate) * up epilogue
        if ((rc = gemv_phase(P[3], M + 9, y.gate_up_w, y.gate_up_s, y.gate_up_b, 2 * intermediate, hidden, gs)))
            return rc;
        P[3].p.x = h;
        P[3].p.out = mlp_buf;
        P[3].p.norm_w = y.post_norm;
        P[3].p.eps = eps;
        P[3].p.mode = kEpiSiluMul;
        // down + residual
        if ((rc = gemv_phase(P[4], M + 12, y.down_w, y.down_s, y.down_b, hidden, intermediate, gs))) return rc;
        P[4].p.x = mlp_buf;
        P[4].p.out = h;
        P[4].p.residual = h;
        P[4].p.mode = kEpiPlain;
        for (int k : {0, 2, 3, 4}) union_bytes = std::max(union_bytes, gemv_union(P[k]));
    }
    // attention scratch: scores, the query row, the value-pass partials
    const int attn_bytes = (int)(((size_t)max_ctx * 4 + 15) & ~(size_t)15) + 64 * 16 + kAttnParts * 64 * 16;
    union_bytes = std::max(union_bytes, attn_bytes);
    DecLayout L = {kDecMaxRing, (union_bytes + 15) & ~15};
    const size_t limit = dec_smem_limit();
    while (L.ring > 2 && L.bytes() > limit) L.ring--;
    if (L.bytes() > limit) return HQ4_ERR_SHAPE;  // rows too long or the context too large for one CTA

    DecodePlan* pl = new DecodePlan();
    cudaGetDevice(&pl->dev);
    pl->n_phases = n_phases;
    pl->L = L;
    int per_sm = 0;
    if (cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.bytes()) !=
            cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_kernel, kStrThreads, L.bytes()) !=
            cudaSuccess ||
        per_sm < 1) {
        delete pl;
        return HQ4_ERR_LAUNCH;
    }
    pl->grid = G;  // one CTA per SM, all resident (cooperative launch)
    if (cudaMalloc(&pl->d_phases, sizeof(DecPhase) * n_phases) != cudaSuccess ||
        cudaMalloc(&pl->d_maps, sizeof(CUtensorMap) * maps.size()) != cudaSuccess ||
        cudaMalloc(&pl->d_sync, sizeof(DecSync)) != cudaSuccess ||
        cudaMemcpy(pl->d_phases, ph.data(), sizeof(DecPhase) * n_phases, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(pl->d_maps, maps.data(), sizeof(CUtensorMap) * maps.size(), cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        cudaMemset(pl->d_sync, 0, sizeof(DecSync)) != cudaSuccess) {
        free_plan(pl);
        return HQ4_ERR_LAUNCH;
    }
    *plan = pl;
    return HQ4_OK;
}

extern "C" int hq4_decode_plan_run(void* plan, void* stream) {
    DecodePlan* pl = static_cast<DecodePlan*>(plan);
    if (!pl) return HQ4_ERR_SHAPE;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != pl->dev) return HQ4_ERR_DEVICE;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(pl->grid);
    lc.blockDim = dim3(kStrThreads);
    lc.dynamicSmemBytes = pl->L.bytes();
    lc.stream = static_cast<cudaStream_t>(stream);
    lc.attrs = attr;
    lc.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&lc, decode_kernel, (const DecPhase*)pl->d_phases,
                                             (const CUtensorMap*)pl->d_maps, pl->n_phases, pl->d_sync,
                                             status_word(), pl->L, pl->fault);
    return e == cudaSuccess ? HQ4_OK : HQ4_ERR_LAUNCH;
}

extern "C" int hq4_decode_plan_fault(void* plan, int skip_cta, long long barrier_ns) {
    DecodePlan* pl = static_cast<DecodePlan*>(plan);
    if (!pl || skip_cta >= pl->grid) return HQ4_ERR_SHAPE;
    pl->fault.skip_cta = skip_cta < 0 ? -1 : skip_cta;
    pl->fault.barrier_ns = barrier_ns > 0 ? (unsigned long long)barrier_ns : kDecBarrierNs;
    return HQ4_OK;
}

extern "C" int hq4_decode_plan_info(void* plan, int* info) {
    DecodePlan* pl = static_cast<DecodePlan*>(plan);
    if (!pl || !info) return HQ4_ERR_SHAPE;
    info[0] = pl->grid;
    info[1] = pl->L.ring;
    info[2] = (int)pl->L.bytes();
    info[3] = pl->n_phases;
    return HQ4_OK;
}

extern "C" void hq4_decode_plan_destroy(void* plan) { free_plan(static_cast<DecodePlan*>(plan)); }
