/* hq4 -- B200 (sm_100a) int4 GEMV / dequant kernels behind a C ABI.
 *
 * Drop-in device-side replacement for the reference's native kernel,
 * hetero-infer kernel/q4gemv.c, which its NumPy backend binds through ctypes
 * (hetero/cpu_model.py:33-45).  Plain pointers and sizes only: every pointer
 * argument is a CUDA device pointer unless stated otherwise, `stream` is a
 * cudaStream_t passed as void*, and every call is asynchronous on it.
 *
 * Weight layout (identical to the reference, kernel/q4gemv.c:7-11):
 *   w       [n_out][n_in/8]   uint32, eight 4-bit values, low nibble first
 *   scales  [n_out][n_in/gs]  IEEE fp16 bits
 *   biases  [n_out][n_in/gs]  IEEE fp16 bits
 *   value = q * scale + bias
 *
 * Return codes follow the reference convention (0 ok, -1 bad shape) with
 * further negative codes for the device side.
 */
#ifndef HQ4_H
#define HQ4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HQ4_OK 0
#define HQ4_ERR_SHAPE (-1)     /* n_in % gs, unsupported gs, n_out/n_in/m <= 0 */
#define HQ4_ERR_ALIGN (-2)     /* w not 32-byte aligned, x not 16-byte, out not 4-byte */
#define HQ4_ERR_LAUNCH (-4)    /* a CUDA launch failed (cudaGetLastError) */
#define HQ4_ERR_DEVICE (-5)    /* current device is not sm_100 */

/* Library version, (major << 16) | minor. */
int hq4_version(void);

/* Device status word of the current device (synchronising): bit 0 is set
 * when a kernel's bounded wait (a bulk copy or pipeline barrier) ran out --
 * that kernel's output is not valid; bit 1 when hq4_embed_f16 met a token id
 * outside [0, vocab) -- that row was written as zeros; bit 2 when
 * hq4_gemm_w4a16 met an activation outside fp16 range; bit 3 when hq4_sample
 * met logits without a usable distribution (NaN).  Non-zero `clear`
 * resets it.  No counterpart in the reference: its CPU kernel cannot stall,
 * its table indexing raises IndexError on a bad id, and it computes in fp32. */
int hq4_device_status(int clear);

/* out[m][n_out] = x[m][n_in] . W^T with W dequantised on the fly.
 * Replaces  int q4_gemv(w, scales, biases, x, out, n_out, n_in, gs, nthreads)
 * (kernel/q4gemv.c:232-233): same pointer order and shape arguments; the
 * host thread count becomes the token count m and the CUDA stream.
 * x and out are fp32 row-major.  Supported gs: 32, and 64 * 2^k.
 * Needs no workspace; the x row must fit one CTA's shared memory
 * (n_in up to ~64K values).
 * Arithmetic: exact nibble dequantisation, products exact in fp32, per-group
 * fp32 scale and bias as the reference's float path (kernel/q4gemv.c:113-139,
 * 177-181): results match it to fp32 summation-order rounding. */
int hq4_gemv(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
             const float* x, float* out, int n_out, int n_in, int gs, int m, void* stream);

/* hq4_gemv with the projection's epilogue fused into the store:
 *   out[i][r] = (x[i] . W[r]) + row_add[r] + residual[i][r]
 * row_add (length n_out, e.g. the q/k/v bias of hetero/cpu_model.py:156-157)
 * and residual ([m][n_out], the decoder's residual stream,
 * hetero/cpu_model.py:305-306) may each be NULL.  out may alias residual. */
int hq4_gemv_fused(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                   const float* x, float* out, int n_out, int n_in, int gs, int m,
                   const float* row_add, const float* residual, void* stream);

/* hq4_gemv_fused with launch options.  No reference counterpart (the
 * reference's q4_gemv is synchronous).  hq4_gemv and hq4_gemv_fused start
 * streaming the weights before waiting for the preceding kernel on the
 * stream (programmatic dependent launch): only x, the residual and the
 * outputs are ordered after it.  A caller whose weights were written by the
 * kernel immediately before (a repack, a dequantise-requantise, an upload
 * kernel) passes HQ4_GEMV_WEIGHTS_AFTER_WAIT, and the weights are then read
 * only after that kernel has completed.  Unknown flag bits: -1. */
#define HQ4_GEMV_WEIGHTS_AFTER_WAIT 1
int hq4_gemv_ex(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, const float* x,
                float* out, int n_out, int n_in, int gs, int m, const float* row_add,
                const float* residual, int flags, void* stream);

/* hq4_gemv_fused with the activations and outputs in host memory, the
 * calling convention of q4_gemv itself (kernel/q4gemv.c:232: host x and out,
 * the call returns when out is written).  The weights stay on the device;
 * x_host [m][n_in] is copied to x_dev, the product (+ row_add) is written to
 * out_dev and copied to out_host, and the call waits for `stream`.  x_dev and
 * out_dev are caller-owned device buffers of at least m*n_in and m*n_out
 * floats; pinned host buffers keep the copies at full speed.  When out_host
 * is pinned and mapped for the device (cudaHostAlloc / pinned tensors), the
 * kernel writes the products into it directly and out_dev is not used; when
 * x_host is pinned and mapped (and 16-byte aligned), a small kernel fetches
 * it into x_dev instead of a copy, and the GEMV streams its first weights
 * while that kernel runs. */
int hq4_gemv_host(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                  const float* row_add, const float* x_host, float* out_host, int n_out, int n_in,
                  int gs, int m, float* x_dev, float* out_dev, void* stream);

/* Rows [row0,row1) of W expanded to fp32 into out [row1-row0][n_in].
 * Replaces  int q4_dequant(w, scales, biases, out, row0, row1, n_in, gs,
 * nthreads)  (kernel/q4gemv.c:359-360).  Bit-exact with the reference. */
int hq4_dequant(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                float* out, int row0, int row1, int n_in, int gs, void* stream);

/* W4A16 GEMM on the tcgen05 tensor cores for token counts where the product
 * is a dense contraction (microbatched decode, prefill):
 *   out[t][n] = sum_k x[t][k] * (q[n][k]*scales[n][g] + biases[n][g])
 *               (+ row_add[n]) (+ residual[t][n])
 * Replaces QLinear._gemm (hetero/cpu_model.py:118-136: q4_dequant of 512-row
 * blocks, kernel/q4gemv.c:311-379, then a BLAS matmul).  Weight layout as
 * hq4_gemv; x is [m][n_in] bf16 (x_is_f32 = 0) or fp32 (x_is_f32 = 1), 16-byte
 * aligned; out fp32 [m][n_out].  One token goes through hq4_gemv's
 * streaming kernel when the shape suits it (x widened to fp32, exact
 * digits).  Up to 16 bf16 (8 fp32) tokens the weights
 * stay exact (128+q in bf16 MMAs, the scale and bias folded per group in
 * fp32) and fp32 x is carried as bf16 hi + lo (16 significant bits); above,
 * the tcgen05 kernel rounds the weights once to fp16 and converts x to fp16
 * (exact for bf16 x with |x| < 65520; larger magnitudes set status bit 2).
 * Products and sums are fp32.  gs must be a power of two >= 64
 * dividing n_in (the reference's AVX2 build has the same gs % 64 rule,
 * q4gemv.c:234-240), else -1.
 * `workspace` (caller-owned, 128-byte aligned, at least
 * hq4_gemm_workspace_bytes(n_out, n_in, m) bytes, else -1) receives the fp16
 * activations in the tensor cores' tile layout; two calls in flight at once
 * must not share it.  Deterministic; allocates nothing. */
int hq4_gemm_w4a16(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, const void* x,
                   int x_is_f32, float* out, int n_out, int n_in, int gs, int m,
                   const float* row_add, const float* residual, void* workspace,
                   long long workspace_bytes, void* stream);

/* Workspace bytes hq4_gemm_w4a16 needs for a shape (host only; -1 for a bad
 * shape).  No reference counterpart: the reference dequantises into a
 * NumPy buffer it allocates per call (cpu_model.py:125-134). */
long long hq4_gemm_workspace_bytes(int n_out, int n_in, int m);

/* Launch plan hq4_gemm_w4a16 would use (no launch): info[0..7] = row tiles,
 * K-split cluster size, token tiles, tokens per tile, activation stages,
 * shared memory bytes, packed-weight ring slots, kernel (0: tcgen05 with the
 * A operand in TMEM, for larger token counts; 1: warp-level MMAs with the
 * weights exact as 128+q in bf16, for up to 16 bf16 / 8 fp32 tokens; 2: one
 * token through the streaming GEMV of hq4_gemv, info[0..6] then 0 -- reported
 * for group size 64 with 16-byte aligned scales and biases, which that kernel
 * needs; other one-token calls take kernel 1; 3: 2..8 tokens through the
 * multi-token streaming kernel, the one-token kernel's exact digit product
 * with the tokens sharing each weight fragment, info[0..6] then 0 --
 * reported for group size 64 where n_in is a multiple of 256 and the x
 * image fits shared memory; kernels 1 and 0 take the rest).  No reference
 * counterpart. */
int hq4_gemm_plan(int n_out, int n_in, int m, int x_is_f32, int* info);

/* hq4_gemm_w4a16 without a caller workspace: the workspace is a fixed
 * HQ4_GEMM_STATIC_SCRATCH_BYTES area of the library's static device memory,
 * one per device, so the call allocates nothing and needs no buffer from the
 * caller.  Shapes whose hq4_gemm_workspace_bytes(n_out, n_in, m) exceeds that
 * size return -1.  All calls on a device share the area: calls ordered on one
 * stream are safe; calls that can run at the same time (different streams,
 * host threads without a common stream) race on it and must be serialised by
 * the caller.  The first call on each device resolves the area's address
 * (cudaGetSymbolAddress, which may load the module) and must be made outside
 * stream capture.  No reference counterpart. */
#define HQ4_GEMM_STATIC_SCRATCH_BYTES (16ll << 20)
int hq4_gemm_w4a16_static(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                          const void* x, int x_is_f32, float* out, int n_out, int n_in, int gs,
                          int m, const float* row_add, const float* residual, void* stream);

/* ---- qwen2 stage forward (hetero/cpu_model.py:164-368) ---------------------
 * Hidden states, KV cache and attention are fp32 as in the reference's NumPy
 * stage.  `pos` is a device int: the position of the call's first token
 * (the reference's KVCache.offset, cpu_model.py:207-230); it lets a whole
 * decode step be replayed as one CUDA graph. */

/* out[t] = fp32(table[ids[t]]) for an fp16 embedding table [vocab][hidden];
 * ids is a device int array of n_tokens.  An id outside [0, vocab) reads
 * nothing: its row is zeros and status bit 1 is set (hq4_device_status). */
int hq4_embed_f16(const uint16_t* table, const int* ids, int n_tokens, int hidden,
                  int vocab, float* out, void* stream);

/* GEMV with RMSNorm of x fused into its prologue (cpu_model.py:164-166):
 *   x' = (x * (1/sqrt(mean(x^2) + eps))) * norm_w          (norm_w may be NULL)
 * silu_mul = 0: out[m][n_out] = x'.W^T (+ row_add) (+ residual)
 * silu_mul = 1: W holds gate and up rows interleaved per 16-row strip (rows
 *   0-7 = gate rows 8s..8s+7, rows 8-15 = up rows 8s..8s+7) and
 *   out[m][n_out/2] = silu(gate) * up  (cpu_model.py:169-170, 291-292). */
int hq4_gemv_norm(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                  const float* x, float* out, int n_out, int n_in, int gs, int m,
                  const float* norm_w, float eps, int silu_mul, const float* row_add,
                  const float* residual, void* stream);

/* The attention block's input projections for m tokens at positions
 * *pos .. *pos+m-1 (cpu_model.py:269-278): RMSNorm(x) . [Wq;Wk;Wv]^T + bias,
 * rotary embedding of q and k (half-split, cos/sin tables [max_ctx][head_dim/2]
 * built on the host as cpu_model.py:173-204 builds them), k and v appended to
 * the caches [n_kv][max_ctx][head_dim], rotated q written to q_out
 * [m][n_heads][head_dim].  W/scales/biases/bias rows are q, k, v concatenated
 * with the q and k rows of each head permuted so that every 16-row strip
 * holds 8 rotation pairs: rows 0-7 = dims j..j+7, rows 8-15 = dims
 * j+hd/2..j+hd/2+7 (j = 0, 8, ..., hd/2-8). */
int hq4_qkv_rope(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                 const float* x, int n_heads, int n_kv, int head_dim, int n_in, int gs, int m,
                 const float* norm_w, float eps, const float* bias, const int* pos,
                 const float* rope_cos, const float* rope_sin, int max_ctx, float* q_out,
                 float* k_cache, float* v_cache, void* stream);

/* Grouped-query attention for n_tokens queries q [n_tokens][n_heads][head_dim]
 * at positions *pos + i over cache entries [0, *pos + i] (causal), scores
 * scaled by `scale`, fp32 softmax (cpu_model.py:233-252); out has the layout
 * of q. head_dim a multiple of 32 up to 256; max_ctx * 4 bytes <= 200 KB.
 * Queries whose position is outside [0, max_ctx) write nothing (likewise the
 * cache writes of hq4_qkv_rope). */
int hq4_attention(const float* q, const float* k_cache, const float* v_cache, float* out,
                  int n_heads, int n_kv, int head_dim, int max_ctx, const int* pos,
                  int n_tokens, float scale, void* stream);

/* int8 activation codec, the reference's pipeline hand-off at half the bytes
 * of fp16 (hetero/transport.py:198-225).  payload = [rows] fp32 scales then
 * [rows][cols] int8 -- byte for byte what transport.encode(x, "int8")
 * returns as its payload.  encode: scale = max|x_row| / 127 (1 for an
 * all-zero row), q = clip(rint(x / scale), -127, 127).  decode: fp16(q *
 * scale) into out_f16 and/or, widened exactly, into out_f32 (either may be
 * NULL, not both).  Bit-identical to the NumPy codec for finite inputs. */
int hq4_act_encode_i8(const float* x, int rows, int cols, void* payload, void* stream);
int hq4_act_decode_i8(const void* payload, int rows, int cols, uint16_t* out_f16, float* out_f32,
                      void* stream);

/* The int8 frame the reference's engine sends (hetero/engine.py:97:
 * transport.encode(backend.to_wire(y), "int8")): every value of the fp32
 * hidden state x is rounded to fp16 first (NumpyBackend.to_wire,
 * hetero/backends.py:100-101), then encoded as hq4_act_encode_i8 does. */
int hq4_act_encode_i8_wire(const float* x, int rows, int cols, void* payload, void* stream);

/* Greedy sampling (hetero/backends.py:106-109): numpy argmax of x[0..n) --
 * the first NaN if there is one, else the largest value, lowest index among
 * equals (the result is always in [0, n)) -- written to *idx_out; also to history[*pos] when
 * history is not NULL and 0 <= *pos < hist_len; the largest value to *val_out
 * when val_out is not NULL (a row-sharded head reduces (value, index) pairs). */
int hq4_argmax(const float* x, int n, int* idx_out, int* history, int hist_len, const int* pos,
               float* val_out, void* stream);

/* Temperature / top-p sampling (hetero/backends.py:110-120, temperature > 0;
 * temperature 0 is hq4_argmax): z = x / temperature, p = exp(z - max z) /
 * sum; with top_p < 1 only the nucleus is kept (every probability whose
 * strictly larger probabilities hold less than top_p of the mass) and
 * renormalised; then the draw rng.choice(n, p=p) makes for the uniform
 * variate u in [0, 1) -- the caller draws u = rng.random() from the same
 * generator, so the generator advances as the reference's does -- written to
 * *tok.  n up to 8 x 51200.  Sums are fp32 in a fixed order that differs from
 * NumPy's, so a draw can differ only where u falls within rounding of a
 * cumulative boundary.  Non-finite logits set status bit 3.  -1 for
 * temperature <= 0 or top_p <= 0. */
int hq4_sample(const float* x, int n, float temperature, float top_p, double u, int* tok, void* stream);

/* Fill an fp16 [vocab][hidden] table with the benchmark's counter-based
 * synthetic N(0, std) embedding (seeded; see hetero_infer_b200/synth.py,
 * which evaluates the same rows on the host).  No reference counterpart: the
 * reference loads its embedding from a checkpoint. */
int hq4_synth_embed_f16(long long seed, int vocab, int hidden, float std, uint16_t* out,
                        void* stream);

/* One shard of a row-sharded greedy pick (hetero/backends.py:106-109 over a
 * vocabulary split across ranks): pair[0] = float bits of the numpy-order best
 * of x[0..n), pair[1] = offset + its index.  For an all-gather of pairs. */
int hq4_argmax_pair(const float* x, int n, int offset, int* pair, void* stream);

/* The greedy token from `world` gathered pairs (hq4_argmax_pair): numpy argmax
 * over the whole vocabulary -- the first NaN, else the largest value with the
 * lowest index.  Written to *tok and, when history is not NULL, to
 * history[slot].  No reference counterpart (the reference samples one
 * unsharded logits vector on the host). */
int hq4_pick_token(const int* pairs, int world, int* tok, int* history, int slot, void* stream);

/* hq4_pick_token whose history slot is a device counter: writes the token to
 * *tok and to history[*count] (when *count < hist_len), then advances
 * *count, so a CUDA graph that holds the call appends one token per replay.
 * No reference counterpart (the reference appends on the host). */
int hq4_pick_token_next(const int* pairs, int world, int* tok, int* history, int* count, int hist_len,
                        void* stream);

/* *pos += delta on the device (advances the decode position inside a graph). */
int hq4_advance_position(int* pos, int delta, void* stream);

/* ---- persistent decode ----------------------------------------------------
 * One token through n_layers qwen2 decoder layers (hetero/cpu_model.py:280-310
 * per layer) as ONE cooperative launch: per layer the q|k|v GEMV (RMSNorm,
 * bias, RoPE, cache append at *pos), attention over the cache, o GEMV +
 * residual, gate|up GEMV (RMSNorm, silu*up) and down GEMV + residual, in place
 * on h.  Same results, bit for bit, as hq4_qkv_rope, hq4_attention,
 * hq4_gemv_fused and hq4_gemv_norm called per layer.  No reference counterpart
 * (the reference runs a layer as NumPy calls around q4_gemv); it replaces the
 * per-layer launches of a decode step.
 *
 * Weights in the device layout of those entry points: q|k|v rows
 * concatenated, q and k rows permuted for the RoPE pairs; gate and up rows
 * interleaved in blocks of 8.  All buffers are device memory, 16-byte aligned
 * (weights 32-byte); caches [n_kv][max_ctx][head_dim] fp32. */
typedef struct hq4_decode_layer {
    const uint32_t* qkv_w;
    const uint16_t* qkv_s;
    const uint16_t* qkv_b;
    const float* qkv_bias;   /* [(n_heads + 2 n_kv) head_dim], may be NULL */
    const float* input_norm; /* [hidden] */
    const uint32_t* o_w;
    const uint16_t* o_s;
    const uint16_t* o_b;
    const float* post_norm;  /* [hidden] */
    const uint32_t* gate_up_w;
    const uint16_t* gate_up_s;
    const uint16_t* gate_up_b;
    const uint32_t* down_w;
    const uint16_t* down_s;
    const uint16_t* down_b;
    float* k_cache;
    float* v_cache;
} hq4_decode_layer;

/* Build a plan: the phase program and tensor maps in device memory, bound to
 * these buffers (h [hidden], q_buf [n_heads head_dim], attn_buf
 * [n_heads head_dim], mlp_buf [intermediate] fp32; pos the device position).
 * `layers` is a host array.  Shapes: group size 64, 128 or 256, every
 * projection's n_in a multiple of 256 with n_in / gs a multiple of 8,
 * head_dim a multiple of 32 up to 256; max_ctx must leave the scores in one
 * CTA's shared memory.  -1 when a shape does not fit. */
int hq4_decode_plan_create(const hq4_decode_layer* layers, int n_layers, int hidden, int n_heads, int n_kv,
                           int head_dim, int intermediate, int gs, float eps, float attn_scale,
                           const float* rope_cos, const float* rope_sin, int max_ctx, float* h,
                           const int* pos, float* q_buf, float* attn_buf, float* mlp_buf, void** plan);

/* One decode step of the plan on `stream` (capturable in a CUDA graph). */
int hq4_decode_plan_run(void* plan, void* stream);

/* info[0..3] = grid, ring stages, dynamic shared memory bytes, phases. */
int hq4_decode_plan_info(void* plan, int* info);

/* Failure-path testing of the plan's grid barrier (no reference
 * counterpart; the reference's pipeline has no device waits).  skip_cta >= 0
 * makes that CTA withhold its arrival at the plan's first grid barrier of
 * every later run, so the barrier never completes: every CTA's wait ends
 * after barrier_ns (<= 0: the default 1 s), status bit 0 is set, the run
 * returns with its outputs invalid, and the barrier words are reset for the
 * next run.  skip_cta = -1 and barrier_ns = 0 restore normal runs. */
int hq4_decode_plan_fault(void* plan, int skip_cta, long long barrier_ns);

void hq4_decode_plan_destroy(void* plan);

#ifdef __cplusplus
}
#endif

#endif /* HQ4_H */
