/* CPU oracle for the fused int4 GEMV path -- TEST INFRASTRUCTURE ONLY.
 *
 * This is a restatement, in plain C, of the arithmetic of the reference's
 * kernel/q4gemv.c (hetero-infer).  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load it, and only as the checker; the
 * product path never calls it.  Built with -ffp-contract=off so every
 * multiply and add rounds exactly where the statement below says it does.
 *
 * Weight layout (kernel/q4gemv.c:7-11, MLX affine quantisation):
 *   w       [n_out][n_in/8]   uint32, eight 4-bit values each, low nibble first
 *   scales  [n_out][n_in/gs]  float16 bits
 *   biases  [n_out][n_in/gs]  float16 bits
 *   value = q * scale + bias
 *
 * Two GEMV semantics exist in the reference, chosen there by compiler flags:
 *   oracle_q4_gemv_f32  the portable float path: per group an fp32 dot
 *                       s += q * x (kernel/q4gemv.c:131-137), then
 *                       acc += scale*dot + bias*xsum (:177-181, :196-197).
 *   oracle_q4_gemv_i16  the x86 AVX2 path: x quantised once to int16 with
 *                       scale amax/32767 and round-half-away (:258-269), an
 *                       exact integer group dot (:80-111), dot = xscale*idot
 *                       (:173), then the same per-group accumulation, which
 *                       gcc contracts into one fused multiply-add
 *                       (fma(scale, dot, bias*xsum)); `contract` selects it.
 * Both compute xsum[g] as a sequential fp32 sum (:244-248).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* IEEE half -> float, exact (kernel/q4gemv.c:56-70 states the same mapping). */
float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {                               /* subnormal: normalise */
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; sh++; }
            bits = sign | ((uint32_t)(113 - sh) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static int shape_ok(int n_in, int gs) {
    return gs > 0 && n_in > 0 && n_in % gs == 0 && gs % 8 == 0;
}

static void group_sums(const float *x, int n_in, int gs, float *xsum) {
    for (int g = 0; g < n_in / gs; g++) {
        float s = 0.0f;
        for (int i = 0; i < gs; i++) s += x[g * gs + i];
        xsum[g] = s;
    }
}

/* Float semantics (kernel/q4gemv.c:113-139 scalar branch + :158-200). */
int oracle_q4_gemv_f32(const uint32_t *w, const uint16_t *scales, const uint16_t *biases,
                       const float *x, float *out, int n_out, int n_in, int gs) {
    if (!shape_ok(n_in, gs)) return -1;
    const int ng = n_in / gs, wpg = gs / 8, wpr = n_in / 8;
    float *xsum = (float *)malloc(sizeof(float) * (size_t)ng);
    if (!xsum) return -3;
    group_sums(x, n_in, gs, xsum);
    for (int o = 0; o < n_out; o++) {
        const uint32_t *wr = w + (size_t)o * wpr;
        float acc = 0.0f;
        for (int g = 0; g < ng; g++) {
            float dot = 0.0f;
            for (int k = 0; k < wpg; k++) {
                uint32_t d = wr[g * wpg + k];
                for (int j = 0; j < 8; j++) {
                    float p = (float)((d >> (4 * j)) & 0xFu) * x[g * gs + 8 * k + j];
                    dot = dot + p;
                }
            }
            size_t idx = (size_t)o * ng + g;
            float t1 = oracle_f16_to_f32(scales[idx]) * dot;
            float t2 = oracle_f16_to_f32(biases[idx]) * xsum[g];
            acc = acc + (t1 + t2);
        }
        out[o] = acc;
    }
    free(xsum);
    return 0;
}

/* The int16 quantisation of x used by the AVX2 path (kernel/q4gemv.c:258-269).
 * Writes xq in natural order (the reference's evens-then-odds permutation only
 * reorders an exact integer sum) and returns xscale. */
float oracle_quantise_x_i16(const float *x, int n, int16_t *xq) {
    float amax = 0.0f;
    for (int i = 0; i < n; i++) {
        float v = x[i] < 0 ? -x[i] : x[i];
        if (v > amax) amax = v;
    }
    float xscale = amax > 0.0f ? amax / 32767.0f : 1.0f;
    float inv = 1.0f / xscale;
    for (int i = 0; i < n; i++) {
        float a = x[i] * inv;
        float r = a < 0 ? a - 0.5f : a + 0.5f;
        xq[i] = (int16_t)r;
    }
    return xscale;
}

/* AVX2 semantics.  contract: 0 = acc + (s*dot + b*xsum) with every op rounded;
 * 1 = acc + fma(s, dot, b*xsum); 2 = acc + fma(b, xsum, s*dot). */
int oracle_q4_gemv_i16(const uint32_t *w, const uint16_t *scales, const uint16_t *biases,
                       const float *x, float *out, int n_out, int n_in, int gs, int contract) {
    if (!shape_ok(n_in, gs) || gs % 64) return -1;
    const int ng = n_in / gs, wpg = gs / 8, wpr = n_in / 8;
    float *xsum = (float *)malloc(sizeof(float) * (size_t)ng);
    int16_t *xq = (int16_t *)malloc(sizeof(int16_t) * (size_t)n_in);
    if (!xsum || !xq) { free(xsum); free(xq); return -3; }
    group_sums(x, n_in, gs, xsum);
    const float xscale = oracle_quantise_x_i16(x, n_in, xq);
    for (int o = 0; o < n_out; o++) {
        const uint32_t *wr = w + (size_t)o * wpr;
        float acc = 0.0f;
        for (int g = 0; g < ng; g++) {
            int32_t idot = 0;
            for (int k = 0; k < wpg; k++) {
                uint32_t d = wr[g * wpg + k];
                for (int j = 0; j < 8; j++)
                    idot += (int32_t)((d >> (4 * j)) & 0xFu) * (int32_t)xq[g * gs + 8 * k + j];
            }
            float dot = xscale * (float)idot;
            size_t idx = (size_t)o * ng + g;
            float s = oracle_f16_to_f32(scales[idx]), b = oracle_f16_to_f32(biases[idx]);
            float term;
            if (contract == 1) term = fmaf(s, dot, b * xsum[g]);
            else if (contract == 2) term = fmaf(b, xsum[g], s * dot);
            else term = s * dot + b * xsum[g];
            acc = acc + term;
        }
        out[o] = acc;
    }
    free(xsum);
    free(xq);
    return 0;
}

/* Block dequantisation (kernel/q4gemv.c:316-354, 359-379): rows [row0,row1)
 * into out as fp32 [row1-row0][n_in].  q*scale is exact in fp32 (4-bit times
 * 11-bit significand), so the fused and unfused forms agree bit for bit. */
int oracle_q4_dequant(const uint32_t *w, const uint16_t *scales, const uint16_t *biases,
                      float *out, int row0, int row1, int n_in, int gs) {
    if (!shape_ok(n_in, gs)) return -1;
    const int ng = n_in / gs, wpr = n_in / 8;
    for (int o = row0; o < row1; o++) {
        const uint32_t *wr = w + (size_t)o * wpr;
        float *dst = out + (size_t)(o - row0) * n_in;
        for (int k = 0; k < n_in; k++) {
            int g = k / gs;
            float s = oracle_f16_to_f32(scales[(size_t)o * ng + g]);
            float b = oracle_f16_to_f32(biases[(size_t)o * ng + g]);
            float q = (float)((wr[k / 8] >> (4 * (k % 8))) & 0xFu);
            dst[k] = q * s + b;
        }
    }
    return 0;
}
