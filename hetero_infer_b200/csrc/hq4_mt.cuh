// Launch parameters and host entry points of the multi-token streaming
// W4A16 product (hq4_gemv_mt.cu), shared with the GEMV, GEMM and stage
// entry points that route token counts above one to it.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace hq4 {

constexpr int kMtMaxTok = 8;  // tokens per pass

struct MtParams {
    const uint32_t* w;
    const uint16_t* sc;
    const uint16_t* bi;
    const void* x;   // [m][x_stride]: fp32, or bf16 when x_bf16
    int x_stride;    // elements between tokens
    int x_bf16;
    float* out;      // plain: [m][out_stride]; SiLU(gate) * up: [m][out_stride] (n_out / 2 used)
    int out_stride;  // floats between tokens
    int n_out, n_in, m;
    // filled by the launcher
    int n_chunks, sg_shift, n_sg, n_strips, ks, n_clusters;
    const float* row_add;   // optional: [n_out], added to every token
    const float* residual;  // optional (plain): [m][out_stride]
    const float* norm_w;    // optional (fp32 x): RMSNorm of each token before the product
    float eps;
    int mode;               // kEpiPlain, kEpiSiluMul or kEpiQkvRope
    int weights_after_wait; // read the weights only after the dependency wait
    // kEpiQkvRope: as the one-token kernel's, token j at position *pos + tok0 + j
    int q_strips, k_strips, head_dim, max_ctx;
    const int* pos;
    const float* rope_cos;
    const float* rope_sin;
    float* q_out;  // [m][q_stride]
    int q_stride;
    float* k_cache;
    float* v_cache;
    int tok0;
    int* status;
};

// First chunk of rank r of ks over n_chunks k-chunks: an even share rounded
// to `align` chunks, so that every rank's scale tiles start on a 16-byte
// boundary (align = 2 << sg_shift).  Ranks may be empty on short rows.
__host__ __device__ inline int mt_chunk_start(int r, int ks, int n_chunks, int align) {
    if (r >= ks) return n_chunks;
    const long long base = (long long)r * n_chunks / ks;
    const int c = (int)((base + align / 2) / align * align);
    return c < n_chunks ? c : n_chunks;
}

// One pass of up to kMtMaxTok tokens; *used is false when the shape or
// pointers do not suit it (nothing was launched).
int gemv_mt_pass(MtParams prm, int gs, cudaStream_t st, bool* used);
// All m_total tokens in passes of up to 4; *used false when the shape does
// not suit.
int gemv_mt_tokens(MtParams prm, int gs, int m_total, cudaStream_t st, bool* used);
// Whether a pass of m tokens of this shape runs on the multi-token kernel.
bool gemv_mt_fits(int n_out, int n_in, int gs, int m);

}  // namespace hq4
