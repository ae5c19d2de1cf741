// Device fill of the counter-based synthetic fp16 embedding table used by the
// benchmark models (the host evaluates the same rows in
// hetero_infer_b200/synth.py:embed_rows).  Element (r, c):
//   key = seed * 0x9E3779B97F4A7C15 + r * hidden + c
//   s   = sum_{i<12} (splitmix64(key * 12 + i) >> 40)        (exact, int64)
//   out = fp16( fp32(s - 6 * 2^24) * 2^-24 * std )
#include "hq4_common.cuh"
#include "hq4.h"

namespace hq4 {
int check_device_cap();

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void synth_embed_kernel(uint64_t seed, long long total, int hidden, float std, __half* out) {
    const uint64_t base = seed * 0x9E3779B97F4A7C15ull;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (long long)gridDim.x * blockDim.x) {
        const uint64_t key = base + (uint64_t)e;  // r * hidden + c == e
        long long acc = 0;
#pragma unroll
        for (int i = 0; i < 12; i++) acc += (long long)(splitmix64(key * 12ull + (uint64_t)i) >> 40);
        acc -= 6ll * (1ll << 24);
        const float v = __fmul_rn((float)acc, 1.0f / 16777216.0f);
        out[e] = __float2half_rn(__fmul_rn(v, std));
    }
    (void)hidden;
}
}  // namespace hq4

extern "C" int hq4_synth_embed_f16(long long seed, int vocab, int hidden, float std, uint16_t* out,
                                   void* stream) {
    if (int rc = hq4::check_device_cap()) return rc;
    if (vocab <= 0 || hidden <= 0 || seed < 0) return HQ4_ERR_SHAPE;
    const long long total = (long long)vocab * hidden;
    hq4::synth_embed_kernel<<<148 * 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        (uint64_t)seed, total, hidden, std, reinterpret_cast<__half*>(out));
    return cudaGetLastError() == cudaSuccess ? HQ4_OK : HQ4_ERR_LAUNCH;
}
