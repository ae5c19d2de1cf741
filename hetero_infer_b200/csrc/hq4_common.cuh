// Shared device helpers for the hq4 kernels (sm_100a only).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "hq4 kernels are written for sm_100a (B200) only"
#endif

namespace hq4 {

constexpr int kWarp = 32;

// ---- programmatic dependent launch -------------------------------------
// launch_dependents lets the next kernel in the stream be scheduled while this
// one drains; wait blocks until the previous kernel has completed and its
// writes are visible.  Both are no-ops when the launch carries no
// programmatic dependency.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---- global loads -------------------------------------------------------
// Streaming 256-bit load of packed weights: read once, do not keep in L1.
__device__ __forceinline__ void ldg256_stream(const uint32_t* p, uint32_t (&v)[8]) {
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]),
                   "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "l"(p));
}
__device__ __forceinline__ void ldg128_stream(const uint32_t* p, uint32_t (&v)[4]) {
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "l"(p));
}
// Scales/biases: 16-bit, re-used by neighbouring units through L1.
__device__ __forceinline__ uint32_t ldg_u16(const uint16_t* p) {
    unsigned short v;
    asm volatile("ld.global.nc.L1::evict_last.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}
// Coherent (L1-bypassing) load for values written by other CTAs this launch.
__device__ __forceinline__ float ldcg_f32(const float* p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}

// ---- int4 -> fp16 exact dequantisation ---------------------------------
// d = (a & b) | c
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t h2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// From one packed word w (nibbles q0..q7, low first) produce the half2 pairs
//   lo = {q0, q4}   hi = {q1, q5}
// exactly: OR-ing a nibble into the mantissa of 1024.0h gives 1024+q, and a
// nibble at bits 4..7 gives 1024+16q, which *1/16 - 64 maps back to q.
__device__ __forceinline__ void dq_pair(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t kMagic = 0x64006400u;      // {1024, 1024}
    const uint32_t kSixteenth = 0x2C002C00u;  // {1/16, 1/16}
    const uint32_t kNeg64 = 0xD400D400u;      // {-64, -64}
    lo = h2_sub(lop3_and_or(w, 0x000F000Fu, kMagic), kMagic);
    hi = h2_fma(lop3_and_or(w, 0x00F000F0u, kMagic), kSixteenth, kNeg64);
}

// ---- int4 -> u8 unpack ----------------------------------------------------
// One packed word w (nibbles q0..q7, low first) -> two u8x4 registers
//   even = {q0, q2, q4, q6}   odd = {q1, q3, q5, q7}
__device__ __forceinline__ void unpack_u8(uint32_t w, uint32_t& even, uint32_t& odd) {
    even = w & 0x0F0F0F0Fu;
    odd = (w >> 4) & 0x0F0F0F0Fu;
}

// ---- tensor core --------------------------------------------------------
// D(16x8,s32) += A(16x32,u8,row) * B(32x8,s8,col): exact integer products/sums
__device__ __forceinline__ void mma_u8s8_16832(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D(16x8,f32) += A(16x16,f16,row) * B(16x8,f16,col)
__device__ __forceinline__ void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)bits16));
}

// Exponent E with amax < 2^E (E = floor(log2 amax) + 1 for normal amax), so
// that x * 2^(22-E) is an integer grid of 22 bits plus sign.  Clamped so both
// 2^(22-E) and 2^(E-22) are normal fp32; groups below 2^-100 round to zero.
__device__ __forceinline__ int group_exponent(float amax) {
    if (!(amax > 0.0f)) return 0;
    int e = (int)((__float_as_uint(amax) >> 23) & 0xFF) - 126;
    if (e < -100) e = -100;
    if (e > 128) e = 128;
    return e;
}

// Balanced base-256 digits of |v| <= 2^22:  v = d2*65536 + d1*256 + d0 with
// d0, d1 in [-128, 127] and d2 in [-64, 64]; returned as raw bytes.
__device__ __forceinline__ void digits3(int v, uint32_t& d2, uint32_t& d1, uint32_t& d0) {
    const int a = ((v + 128) & 255) - 128;
    const int v1 = (v - a) >> 8;
    const int b = ((v1 + 128) & 255) - 128;
    const int c = (v1 - b) >> 8;
    d0 = (uint32_t)a & 255u;
    d1 = (uint32_t)b & 255u;
    d2 = (uint32_t)c & 255u;
}
__device__ __forceinline__ float exp2i(int e) {  // 2^e for |e| <= 126
    return __uint_as_float((uint32_t)(e + 127) << 23);
}

}  // namespace hq4
