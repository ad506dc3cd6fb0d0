// common.cuh — device helpers shared by every kernel of the decode step and the
// flow head: bf16 rounding at MLX's points, tensor-core fragments, and the
// in-register dequantisation of the repacked weight tiles (see pack.h for the
// tile layout these functions read).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define MING_DEV __device__ __forceinline__

namespace ming {

// ---- bf16 ----
MING_DEV float bf2f(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }
MING_DEV uint16_t f2bf(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
// Round an f32 to the nearest bf16 (ties to even), as MLX does at every op.
MING_DEV float rb(float f) { return bf2f(f2bf(f)); }

MING_DEV uint32_t pack_bf16x2(float lo, float hi) {
    return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}
MING_DEV uint32_t pack_f16x2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}
MING_DEV float2 unpack_bf16x2(uint32_t u) {
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

// ---- tensor cores: mma.sync m16n8k16, f32 accumulate ----
// A (weights) 16x16 row-major fragment a[4], B (activations) 16x8 col fragment
// b[2], D 16x8: d0,d1 = (row g, cols 2t,2t+1), d2,d3 = (row g+8, same cols),
// with g = lane/4, t = lane%4.
MING_DEV void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
MING_DEV void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int LUT>
MING_DEV uint32_t lop3(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, %4;\n" : "=r"(r) : "r"(a), "r"(b), "r"(c), "n"(LUT));
    return r;
}

MING_DEV uint32_t hsub2_u(uint32_t a, uint32_t b) {
    __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}
MING_DEV uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    __half2 r = __hfma2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b), *reinterpret_cast<__half2*>(&c));
    return *reinterpret_cast<uint32_t*>(&r);
}

// One 32-bit word of a 4-bit tile holds the 8 codes this lane needs for one
// m16k16 step: nibble i at bits 4i with (n0,n4)=A[g][2t..2t+1],
// (n1,n5)=A[g+8][2t..], (n2,n6)=A[g][2t+8..], (n3,n7)=A[g+8][2t+8..].
// Codes become exact fp16 integers: (x | 0x6400) is 1024 + x.
MING_DEV void dq4(uint32_t u, uint32_t (&a)[4]) {
    const uint32_t MAGIC = 0x64006400u;   // half2(1024, 1024)
    const uint32_t SCALE16 = 0x2C002C00u; // half2(1/16, 1/16)
    const uint32_t NEG64 = 0xD400D400u;   // half2(-64, -64)
    const uint32_t lo0 = lop3<(0xF0 & 0xCC) | 0xAA>(u, 0x000F000Fu, MAGIC);
    const uint32_t hi0 = lop3<(0xF0 & 0xCC) | 0xAA>(u, 0x00F000F0u, MAGIC);
    const uint32_t u8 = u >> 8;
    const uint32_t lo1 = lop3<(0xF0 & 0xCC) | 0xAA>(u8, 0x000F000Fu, MAGIC);
    const uint32_t hi1 = lop3<(0xF0 & 0xCC) | 0xAA>(u8, 0x00F000F0u, MAGIC);
    a[0] = hsub2_u(lo0, MAGIC);
    a[1] = hfma2_u(hi0, SCALE16, NEG64);
    a[2] = hsub2_u(lo1, MAGIC);
    a[3] = hfma2_u(hi1, SCALE16, NEG64);
}

// Two words of an 8-bit tile per m16k16 step: w0 = (A[g][2t], A[g][2t+1],
// A[g+8][2t], A[g+8][2t+1]), w1 = the same at k+8. Bytes become 1024 + x.
MING_DEV void dq8(uint32_t w0, uint32_t w1, uint32_t (&a)[4]) {
    const uint32_t MAGIC = 0x64006400u;
    a[0] = hsub2_u(__byte_perm(w0, 0x64u, 0x4140), MAGIC);
    a[1] = hsub2_u(__byte_perm(w0, 0x64u, 0x4342), MAGIC);
    a[2] = hsub2_u(__byte_perm(w1, 0x64u, 0x4140), MAGIC);
    a[3] = hsub2_u(__byte_perm(w1, 0x64u, 0x4342), MAGIC);
}

// ---- memory ----
MING_DEV uint4 ldg_nc16(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
MING_DEV uint2 ldg_nc8(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];\n" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

// Global nanosecond timer (comparable across SMs; launch-trace stamps).
MING_DEV long long gtimer() {
    long long t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}

MING_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
MING_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace ming
