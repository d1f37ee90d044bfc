// Shared device helpers: the fp32 Hadamard-128 butterfly and small load/store
// wrappers.  All fp32 arithmetic that must match the reference's rounding goes
// through __fadd_rn/__fsub_rn/__fmul_rn, which the compiler never contracts into
// an FMA, so each value sees exactly the operations of the reference loop.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace exl3cu {

// 1/sqrt(128) as the fp32 literal the reference multiplies by (src/exl3_codec.cpp:151).
constexpr float kH128Norm = 0.08838834764831844055f;

// Orthonormal H128 over 128 values spread across one warp, lane l holding
// elements 4l..4l+3.  Butterfly strides 1, 2 (inside the lane) then 4..64
// (lane xor 1..16), each stage forming (a+b, a-b) on the pair (i, i+stride)
// as the reference does (src/exl3_codec.cpp:147-167), then one multiply by the
// normaliser.  Results are bit-identical to the reference.
__device__ __forceinline__ void h128_warp4(float (&v)[4]) {
    const int lane = threadIdx.x & 31;
    {
        const float a0 = v[0], b0 = v[1], a1 = v[2], b1 = v[3];
        v[0] = __fadd_rn(a0, b0); v[1] = __fsub_rn(a0, b0);
        v[2] = __fadd_rn(a1, b1); v[3] = __fsub_rn(a1, b1);
    }
    {
        const float a0 = v[0], a1 = v[1], b0 = v[2], b1 = v[3];
        v[0] = __fadd_rn(a0, b0); v[2] = __fsub_rn(a0, b0);
        v[1] = __fadd_rn(a1, b1); v[3] = __fsub_rn(a1, b1);
    }
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const bool upper = (lane & m) != 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float other = __shfl_xor_sync(0xffffffffu, v[q], m);
            v[q] = upper ? __fsub_rn(other, v[q]) : __fadd_rn(v[q], other);
        }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = __fmul_rn(v[q], kH128Norm);
}

__device__ __forceinline__ uint4 ldg_stream_v4(const uint32_t * p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint2 ldg_stream_v2(const uint32_t * p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}

// Load this lane's 2*BITS segment words (8*BITS bytes, 8-byte aligned; 16-byte
// aligned when BITS is even).
template <int BITS>
__device__ __forceinline__ void load_segment(const uint32_t * p, uint32_t (&w)[2 * BITS]) {
    if constexpr ((BITS & 1) == 0) {
#pragma unroll
        for (int i = 0; i < BITS / 2; ++i) {
            const uint4 r = ldg_stream_v4(p + 4 * i);
            w[4 * i] = r.x; w[4 * i + 1] = r.y; w[4 * i + 2] = r.z; w[4 * i + 3] = r.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < BITS; ++i) {
            const uint2 r = ldg_stream_v2(p + 2 * i);
            w[2 * i] = r.x; w[2 * i + 1] = r.y;
        }
    }
}

__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

}  // namespace exl3cu
