// Device helpers of the mul1 GEMV (exl3cu_gemv_mul1.cu): launch constants,
// the integer tensor-core product and the per-tile trellis state extraction
// from a lane's LSC segment.
#pragma once
#include "exl3cu_internal.h"

namespace exl3cu {

constexpr int kMW = 8;                      // consumer warps
constexpr int kMThreads = (kMW + 1) * 32;   // + one producer warp
constexpr int kMStages = 4;
constexpr int kMStagesMax = 16;
constexpr int kMRows = 4;                   // rows per launch: 2 digits each fill N = 8
constexpr float kCodeA = 1774.0f / 262144.0f;
constexpr float kCodeC = -3.453125f;
constexpr float kQMax = 16000.0f;           // |q| bound: hi in [-127,127], lo in [-64,63]

__device__ __forceinline__ void imma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// The 8 trellis states of tile c for this lane (see the LSC layout in
// exl3cu_decode.cuh), s[e] for positions 8L+e.  The 16 ring bits before the
// lane's slice are state 7 of lane L-1: one shuffle per tile.  w holds the
// lane's segment words from the first tile of interest on.
template <int BITS, int NW>
__device__ __forceinline__ void tile_states(const uint32_t (&w)[NW], int c, int src, uint32_t (&s)[8]) {
    if constexpr (BITS == 4) {
        const uint32_t own = w[c];
        s[7] = own & 0xffffu;
        const uint32_t prior = __shfl_sync(0xffffffffu, s[7], src);
        s[5] = __byte_perm(own, prior, 0x7621);
        s[3] = own >> 16;
        s[1] = __byte_perm(own, prior, 0x7643);
        const uint32_t own4 = __funnelshift_r(own, prior, 4);
        const uint32_t prior4 = prior >> 4;
        s[6] = own4 & 0xffffu;
        s[4] = __byte_perm(own4, prior4, 0x7621);
        s[2] = own4 >> 16;
        s[0] = __byte_perm(own4, prior4, 0x7643);
    } else {
        constexpr int SLICE = 8 * BITS;
        s[7] = seg_field16(w, SLICE * (c + 1) - 16);
        const uint32_t prior = __shfl_sync(0xffffffffu, s[7], src);
        const uint32_t z = (prior << 16) | seg_field16(w, SLICE * c);
#pragma unroll
        for (int e = 0; e < 7; ++e) {
            const int end = (e + 1) * BITS;
            s[e] = end <= 16 ? ((z >> (16 - end)) & 0xffffu) : seg_field16(w, SLICE * c + end - 16);
        }
    }
}

}  // namespace exl3cu
