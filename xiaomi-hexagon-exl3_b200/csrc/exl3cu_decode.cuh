// Device-side EXL3 trellis decode primitives shared by every kernel.
//
// Codebooks (reference: src/exl3_codec.cpp:68-86):
//   mul1   p = state * 0x83dcd12d; s = byte-sum(p) in [0,1020];
//          w = RNE_fp16((1774*s - 905216) / 2^18).
//          Computed as fp16(1024+s) -- the bit pattern 0x6400+s, which one IDP4A
//          produces -- times fp16 0x1eee plus fp16 0xc931 in ONE fp16 fused
//          multiply-add.  The exact value (1774*s-905216)/2^18 has at most 21
//          significant bits, so the reference's fp32 fma is exact and its single
//          fp32->fp16 rounding equals the single fp16 rounding of fma.rn.f16x2.
//          Verified exhaustively over all 65536 states against the oracle.
//   mcg / 3inst  p = state*0xcbac1fed  |  p = state*89226354 + 64248484;
//          m = (p & 0x8fff8fff) ^ 0x3b603b60; w = fp16(lo(m)) + fp16(hi(m)).
//          Both halves are normal with exponents within 3 of each other, so the
//          sum is exact before its one rounding: add.rn.f16 reproduces it.
//
// Trellis tile (src/exl3_codec.cpp:88-115): 16*bits uint16 = 8*bits words,
// word i = u16[2i] | u16[2i+1] << 16, read MSB-first as a ring of 256*bits bits.
// Position p = 8*L + e takes the 16-bit window ending at ring bit (p+1)*bits and
// lands at row (L%4)*2 + (e&1) + 8*((e>>1)&1), column L/4 + 8*(e>>2).  That is
// exactly the mma.m16n8k16 A fragment of W^T for lane L: registers
// {e0,e1} {e4,e5} {e2,e3} {e6,e7} = a0a1, a2a3, a4a5, a6a7.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace exl3cu {

enum : unsigned { CB_3INST = 0, CB_MCG = 1, CB_MUL1 = 2 };

__device__ __forceinline__ uint32_t half2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 bits_half2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Two mul1 states (clean 16-bit values) -> packed fp16x2 {w(s0) lo, w(s1) hi}.
__device__ __forceinline__ uint32_t mul1_pair(uint32_t s0, uint32_t s1) {
    const uint32_t p0 = s0 * 0x83dcd12du;
    const uint32_t p1 = s1 * 0x83dcd12du;
    const uint32_t h0 = __dp4a(p0, 0x01010101u, 0x6400u);  // fp16 bits of 1024 + bytesum
    const uint32_t h1 = __dp4a(p1, 0x01010101u, 0x6400u);
    const uint32_t h = __byte_perm(h0, h1, 0x5410);
    const __half2 r = __hfma2(bits_half2(h), bits_half2(0x1eee1eeeu), bits_half2(0xc931c931u));
    return half2_bits(r);
}

__device__ __forceinline__ uint16_t lcg_one(uint32_t s, unsigned cb) {
    uint32_t p = (cb == CB_MCG) ? s * 0xcbac1fedu : s * 89226354u + 64248484u;
    p = (p & 0x8fff8fffu) ^ 0x3b603b60u;
    const __half2 h = bits_half2(p);
    const __half r = __hadd(__low2half(h), __high2half(h));
    return __half_as_ushort(r);
}

template <unsigned CB>
__device__ __forceinline__ uint32_t decode_pair(uint32_t s0, uint32_t s1) {
    if constexpr (CB == CB_MUL1) {
        return mul1_pair(s0, s1);
    } else {
        return uint32_t(lcg_one(s0, CB)) | (uint32_t(lcg_one(s1, CB)) << 16);
    }
}

// Runtime-codebook variant for the non-hot kernels.
__device__ __forceinline__ uint32_t decode_pair_rt(uint32_t s0, uint32_t s1, unsigned cb) {
    if (cb == CB_MUL1) return mul1_pair(s0, s1);
    return uint32_t(lcg_one(s0, cb)) | (uint32_t(lcg_one(s1, cb)) << 16);
}

// ---------------------------------------------------------------------------
// Lane-sliced chunk layout ("LSC"), the device-resident weight format.
//
// A chunk is one 16-row strip of one 128-column block: 8 tiles (c = 0..7),
// 256*bits bytes.  Chunk (nb, rk) -- nb = column block, rk = 16-row index
// 0..k/16-1 -- sits at byte (nb * (k/16) + rk) * 256 * bits, so one column
// block's whole K extent is contiguous.  Inside a chunk, lane L of a warp owns
// the 8*bits-byte segment at byte 8*bits*L, holding ring bytes
// [bits*L, bits*L + bits) of tiles 0..7 back to back: that is exactly the
// 8*bits ring bits that positions 8L..8L+7 of each tile end inside.  Bytes keep
// the ring's big-endian-in-little-endian-words order (ring byte B at memory byte
// B ^ 3), so a lane reads its segment as 2*bits words whose MSB-first
// concatenation is tile 0's slice, tile 1's slice, ...  The 16 - bits ring bits
// before a slice belong to lane L-1 (lane 31 for lane 0: the ring is
// tail-biting) and arrive by one warp shuffle per two tiles.
// ---------------------------------------------------------------------------

// 16 bits of the lane segment starting at MSB-first bit offset `pos`.
template <int NW>
__device__ __forceinline__ uint32_t seg_field16(const uint32_t (&w)[NW], int pos) {
    const int i = pos >> 5;
    const int o = pos & 31;
    if (o <= 16) return (w[i] >> (16 - o)) & 0xffffu;
    return __funnelshift_l(w[i + 1], w[i], o - 16) & 0xffffu;
}

// Decode the 8 tiles of one chunk held by this lane (segment words w[2*BITS]).
// out[c][0..3] = mma A-fragment registers of tile c (W^T, swap-AB layout).
template <int BITS, unsigned CB>
__device__ __forceinline__ void decode_chunk(const uint32_t (&w)[2 * BITS], uint32_t (&out)[8][4]) {
    constexpr int SLICE = 8 * BITS;  // own ring bits per tile per lane
    const int lane = threadIdx.x & 31;
    const int src = (lane + 31) & 31;
    uint32_t prior[8];  // 16 ring bits just before this lane's slice, per tile
    if constexpr (BITS >= 2) {
#pragma unroll
        for (int c = 0; c < 8; c += 2) {
            const uint32_t t0 = seg_field16(w, SLICE * (c + 1) - 16);
            const uint32_t t1 = seg_field16(w, SLICE * (c + 2) - 16);
            const uint32_t got = __shfl_sync(0xffffffffu, t0 | (t1 << 16), src);
            prior[c] = got & 0xffffu;
            prior[c + 1] = got >> 16;
        }
    } else {
        // bits == 1: a lane owns 8 bits per tile; the window reaches two lanes back.
        const uint32_t p0 = __shfl_sync(0xffffffffu, w[0], src);
        const uint32_t p1 = __shfl_sync(0xffffffffu, w[1], src);
        uint32_t last16[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint32_t mine = c < 4 ? (w[0] >> (24 - 8 * c)) & 0xffu : (w[1] >> (24 - 8 * (c - 4))) & 0xffu;
            const uint32_t prev = c < 4 ? (p0 >> (24 - 8 * c)) & 0xffu : (p1 >> (24 - 8 * (c - 4))) & 0xffu;
            last16[c] = (prev << 8) | mine;
        }
#pragma unroll
        for (int c = 0; c < 8; c += 2) {
            const uint32_t got = __shfl_sync(0xffffffffu, last16[c] | (last16[c + 1] << 16), src);
            prior[c] = got & 0xffffu;
            prior[c + 1] = got >> 16;
        }
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        constexpr int HEAD = SLICE < 16 ? SLICE : 16;  // own bits gathered into z
        uint32_t head;
        if constexpr (BITS >= 2) {
            head = seg_field16(w, SLICE * c);
        } else {
            head = c < 4 ? (w[0] >> (24 - 8 * c)) & 0xffu : (w[1] >> (24 - 8 * (c - 4))) & 0xffu;
        }
        const uint32_t z = (prior[c] << HEAD) | head;  // ring bits ending at own bit HEAD-1
        uint32_t s[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int end = (e + 1) * BITS;  // exclusive end, in own-slice bits
            if (end <= HEAD) {
                s[e] = (z >> (HEAD - end)) & 0xffffu;
            } else {
                s[e] = seg_field16(w, SLICE * c + end - 16);
            }
        }
        out[c][0] = decode_pair<CB>(s[0], s[1]);
        out[c][1] = decode_pair<CB>(s[4], s[5]);
        out[c][2] = decode_pair<CB>(s[2], s[3]);
        out[c][3] = decode_pair<CB>(s[6], s[7]);
    }
}

// Tiles C0 and C0+1 of the chunk only (a quarter of decode_chunk's work):
// out[i] = the mma A-fragment registers of tile C0+i.  All 32 lanes take part
// (the window's prior bits come from the neighbouring lane).
template <int BITS, unsigned CB, int C0, int NW>
__device__ __forceinline__ void decode_tile_pair(const uint32_t (&w)[NW], uint32_t (&out)[2][4]) {
    static_assert(C0 % 2 == 0 && C0 >= 0 && C0 < 8, "tile pair");
    constexpr int SLICE = 8 * BITS;
    constexpr int HEAD = SLICE < 16 ? SLICE : 16;
    const int lane = threadIdx.x & 31;
    const int src = (lane + 31) & 31;
    uint32_t prior[2];
    uint32_t head[2];
    if constexpr (BITS >= 2) {
        const uint32_t t0 = seg_field16(w, SLICE * (C0 + 1) - 16);
        const uint32_t t1 = seg_field16(w, SLICE * (C0 + 2) - 16);
        const uint32_t got = __shfl_sync(0xffffffffu, t0 | (t1 << 16), src);
        prior[0] = got & 0xffffu;
        prior[1] = got >> 16;
        head[0] = seg_field16(w, SLICE * C0);
        head[1] = seg_field16(w, SLICE * (C0 + 1));
    } else {
        // bits == 1: a lane owns 8 bits per tile; the window reaches two lanes back.
        constexpr int WI = C0 < 4 ? 0 : 1;
        constexpr int SH0 = 24 - 8 * (C0 & 3), SH1 = 24 - 8 * ((C0 + 1) & 3);
        const uint32_t pw = __shfl_sync(0xffffffffu, w[WI], src);
        head[0] = (w[WI] >> SH0) & 0xffu;
        head[1] = (w[WI] >> SH1) & 0xffu;
        const uint32_t l0 = (((pw >> SH0) & 0xffu) << 8) | head[0];
        const uint32_t l1 = (((pw >> SH1) & 0xffu) << 8) | head[1];
        const uint32_t got = __shfl_sync(0xffffffffu, l0 | (l1 << 16), src);
        prior[0] = got & 0xffffu;
        prior[1] = got >> 16;
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int c = C0 + i;
        const uint32_t z = (prior[i] << HEAD) | head[i];
        uint32_t s[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int end = (e + 1) * BITS;
            if (end <= HEAD) {
                s[e] = (z >> (HEAD - end)) & 0xffffu;
            } else {
                s[e] = seg_field16(w, SLICE * c + end - 16);
            }
        }
        out[i][0] = decode_pair<CB>(s[0], s[1]);
        out[i][1] = decode_pair<CB>(s[4], s[5]);
        out[i][2] = decode_pair<CB>(s[2], s[3]);
        out[i][3] = decode_pair<CB>(s[6], s[7]);
    }
}

}  // namespace exl3cu
