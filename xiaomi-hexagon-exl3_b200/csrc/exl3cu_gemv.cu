// The packed EXL3 matrix multiply for small batches (rows <= 8 per launch):
//
//   y[r, :] = sv * H128( sum_kb H128(x[r, kb] * su[kb]) . W_inner[kb, nb] )
//
// per 128-column block nb -- the operator of the reference's
// ggml_exl3_mul_mat (src/exl3-ggml.cpp:51-92) and op_exl3_matmul
// (src/exl3-htp.c:159-232), re-designed for sm_100a:
//
// * Grid = (column block nb, K split).  A CTA owns a contiguous range of
//   16-row chunks of one column block, so its weights are one contiguous span
//   of the device layout (LSC, exl3cu_decode.cuh) and every warp streams its
//   chunks with 128-bit (even bitrates) or 64-bit (odd) coalesced loads issued
//   before the prologue runs.
// * Prologue: the CTA rotates the activations it needs, xh = H128(x * su),
//   with warp-shuffle butterflies and stores them as fp16 in shared memory
//   (the reference's HMX path also feeds fp16 activations, src/exl3-htp.c:211-226).
// * Hot loop: each lane rebuilds its 8 trellis states per tile in registers
//   (funnel shifts + one shuffle per two tiles for the tail-biting bits of the
//   previous lane), applies the codebook (mul1: IMAD + IDP4A + PRMT + HFMA2 per
//   pair) straight into mma.m16n8k16 A fragments of W^T (swap-AB: 16 output
//   columns x 16 K rows per tile, the batch in N=8), accumulating in fp32.
// * Epilogue: warps reduce in shared memory; with K split, each CTA stores its
//   fp32 partial in the split-K workspace and the last CTA to arrive (atomic
//   ticket, no waiting) sums the partials in split order -- deterministic --
//   then applies H128 and sv and writes y (fp32).  The ticket counter is reset
//   by that CTA, so the workspace is ready for the next stream-ordered call.
#include "exl3cu_internal.h"

#include <algorithm>
#include <cstdlib>

namespace exl3cu {

constexpr int kGemvWarps = 8;
constexpr int kGemvDepth = 4;  // chunks a warp holds in flight per batch

template <int BITS, unsigned CB>
__global__ void __launch_bounds__(kGemvWarps * 32) k_gemv(const GemvArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int SEGW = 2 * BITS;           // words per lane per chunk
    constexpr int CHUNKW = 64 * BITS;        // words per chunk
    constexpr int NW = kGemvWarps;
    const int nb = blockIdx.x;
    const int split = blockIdx.y;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int c0 = split * a.cps;
    const int c1 = min(c0 + a.cps, a.nchunks);
    const int g0 = c0 >> 3;
    const int ng = ((c1 - 1) >> 3) - g0 + 1;
    const int xs_ld = ng * 128 + 8;  // halves; +8 keeps the 8 B-fragment rows on distinct banks
    __half * xs = reinterpret_cast<__half *>(smem);
    const int rows = a.rows;

    // -- issue the first batch of weight loads before anything else --
    const uint32_t * wlane = a.lsc + size_t(nb) * a.nchunks * CHUNKW + size_t(lane) * SEGW;
    uint32_t w[kGemvDepth][SEGW];
    int rk0 = c0 + warp;
#pragma unroll
    for (int d = 0; d < kGemvDepth; ++d) {
        const int rk = rk0 + d * NW;
        if (rk < c1) load_segment<BITS>(wlane + size_t(rk) * CHUNKW, w[d]);
    }

    // -- prologue: xh = H128(x * su) for groups g0 .. g0+ng-1, rows 0..rows-1 --
    for (int item = warp; item < ng * rows; item += NW) {
        const int gi = item / rows;
        const int r = item - gi * rows;
        const int kcol = (g0 + gi) * 128 + lane * 4;
        float v[4];
        if (a.x_f16) {
            const uint2 raw = *reinterpret_cast<const uint2 *>(static_cast<const __half *>(a.x) +
                                                               size_t(r) * a.x_stride + kcol);
            const __half2 lo = bits_half2(raw.x), hi = bits_half2(raw.y);
            v[0] = __low2float(lo); v[1] = __high2float(lo); v[2] = __low2float(hi); v[3] = __high2float(hi);
        } else {
            const float4 f = *reinterpret_cast<const float4 *>(static_cast<const float *>(a.x) +
                                                               size_t(r) * a.x_stride + kcol);
            v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
        }
        const uint2 sraw = *reinterpret_cast<const uint2 *>(a.su + kcol);
        const __half2 s01 = bits_half2(sraw.x), s23 = bits_half2(sraw.y);
        v[0] = __fmul_rn(v[0], __low2float(s01));
        v[1] = __fmul_rn(v[1], __high2float(s01));
        v[2] = __fmul_rn(v[2], __low2float(s23));
        v[3] = __fmul_rn(v[3], __high2float(s23));
        h128_warp4(v);
        const __half2 o01 = __floats2half2_rn(v[0], v[1]);
        const __half2 o23 = __floats2half2_rn(v[2], v[3]);
        *reinterpret_cast<uint2 *>(xs + r * xs_ld + gi * 128 + lane * 4) = make_uint2(half2_bits(o01), half2_bits(o23));
    }
    __syncthreads();

    // -- hot loop --
    const int g = lane >> 2, t = lane & 3;
    const bool row_ok = g < rows;
    const __half * xrow = xs + (row_ok ? g : 0) * xs_ld + 2 * t;
    float acc[8][4];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c][0] = acc[c][1] = acc[c][2] = acc[c][3] = 0.f;

    // Rolling prefetch: slot d is refilled with the chunk kGemvDepth*NW ahead as
    // soon as it has been decoded, so each warp keeps kGemvDepth chunks in flight.
    for (; rk0 < c1; rk0 += kGemvDepth * NW) {
#pragma unroll
        for (int d = 0; d < kGemvDepth; ++d) {
            const int rk = rk0 + d * NW;
            if (rk < c1) {
                uint32_t frag[8][4];
                decode_chunk<BITS, CB>(w[d], frag);
                const int ahead = rk + kGemvDepth * NW;
                if (ahead < c1) load_segment<BITS>(wlane + size_t(ahead) * CHUNKW, w[d]);
                const int kl = (rk - g0 * 8) * 16;
                uint32_t b0 = 0, b1 = 0;
                if (row_ok) {
                    b0 = *reinterpret_cast<const uint32_t *>(xrow + kl);
                    b1 = *reinterpret_cast<const uint32_t *>(xrow + kl + 8);
                }
#pragma unroll
                for (int c = 0; c < 8; ++c) mma_16816(acc[c], frag[c], b0, b1);
            }
        }
    }

    // -- epilogue: reduce warps, then splits, then H128 + sv --
    __syncthreads();  // xs is dead; reuse shared memory
    float * red = reinterpret_cast<float *>(smem);           // [NW][rows][128]
    float * part = red + size_t(NW) * rows * 128;            // [rows][128]
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const int j0 = c * 16 + g, j1 = j0 + 8;
        const int r0 = 2 * t, r1 = r0 + 1;
        if (r0 < rows) {
            red[(warp * rows + r0) * 128 + j0] = acc[c][0];
            red[(warp * rows + r0) * 128 + j1] = acc[c][2];
        }
        if (r1 < rows) {
            red[(warp * rows + r1) * 128 + j0] = acc[c][1];
            red[(warp * rows + r1) * 128 + j1] = acc[c][3];
        }
    }
    __syncthreads();
    const int elems = rows * 128;
    for (int e = threadIdx.x; e < elems; e += NW * 32) {
        float s = red[e];
#pragma unroll
        for (int ww = 1; ww < NW; ++ww) s = __fadd_rn(s, red[ww * elems + e]);
        part[e] = s;
    }
    if (a.splits > 1) {
        __shared__ int is_last;
        float * slot = a.ws_partial + (size_t(nb) * a.splits + split) * (8 * 128);
        __syncthreads();
        for (int e = threadIdx.x; e < elems; e += NW * 32) __stcg(slot + e, part[e]);
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) {
            const unsigned prev = atomicAdd(a.ws_count + nb, 1u);
            is_last = (prev == unsigned(a.splits - 1));
        }
        __syncthreads();
        if (!is_last) return;
        __threadfence();
        const float * base = a.ws_partial + size_t(nb) * a.splits * (8 * 128);
        for (int e = threadIdx.x; e < elems; e += NW * 32) {
            float s = __ldcg(base + e);
            for (int sp = 1; sp < a.splits; ++sp) s = __fadd_rn(s, __ldcg(base + size_t(sp) * (8 * 128) + e));
            part[e] = s;
        }
        if (threadIdx.x == 0) a.ws_count[nb] = 0u;  // ready for the next stream-ordered call
    }
    __syncthreads();
    for (int r = warp; r < rows; r += NW) {
        float v[4];
        const float4 p = *reinterpret_cast<const float4 *>(part + r * 128 + lane * 4);
        v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w;
        h128_warp4(v);
        const uint2 sraw = *reinterpret_cast<const uint2 *>(a.sv + nb * 128 + lane * 4);
        const __half2 s01 = bits_half2(sraw.x), s23 = bits_half2(sraw.y);
        float4 o;
        o.x = __fmul_rn(v[0], __low2float(s01));
        o.y = __fmul_rn(v[1], __high2float(s01));
        o.z = __fmul_rn(v[2], __low2float(s23));
        o.w = __fmul_rn(v[3], __high2float(s23));
        *reinterpret_cast<float4 *>(a.y + size_t(r) * a.y_stride + nb * 128 + lane * 4) = o;
    }
}

// ---------------------------------------------------------------------------

GemvPlan plan_gemv(int device_sms, size_t k, size_t nblocks, int rows) {
    GemvPlan p{};
    const int nchunks = int(k / 16);
    const char * env = std::getenv("EXL3CU_GEMV_CPS");  // tuning experiments only
    int cps;
    if (env && std::atoi(env) > 0) {
        cps = std::atoi(env);
    } else {
        const long target_ctas = long(device_sms) * 4;
        long splits = (target_ctas + long(nblocks) - 1) / long(nblocks);
        splits = std::max(1L, std::min(splits, long(nchunks)));
        cps = int((nchunks + splits - 1) / splits);
        cps = std::max(cps, kGemvWarps);
    }
    cps = std::min(cps, 128);  // bounds shared memory: <= 17 groups of rotated activations
    cps = std::min(cps, nchunks);
    p.cps = cps;
    p.splits = (nchunks + cps - 1) / cps;
    const int ng_max = (cps + 7) / 8 + 1;
    const size_t xs_bytes = size_t(rows) * (ng_max * 128 + 8) * 2;
    const size_t red_bytes = size_t(kGemvWarps + 1) * rows * 128 * 4;
    p.smem = std::max(xs_bytes, red_bytes);
    return p;
}

size_t gemv_workspace_bytes(size_t nblocks, int splits) {
    if (splits <= 1) return 0;
    return nblocks * size_t(splits) * 8 * 128 * sizeof(float) + nblocks * sizeof(unsigned);
}

template <int BITS, unsigned CB>
static cudaError_t launch_one(const GemvArgs & a, const GemvPlan & p, cudaStream_t st) {
    auto kern = k_gemv<BITS, CB>;
    if (p.smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(p.smem));
        if (e != cudaSuccess) return e;
    }
    dim3 grid(unsigned(a.nblocks), unsigned(p.splits));
    kern<<<grid, kGemvWarps * 32, p.smem, st>>>(a);
    return cudaGetLastError();
}

template <int BITS>
static cudaError_t launch_bits(const GemvArgs & a, const GemvPlan & p, unsigned cb, cudaStream_t st) {
    switch (cb) {
        case CB_MUL1: return launch_one<BITS, CB_MUL1>(a, p, st);
        case CB_MCG: return launch_one<BITS, CB_MCG>(a, p, st);
        default: return launch_one<BITS, CB_3INST>(a, p, st);
    }
}

cudaError_t launch_gemv(const GemvArgs & a, const GemvPlan & p, unsigned bits, unsigned cb, cudaStream_t st) {
    switch (bits) {
        case 1: return launch_bits<1>(a, p, cb, st);
        case 2: return launch_bits<2>(a, p, cb, st);
        case 3: return launch_bits<3>(a, p, cb, st);
        case 4: return launch_bits<4>(a, p, cb, st);
        case 5: return launch_bits<5>(a, p, cb, st);
        case 6: return launch_bits<6>(a, p, cb, st);
        case 7: return launch_bits<7>(a, p, cb, st);
        case 8: return launch_bits<8>(a, p, cb, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace exl3cu
