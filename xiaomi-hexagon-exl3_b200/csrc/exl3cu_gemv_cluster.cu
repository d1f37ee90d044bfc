// Grouped EXL3 GEMV with cluster split-K (the operator behind exl3cu_mul_mat).
//
// Same math as k_gemv (exl3cu_gemv.cu) and the reference's ggml_exl3_mul_mat
// (src/exl3-ggml.cpp:51-92):  y = sv * H128( sum_kb H128(x * su) . W_inner ).
// What changes is how the work meets the machine:
//
// * One launch serves a list of independent problems (different weights,
//   activations and outputs that share a bitrate and codebook): the grid is a
//   flat list of units (problem, 128-column block), each unit a thread-block
//   cluster of S CTAs that split the unit's K range.  A decoder issues one
//   launch for q/k/v, one for gate/up, one each for o and down.
// * The K-split partials meet in distributed shared memory: every CTA leaves its
//   fp32 partial in its own shared memory, the cluster barrier publishes them,
//   and cluster rank 0 sums them in rank order (deterministic), applies H128 and
//   sv and stores y.  No global workspace, atomics or GPU-scope fences.
// * Programmatic dependent launch: each CTA lets the next kernel in the stream
//   launch as soon as it starts, and waits for the previous kernel
//   (griddepcontrol.wait) only after issuing its weight loads -- weights never
//   depend on earlier kernels, activations may.  Back-to-back GEMVs therefore
//   overlap one's epilogue with the next one's weight stream.
#include "exl3cu_internal.h"

#include <cooperative_groups.h>

#include <algorithm>
#include <cstdlib>

namespace cg = cooperative_groups;

namespace exl3cu {

constexpr int kCWarps = 8;
constexpr int kCDepth = 4;

__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <int BITS, unsigned CB>
__global__ void __launch_bounds__(kCWarps * 32) k_gemv_cluster(const GemvBatch b) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int SEGW = 2 * BITS;
    constexpr int CHUNKW = 64 * BITS;
    constexpr int NW = kCWarps;
    pdl_launch_dependents();

    cg::cluster_group cluster = cg::this_cluster();
    const int S = b.splits;
    const int split = int(cluster.block_rank());
    const int unit = blockIdx.x / S;
    int p = 0;
#pragma unroll
    for (int i = 1; i < kMaxBatch; ++i)
        if (i < b.count && b.prob[i].unit_base <= unit) p = i;
    const GemvProblem & P = b.prob[p];
    const int nb = unit - P.unit_base;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int rows = P.rows;
    const int c0 = min(split * P.cps, P.nchunks);
    const int c1 = min(c0 + P.cps, P.nchunks);
    const bool has_work = c0 < c1;

    // -- weight loads first: they do not depend on any earlier kernel --
    const uint32_t * wlane = P.lsc + size_t(nb) * P.nchunks * CHUNKW + size_t(lane) * SEGW;
    uint32_t w[kCDepth][SEGW];
    int rk0 = c0 + warp;
#pragma unroll
    for (int d = 0; d < kCDepth; ++d) {
        const int rk = rk0 + d * NW;
        if (rk < c1) load_segment<BITS>(wlane + size_t(rk) * CHUNKW, w[d]);
    }
    pdl_wait();  // activations may come from the previous kernel

    const int g0 = c0 >> 3;
    const int ng = has_work ? ((c1 - 1) >> 3) - g0 + 1 : 0;
    const int xs_ld = ng * 128 + 8;
    __half * xs = reinterpret_cast<__half *>(smem);
    for (int item = warp; item < ng * rows; item += NW) {
        const int gi = item / rows;
        const int r = item - gi * rows;
        const int kcol = (g0 + gi) * 128 + lane * 4;
        float v[4];
        if (P.x_f16) {
            const uint2 raw = *reinterpret_cast<const uint2 *>(static_cast<const __half *>(P.x) +
                                                               size_t(r) * P.x_stride + kcol);
            const __half2 lo = bits_half2(raw.x), hi = bits_half2(raw.y);
            v[0] = __low2float(lo); v[1] = __high2float(lo); v[2] = __low2float(hi); v[3] = __high2float(hi);
        } else {
            const float4 f = *reinterpret_cast<const float4 *>(static_cast<const float *>(P.x) +
                                                               size_t(r) * P.x_stride + kcol);
            v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
        }
        const uint2 sraw = *reinterpret_cast<const uint2 *>(P.su + kcol);
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

    const int g = lane >> 2, t = lane & 3;
    const bool row_ok = g < rows;
    const __half * xrow = xs + (row_ok ? g : 0) * xs_ld + 2 * t;
    float acc[8][4];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c][0] = acc[c][1] = acc[c][2] = acc[c][3] = 0.f;
    for (; rk0 < c1; rk0 += kCDepth * NW) {
#pragma unroll
        for (int d = 0; d < kCDepth; ++d) {
            const int rk = rk0 + d * NW;
            if (rk < c1) {
                uint32_t frag[8][4];
                decode_chunk<BITS, CB>(w[d], frag);
                const int ahead = rk + kCDepth * NW;
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

    // -- CTA reduction: warps -> part[rows][128] --
    __syncthreads();
    float * red = reinterpret_cast<float *>(smem);
    float * part = red + size_t(NW) * rows * 128;
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

    // -- cluster reduction through distributed shared memory --
    cluster.sync();
    if (split == 0) {
        for (int e = threadIdx.x; e < elems; e += NW * 32) {
            float s = part[e];
            for (int r = 1; r < S; ++r) s = __fadd_rn(s, *cluster.map_shared_rank(part + e, r));
            part[e] = s;
        }
        __syncthreads();
        for (int r = warp; r < rows; r += NW) {
            float v[4];
            const float4 pv = *reinterpret_cast<const float4 *>(part + r * 128 + lane * 4);
            v[0] = pv.x; v[1] = pv.y; v[2] = pv.z; v[3] = pv.w;
            h128_warp4(v);
            const uint2 sraw = *reinterpret_cast<const uint2 *>(P.sv + nb * 128 + lane * 4);
            const __half2 s01 = bits_half2(sraw.x), s23 = bits_half2(sraw.y);
            float4 o;
            o.x = __fmul_rn(v[0], __low2float(s01));
            o.y = __fmul_rn(v[1], __high2float(s01));
            o.z = __fmul_rn(v[2], __low2float(s23));
            o.w = __fmul_rn(v[3], __high2float(s23));
            *reinterpret_cast<float4 *>(P.y + size_t(r) * P.y_stride + nb * 128 + lane * 4) = o;
        }
    }
    cluster.sync();  // keep every rank's shared memory alive until rank 0 has read it
}

// ---------------------------------------------------------------------------

int choose_cluster_splits(int sms, int nunits, int min_nchunks) {
    const char * env = std::getenv("EXL3CU_CLUSTER_SPLITS");  // tuning experiments only
    if (env && std::atoi(env) > 0) return std::min(16, std::atoi(env));
    int s = 1;
    while (s < 16 && long(nunits) * (s * 2) <= long(sms) * 4 && min_nchunks / (s * 2) >= kCWarps) s *= 2;
    return s;
}

size_t cluster_smem_bytes(int max_cps, int rows) {
    const int ng_max = (max_cps + 7) / 8 + 1;
    const size_t xs_bytes = size_t(rows) * (ng_max * 128 + 8) * 2;
    const size_t red_bytes = size_t(kCWarps + 1) * rows * 128 * 4;
    return std::max(xs_bytes, red_bytes);
}

template <int BITS, unsigned CB>
static cudaError_t launch_cluster_one(const GemvBatch & b, int nunits, size_t smem, bool pdl, cudaStream_t st) {
    auto kern = k_gemv_cluster<BITS, CB>;
    cudaError_t e;
    if (b.splits > 8) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    if (smem > 48 * 1024) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(nunits * b.splits), 1, 1);
    cfg.blockDim = dim3(kCWarps * 32, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = unsigned(b.splits);
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, b);
}

template <int BITS>
static cudaError_t launch_cluster_bits(const GemvBatch & b, int nunits, size_t smem, unsigned cb, bool pdl,
                                       cudaStream_t st) {
    switch (cb) {
        case CB_MUL1: return launch_cluster_one<BITS, CB_MUL1>(b, nunits, smem, pdl, st);
        case CB_MCG: return launch_cluster_one<BITS, CB_MCG>(b, nunits, smem, pdl, st);
        default: return launch_cluster_one<BITS, CB_3INST>(b, nunits, smem, pdl, st);
    }
}

cudaError_t launch_gemv_cluster(const GemvBatch & b, int nunits, size_t smem, unsigned bits, unsigned cb, bool pdl,
                                cudaStream_t st) {
    switch (bits) {
        case 1: return launch_cluster_bits<1>(b, nunits, smem, cb, pdl, st);
        case 2: return launch_cluster_bits<2>(b, nunits, smem, cb, pdl, st);
        case 3: return launch_cluster_bits<3>(b, nunits, smem, cb, pdl, st);
        case 4: return launch_cluster_bits<4>(b, nunits, smem, cb, pdl, st);
        case 5: return launch_cluster_bits<5>(b, nunits, smem, cb, pdl, st);
        case 6: return launch_cluster_bits<6>(b, nunits, smem, cb, pdl, st);
        case 7: return launch_cluster_bits<7>(b, nunits, smem, cb, pdl, st);
        case 8: return launch_cluster_bits<8>(b, nunits, smem, cb, pdl, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace exl3cu
