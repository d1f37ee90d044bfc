// The mul1 EXL3 GEMV (rows <= 4 per launch, bitrates 2..8): the operator
// behind exl3cu_mul_mat for the runtime format's codebook.
//
// Math (reference: ggml_exl3_mul_mat, src/exl3-ggml.cpp:51-92; codebook
// src/exl3_codec.cpp:68-76).  A mul1 weight is w = a*(1024 + s) + b with
// s = bytesum(state * 0x83dcd12d), a = fp16 0x1eee = 1774/2^18 and
// b = fp16 0xc931 = -1329/128; the reference evaluates a*(1024+s)+b exactly
// (it has at most 21 significant bits) and rounds it once to fp16.  So for
// rotated activations xh,
//
//     sum_k xh_k w_k  =  a * sum_k xh_k s_k  +  c * sum_k xh_k,   c = 1024a + b = -3.453125,
//
// evaluated here with the codebook's exact values (the reference's fp16
// rounding of w moves y by ~1e-4 relative, far inside the 2e-3 bar).  The
// activations are held as fixed point, xh = scale * q, q split into signed
// 7/8-bit digits: three (22 bits) when a problem has one or two rows, two (15
// bits) for three or four.  sum_k q_k s_k is one integer tensor-core product:
// mma.m16n8k32 u8 x s8 -> s32 with A = the four bytes of every state's
// product (so the K dimension sums the bytes: the byte sum costs nothing),
// B = the digits of q replicated over each product's four bytes.  The row x
// digit columns fill the instruction's N = 8.  Per 8 trellis states a lane spends ~10 integer ops extracting
// the 16-bit windows (byte permutes on a nibble-shifted copy at 4 bpw), 8
// IMADs and 2 IMMAs -- no fp16 conversion, no packing, no HMMA.
//
// Pipeline: one producer warp streams the CTA's contiguous weight range into
// a 4-stage shared-memory ring with bulk copies (cp.async.bulk, no
// multicast) on mbarriers; eight consumer warps decode from shared memory.
// The K split runs across a thread-block cluster and is reduced through
// distributed shared memory by cluster rank 0, which applies H128 and sv.
// With a peer output (a column split over GPUs) rank 0 of every column block
// stores its y block into every rank's buffer over NVLink as self-validating
// (epoch, value) words: the GEMV and its all-gather are one kernel, with no
// fence and no flag.
// Programmatic dependent launch: weights stream before griddepcontrol.wait
// (marked evict-first in L2, so activations stay there); only the activation
// prologue waits for the previous kernel.  Warp reductions use redux.sync.
// Every mbarrier wait is bounded (exl3cu_async.cuh).
#include "exl3cu_async.cuh"
#include "exl3cu_internal.h"
#include "exl3cu_mul1.cuh"

#include <cooperative_groups.h>

#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>

namespace cg = cooperative_groups;

namespace exl3cu {

static __device__ unsigned g_mul1_status;
static_assert(kMRows <= kMW, "the epilogue gives each row its own consumer warp");  // kStatus* bits raised by k_gemv_mul1

constexpr int kQLim2 = 16000;    // |q| with two digits: hi in [-125,125], lo in [-64,63]
constexpr int kQLim3 = 2000000;  // |q| with three digits: hi in [-123,123]

__host__ __device__ inline int mul1_digits(int rows) { return rows <= 2 ? 3 : 2; }

struct Mul1Layout {
    int ring_off, xq_off, acc_off, part_off, slot_off, gmax_off, qs_off, nw_off, bar_off;
    size_t bytes;
};

// ring: kMStages stages of kMW chunks; xq: activation digits of the CTA's K
// range (64 bytes per digit column per chunk); acc: the CTA's integer sums
// [rows][128][digits]; part: its fp32 partial; slot: the other cluster ranks'
// partials (written remotely, read by rank 0); gmax: max |xh| per (row, own
// group); qs: the digit sum of every (row, own group); nw (RMSNorm form, when
// staged): the norm weights of the CTA's groups; then the mbarriers and per-row
// scale / inverse norm.
__host__ __device__ inline Mul1Layout mul1_layout(int bits, int cps, int rows, int splits, int stages,
                                                  bool nw_smem) {
    Mul1Layout L;
    const int ng = (cps + 7) / 8 + 1;
    const int dig = mul1_digits(rows);
    const size_t ring = size_t(stages) * kMW * 256 * bits;
    const size_t xq = size_t(cps) * 64 * dig * rows;
    const size_t acc = size_t(rows) * 128 * dig * 4;
    const size_t part = size_t(rows) * 128 * 4;
    const size_t slot = size_t(splits > 1 ? splits - 1 : 0) * rows * 128 * 4;
    const size_t gmax = size_t(rows) * ng * 4;
    L.ring_off = 0;
    L.xq_off = int(ring);
    L.acc_off = int((ring + xq + 15) & ~size_t(15));
    L.part_off = int(L.acc_off + acc);
    L.slot_off = int(L.part_off + part);
    L.gmax_off = int(L.slot_off + slot);
    L.qs_off = int(L.gmax_off + gmax);
    L.nw_off = int((L.qs_off + gmax + 15) & ~size_t(15));
    L.bar_off = L.nw_off + (nw_smem ? ng * 128 * 4 : 0);
    L.bytes = L.bar_off + 2 * stages * 8 + 2 * 4 * kMRows;  // + per-row scale, inverse norm
    return L;
}

// The kernel body.  PEER: the output goes to the peers' buffers (a column split).  WIDE: the build
// for long K ranges per CTA (two CTAs per SM, 95 registers), whose decode keeps two tiles' products
// in flight; the default build keeps three CTAs per SM at 72 registers.
template <int BITS, bool PEER, bool WIDE>
__device__ __forceinline__ void gemv_mul1_body(const GemvBatch & b) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int CHUNKB = 256 * BITS;
    pdl_trigger();

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
    const int rows = P.rows;
    const int dig = mul1_digits(rows);
    const int nd = dig * rows;  // B columns in use
    const int xqc = 64 * nd;    // digit bytes per chunk
    const int c0 = min(split * P.cps, P.nchunks);
    const int c1 = min(c0 + P.cps, P.nchunks);
    const int nch = c1 - c0;
    const int nstage = (nch + kMW - 1) / kMW;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    const int NS = b.stages;
    const Mul1Layout L = mul1_layout(BITS, P.cps, rows, S, NS, b.nw_smem != 0);
    unsigned char * ring = smem + L.ring_off;
    unsigned char * xq = smem + L.xq_off;
    int * acc = reinterpret_cast<int *>(smem + L.acc_off);          // [rows][128][2]
    float * part = reinterpret_cast<float *>(smem + L.part_off);    // [rows][128]
    float * slots = reinterpret_cast<float *>(smem + L.slot_off);   // [S-1][rows][128]
    float * gmax = reinterpret_cast<float *>(smem + L.gmax_off);    // [rows][ng]
    int * qs = reinterpret_cast<int *>(smem + L.qs_off);            // [rows][ng] digit sums
    float * nws = reinterpret_cast<float *>(smem + L.nw_off);       // [ng][128] (staged RMSNorm weights)
    uint64_t * full = reinterpret_cast<uint64_t *>(smem + L.bar_off);
    uint64_t * empty = full + NS;
    float * scale_s = reinterpret_cast<float *>(empty + NS);
    float * invn_s = scale_s + kMRows;  // kXRmsNorm: 1/rms of each row
    const int nacc = rows * 128 * dig;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kMW);
        }
        mbar_init_fence();
    }
    for (int e = threadIdx.x; e < nacc; e += kMThreads) acc[e] = 0;
    if (threadIdx.x < kMRows) scale_s[threadIdx.x] = 1.0f;  // a CTA without chunks contributes scale * 0
    __syncthreads();

    uint2 sv_pre = make_uint2(0, 0);                    // rank 0: output signs of this lane's columns
    float4 y_prev = make_float4(0.f, 0.f, 0.f, 0.f);    // rank 0, y_accum: y of row `warp` before this launch
    if (warp == kMW) {
        // ---- producer: the CTA's chunks [c0, c1) are contiguous in the device layout ----
        if (lane == 0 && nch > 0) {
            const uint64_t pol = l2_evict_first_policy();  // weights are read once per pass
            const unsigned char * src = reinterpret_cast<const unsigned char *>(P.lsc) +
                                        (size_t(nb) * P.nchunks + c0) * CHUNKB;
            for (int j = 0, s = 0, round = 0; j < nstage; ++j) {
                if (j >= NS && !mbar_wait(&empty[s], (round - 1) & 1)) {
                    atomicOr(&g_mul1_status, kStatusWaitTimeout);
                    break;
                }
                const int nc = min(kMW, nch - j * kMW);
                mbar_arrive_expect_tx(&full[s], uint32_t(nc * CHUNKB));
                bulk_g2s_hint(ring + size_t(s) * kMW * CHUNKB, src + size_t(j) * kMW * CHUNKB, uint32_t(nc * CHUNKB),
                              &full[s], pol);
                if (++s == NS) {
                    s = 0;
                    ++round;
                }
            }
        }
        __syncwarp();
    } else {
        // ---- consumers ----
        const int g0 = c0 >> 3;
        const int ng = nch > 0 ? ((c1 - 1) >> 3) - g0 + 1 : 0;
        const int kbeg = c0 * 16, kend = c1 * 16;
        constexpr int kItems = 4;
        const int nitems = ng * rows;
        // the input signs are constants: fetch the register-cached items' su before the wait
        uint2 su_pre[kItems];
#pragma unroll
        for (int ii = 0; ii < kItems; ++ii) {
            const int item = warp + ii * kMW;
            su_pre[ii] = make_uint2(0, 0);
            if (item < nitems) su_pre[ii] = *reinterpret_cast<const uint2 *>(P.su + (g0 + item / rows) * 128 + lane * 4);
        }
        if (split == 0) sv_pre = *reinterpret_cast<const uint2 *>(P.sv + nb * 128 + lane * 4);
        const int ktot = P.nchunks * 16;
        // RMSNorm weights of the CTA's groups (a layer constant): staged in shared memory before the
        // wait when the launch has room for them (read after a barrier below), else read from L2
        const bool staged = P.x_mode == kXRmsNorm && b.nw_smem;
        if (staged)
            for (int e = threadIdx.x * 4; e < ng * 128; e += kMW * 32 * 4)
                *reinterpret_cast<float4 *>(nws + e) = g0 * 128 + e < ktot
                                                           ? *reinterpret_cast<const float4 *>(P.nw + g0 * 128 + e)
                                                           : make_float4(0.f, 0.f, 0.f, 0.f);
        auto norm_w4 = [&](int kcol) {  // RMSNorm weights k .. k+3
            return staged ? *reinterpret_cast<const float4 *>(nws + (kcol - g0 * 128))
                          : *reinterpret_cast<const float4 *>(P.nw + kcol);
        };
        pdl_wait_primary();  // activations may be written by the previous kernel
        float v[kItems][4];
        if (P.x_mode == kXRmsNorm) {
            // the register-cached items' raw h goes out with the full-row loads below (one round trip)
#pragma unroll
            for (int ii = 0; ii < kItems; ++ii) {
                const int item = warp + ii * kMW;
                if (item < nitems) {
                    const int gi = item / rows;
                    const float4 hv = *reinterpret_cast<const float4 *>(
                        static_cast<const float *>(P.x) + size_t(item - gi * rows) * P.x_stride + (g0 + gi) * 128 + lane * 4);
                    v[ii][0] = hv.x; v[ii][1] = hv.y; v[ii][2] = hv.z; v[ii][3] = hv.w;
                }
            }
            if (P.x_ss) {
                // the producer's sums of squares per 128-block: warp r adds row r's (fixed tree)
                const int nbk = ktot / 128;
                if (warp < rows) {
                    float ss = 0.f;
                    for (int bk = lane; bk < nbk; bk += 32) ss += P.x_ss[size_t(warp) * nbk + bk];
#pragma unroll
                    for (int sh = 16; sh; sh >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, sh);
                    if (lane == 0) invn_s[warp] = rsqrtf(ss / float(ktot) + P.eps);
                }
                consumer_sync();
            } else {
                // every CTA takes the whole row's mean square (from L2) before normalising its K range
                float * red = part;  // scratch until the epilogue: [kMW][rows]
                for (int r = 0; r < rows; ++r) {
                    const float * hr = static_cast<const float *>(P.x) + size_t(r) * P.x_stride;
                    float ss = 0.f;
                    for (int i = threadIdx.x * 4; i < ktot; i += kMW * 32 * 4) {
                        const float4 v = *reinterpret_cast<const float4 *>(hr + i);
                        ss = fmaf(v.x, v.x, ss);
                        ss = fmaf(v.y, v.y, ss);
                        ss = fmaf(v.z, v.z, ss);
                        ss = fmaf(v.w, v.w, ss);
                    }
#pragma unroll
                    for (int sh = 16; sh; sh >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, sh);
                    if (lane == 0) red[warp * rows + r] = ss;
                }
                consumer_sync();
                if (threadIdx.x < rows) {
                    float ss = 0.f;
                    for (int w = 0; w < kMW; ++w) ss += red[w * rows + threadIdx.x];
                    invn_s[threadIdx.x] = rsqrtf(ss / float(ktot) + P.eps);
                }
                consumer_sync();
            }
        }
        auto load_x = [&](int r, int kcol, float (&o)[4]) {
            if (P.x_mode == kXGlu) {
                const float * xr = static_cast<const float *>(P.x) + size_t(r) * P.x_stride;
                const float4 g = *reinterpret_cast<const float4 *>(xr + kcol);
                const float4 u = *reinterpret_cast<const float4 *>(xr + ktot + kcol);
                o[0] = g.x / (1.0f + expf(-g.x)) * u.x;
                o[1] = g.y / (1.0f + expf(-g.y)) * u.y;
                o[2] = g.z / (1.0f + expf(-g.z)) * u.z;
                o[3] = g.w / (1.0f + expf(-g.w)) * u.w;
                return;
            }
            if (P.x_mode == kXRmsNorm) {
                const float4 hv = *reinterpret_cast<const float4 *>(static_cast<const float *>(P.x) +
                                                                    size_t(r) * P.x_stride + kcol);
                const float4 wv = norm_w4(kcol);
                const float inv = invn_s[r];
                o[0] = hv.x * inv * wv.x;
                o[1] = hv.y * inv * wv.y;
                o[2] = hv.z * inv * wv.z;
                o[3] = hv.w * inv * wv.w;
                return;
            }
            if (P.x_f16) {
                const uint2 raw = *reinterpret_cast<const uint2 *>(static_cast<const __half *>(P.x) +
                                                                   size_t(r) * P.x_stride + kcol);
                const __half2 lo = bits_half2(raw.x), hi = bits_half2(raw.y);
                o[0] = __low2float(lo); o[1] = __high2float(lo); o[2] = __low2float(hi); o[3] = __high2float(hi);
            } else {
                const float4 f = *reinterpret_cast<const float4 *>(static_cast<const float *>(P.x) +
                                                                   size_t(r) * P.x_stride + kcol);
                o[0] = f.x; o[1] = f.y; o[2] = f.z; o[3] = f.w;
            }
        };
        auto apply_su = [&](uint2 sraw, float (&o)[4]) {
            const __half2 s01 = bits_half2(sraw.x), s23 = bits_half2(sraw.y);
            o[0] = __fmul_rn(o[0], __low2float(s01));
            o[1] = __fmul_rn(o[1], __high2float(s01));
            o[2] = __fmul_rn(o[2], __low2float(s23));
            o[3] = __fmul_rn(o[3], __high2float(s23));
        };
        auto load_xsu = [&](int r, int kcol, float (&o)[4]) {
            load_x(r, kcol, o);
            apply_su(*reinterpret_cast<const uint2 *>(P.su + kcol), o);
        };
        // (1) the CTA's (group, row) items round robin over warps: xh = H128(x * su), the
        //     first kItems kept in registers, each group's max |xh| published
        auto rotate_from = [&](int item, float (&o)[4]) {  // o already holds x * su
            const int gi = item / rows;
            const int r = item - gi * rows;
            h128_warp4(o);
            // max over the warp of non-negative floats: their bit patterns order as unsigned integers
            const float m = __uint_as_float(__reduce_max_sync(
                0xffffffffu, __float_as_uint(fmaxf(fmaxf(fabsf(o[0]), fabsf(o[1])), fmaxf(fabsf(o[2]), fabsf(o[3]))))));
            if (lane == 0) gmax[r * ng + gi] = m;
        };
        auto rotate = [&](int item, float (&o)[4]) {
            const int gi = item / rows;
            const int r = item - gi * rows;
            load_xsu(r, (g0 + gi) * 128 + lane * 4, o);
            rotate_from(item, o);
        };
#pragma unroll
        for (int ii = 0; ii < kItems; ++ii) {
            const int item = warp + ii * kMW;
            if (item < nitems) {
                const int gi = item / rows;
                const int kcol = (g0 + gi) * 128 + lane * 4;
                if (P.x_mode == kXRmsNorm) {  // raw h already loaded: normalise
                    const float4 wv = norm_w4(kcol);
                    const float inv = invn_s[item - gi * rows];
                    v[ii][0] = v[ii][0] * inv * wv.x;
                    v[ii][1] = v[ii][1] * inv * wv.y;
                    v[ii][2] = v[ii][2] * inv * wv.z;
                    v[ii][3] = v[ii][3] * inv * wv.w;
                } else {
                    load_x(item - gi * rows, kcol, v[ii]);
                }
            }
        }
#pragma unroll
        for (int ii = 0; ii < kItems; ++ii) {
            const int item = warp + ii * kMW;
            if (item < nitems) {
                apply_su(su_pre[ii], v[ii]);
                rotate_from(item, v[ii]);
            }
        }
        for (int item = warp + kItems * kMW; item < nitems; item += kMW) {
            float o[4];
            rotate(item, o);
        }
        consumer_sync();
        // (2) per row, scale = max |xh| / qlim over the CTA's groups; each warp quantizes the
        //     items it rotated into the digit layout and records their digit sums (integer)
        const int qlim = dig == 3 ? kQLim3 : kQLim2;
        auto quantize = [&](int item, const float (&o)[4]) {
            const int gi = item / rows;
            const int r = item - gi * rows;
            float amax = 0.f;
            for (int q = 0; q < ng; ++q) amax = fmaxf(amax, gmax[r * ng + q]);
            const float scale = amax > 0.f ? amax / float(qlim) : 1.0f;
            const float inv = 1.0f / scale;
            int qsum = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int k = (g0 + gi) * 128 + lane * 4 + e;
                if (k < kbeg || k >= kend) continue;
                int q = __float2int_rn(o[e] * inv);
                q = max(-qlim, min(qlim, q));
                qsum += q;
                const int kl = k - kbeg;
                const int cl = kl >> 4, kk = kl & 15;
                unsigned char * base = xq + size_t(cl) * xqc + ((kk & 7) >> 1) * 16 + ((kk & 1) + 2 * (kk >> 3)) * 4;
                const int lo = ((q + 64) & 127) - 64;
                const int rest = (q - lo) >> 7;
                if (dig == 3) {
                    const int mid = ((rest + 64) & 127) - 64;
                    const int hi = (rest - mid) >> 7;
                    *reinterpret_cast<uint32_t *>(base + (3 * r) * 64) = uint32_t(uint8_t(int8_t(hi))) * 0x01010101u;
                    *reinterpret_cast<uint32_t *>(base + (3 * r + 1) * 64) = uint32_t(uint8_t(int8_t(mid))) * 0x01010101u;
                    *reinterpret_cast<uint32_t *>(base + (3 * r + 2) * 64) = uint32_t(uint8_t(int8_t(lo))) * 0x01010101u;
                } else {
                    *reinterpret_cast<uint32_t *>(base + (2 * r) * 64) = uint32_t(uint8_t(int8_t(rest))) * 0x01010101u;
                    *reinterpret_cast<uint32_t *>(base + (2 * r + 1) * 64) = uint32_t(uint8_t(int8_t(lo))) * 0x01010101u;
                }
            }
            qsum = __reduce_add_sync(0xffffffffu, qsum);  // |qsum| <= 128 * kQLim3 < 2^31
            if (lane == 0) {
                qs[r * ng + gi] = qsum;
                if (gi == 0) scale_s[r] = scale;
            }
        };
#pragma unroll
        for (int ii = 0; ii < kItems; ++ii) {
            const int item = warp + ii * kMW;
            if (item < nitems) quantize(item, v[ii]);
        }
        for (int item = warp + kItems * kMW; item < nitems; item += kMW) {
            // beyond the register cache: rotate again (republishing the same max)
            float o[4];
            rotate(item, o);
            quantize(item, o);
        }
        consumer_sync();
        // (3) decode + integer tensor-core products
        const int src = (lane + 31) & 31;
        const bool b_live = lane < 4 * nd;  // B column lane/4 = dig*row + digit exists
        constexpr uint32_t C = 0x83dcd12du;
        int D[8][4];
#pragma unroll
        for (int c = 0; c < 8; ++c) D[c][0] = D[c][1] = D[c][2] = D[c][3] = 0;
        for (int j = 0, s = 0, round = 0; j < nstage; ++j) {
            const int cl = warp + j * kMW;
            if (cl >= nch) break;
            uint4 bq = make_uint4(0, 0, 0, 0);
            if (b_live) bq = *reinterpret_cast<const uint4 *>(xq + size_t(cl) * xqc + lane * 16);
            if (!mbar_wait(&full[s], round & 1)) {
                atomicOr(&g_mul1_status, kStatusWaitTimeout);
                break;
            }
            uint32_t w[2 * BITS];
            const unsigned char * seg = ring + size_t(s) * kMW * CHUNKB + size_t(warp) * CHUNKB + lane * 8 * BITS;
            if constexpr ((BITS & 1) == 0) {
#pragma unroll
                for (int i = 0; i < BITS / 2; ++i) {
                    const uint4 q4 = *reinterpret_cast<const uint4 *>(seg + 16 * i);
                    w[4 * i] = q4.x; w[4 * i + 1] = q4.y; w[4 * i + 2] = q4.z; w[4 * i + 3] = q4.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < BITS; ++i) {
                    const uint2 q2 = *reinterpret_cast<const uint2 *>(seg + 8 * i);
                    w[2 * i] = q2.x; w[2 * i + 1] = q2.y;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            // products of all 8 tiles first, then the 16 IMMAs ordered so that no two
            // consecutive ones share an accumulator
            if constexpr (WIDE) {
                // tile pairs: the products of two tiles, then their four IMMAs
#pragma unroll
                for (int c = 0; c < 8; c += 2) {
                    uint32_t pa[8], pb[8];
                    {
                        uint32_t st[8];
                        tile_states<BITS>(w, c, src, st);
#pragma unroll
                        for (int e = 0; e < 8; ++e) pa[e] = st[e] * C;
                    }
                    {
                        uint32_t st[8];
                        tile_states<BITS>(w, c + 1, src, st);
#pragma unroll
                        for (int e = 0; e < 8; ++e) pb[e] = st[e] * C;
                    }
                    imma_u8s8(D[c], pa[0], pa[4], pa[1], pa[5], bq.x, bq.y);
                    imma_u8s8(D[c + 1], pb[0], pb[4], pb[1], pb[5], bq.x, bq.y);
                    imma_u8s8(D[c], pa[2], pa[6], pa[3], pa[7], bq.z, bq.w);
                    imma_u8s8(D[c + 1], pb[2], pb[6], pb[3], pb[7], bq.z, bq.w);
                }
            } else {
                uint32_t pr[8][8];
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    uint32_t st[8];
                    tile_states<BITS>(w, c, src, st);
#pragma unroll
                    for (int e = 0; e < 8; ++e) pr[c][e] = st[e] * C;
                }
#pragma unroll
                for (int c = 0; c < 8; ++c) imma_u8s8(D[c], pr[c][0], pr[c][4], pr[c][1], pr[c][5], bq.x, bq.y);
#pragma unroll
                for (int c = 0; c < 8; ++c) imma_u8s8(D[c], pr[c][2], pr[c][6], pr[c][3], pr[c][7], bq.z, bq.w);
            }
            if (++s == NS) {
                s = 0;
                ++round;
            }
        }
        // (4) the warps' integer sums meet in shared memory (exact, any order) ...
        {
            const int g = lane >> 2, t = lane & 3;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int n = 2 * t + i;  // B column: row n / dig, digit n % dig
                if (n < nd) {
                    const int rr = n / dig;
                    int * a0 = acc + (rr * 128 + g) * dig + (n - rr * dig);
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        atomicAdd(a0 + c * 16 * dig, D[c][i]);
                        atomicAdd(a0 + (c * 16 + 8) * dig, D[c][i + 2]);  // column + 8
                    }
                }
            }
        }
        consumer_sync();
        // ... and become the CTA's fp32 partial scale * (a * sum q s + c * sum q), written straight
        //     into rank 0's slot for this rank (rank 0 keeps its own in `part`)
        float * dst = split == 0 ? part : cluster.map_shared_rank(slots, 0) + size_t(split - 1) * rows * 128;
        for (int e = threadIdx.x; e < rows * 128; e += kMW * 32) {
            const int r = e >> 7;
            const int * a = acc + e * dig;
            const double sq = dig == 3 ? (double(a[0]) * 16384.0 + double(a[1]) * 128.0) + double(a[2])
                                       : double(a[0]) * 128.0 + double(a[1]);
            long long qsum = 0;
            for (int q = 0; q < ng; ++q) qsum += qs[r * ng + q];
            dst[e] = float(double(scale_s[r]) * (double(kCodeA) * sq + double(kCodeC) * double(qsum)));
        }
        // the accumulated y goes out before the barrier (nothing else writes it during this launch)
        if (split == 0 && P.y_accum && warp < rows)
            y_prev = *reinterpret_cast<const float4 *>(P.y + size_t(warp) * P.y_stride + nb * 128 + lane * 4);
    }

    // ---- one cluster barrier; rank 0 sums the partials in rank order ----
    cluster.sync();
    if (split == 0 && warp < kMW) {
        const int elems = rows * 128;
        if (S > 1) {
            // every consumer thread sums a few elements over the ranks (in rank order), in place
            for (int e = threadIdx.x; e < elems; e += kMW * 32) {
                float a = part[e];
                for (int rk = 1; rk < S; ++rk) a = __fadd_rn(a, slots[size_t(rk - 1) * elems + e]);
                part[e] = a;
            }
            consumer_sync();
        }
        const __half2 s01 = bits_half2(sv_pre.x), s23 = bits_half2(sv_pre.y);
        // column split over GPUs: this call's epoch picks the half of every rank's y buffer
        constexpr bool to_peers = PEER;  // a separate build, so the plain kernel carries none of this
        const unsigned epoch =
            to_peers ? *reinterpret_cast<const volatile unsigned *>(b.peer.own_state + kPeerEpochWord) + 1u : 0u;
        for (int r = warp; r < rows; r += kMW) {
            float v[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) v[q] = part[r * 128 + lane * 4 + q];
            h128_warp4(v);
            float4 o;
            o.x = __fmul_rn(v[0], __low2float(s01));
            o.y = __fmul_rn(v[1], __high2float(s01));
            o.z = __fmul_rn(v[2], __low2float(s23));
            o.w = __fmul_rn(v[3], __high2float(s23));
            float4 * yp = reinterpret_cast<float4 *>(P.y + size_t(r) * P.y_stride + nb * 128 + lane * 4);
            if (P.y_accum) {  // rows <= kMRows <= kMW: warp r prefetched row r
                o.x += y_prev.x;
                o.y += y_prev.y;
                o.z += y_prev.z;
                o.w += y_prev.w;
            }
            if constexpr (to_peers) {  // NVLink stores of (epoch, value) words into every rank's y
                const long long off = ((epoch & 1u) ? b.peer.y_half : 0) + r * b.peer.y_stride + b.peer.y_col0 +
                                      nb * 128 + lane * 4;
                for (int pi = 0; pi < b.peer.npeers; ++pi) store_pairs4(b.peer.y[pi] + off, o, epoch);
            } else {
                *yp = o;
            }
            if (P.y_ss) {  // this block's sum of squares of the final y, for a later RMSNorm of the row
                float ss = o.x * o.x;
                ss = fmaf(o.y, o.y, ss);
                ss = fmaf(o.z, o.z, ss);
                ss = fmaf(o.w, o.w, ss);
#pragma unroll
                for (int sh = 16; sh; sh >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, sh);
                if (lane == 0) P.y_ss[size_t(r) * P.y_ss_stride + nb] = ss;
            }
        }
    }
}

template <int BITS, bool PEER>
__global__ void __launch_bounds__(kMThreads) k_gemv_mul1(const GemvBatch b) {
    gemv_mul1_body<BITS, PEER, false>(b);
}

template <int BITS, bool PEER>
__global__ void __launch_bounds__(kMThreads, 2) k_gemv_mul1_wide(const GemvBatch b) {
    gemv_mul1_body<BITS, PEER, true>(b);
}

// ---------------------------------------------------------------------------

namespace {

// Kernel variants: bit 0 peer output, bit 1 the wide build.
constexpr int kVarDefault = 0, kVarPeer = 1, kVarWide = 2;
constexpr int kWideMinChunks = 512;  // k / 16 from which a problem takes the wide build

template <int BITS>
void * mul1_kernel(int var) {
    switch (var) {
        case kVarPeer: return reinterpret_cast<void *>(k_gemv_mul1<BITS, true>);
        case kVarWide: return reinterpret_cast<void *>(k_gemv_mul1_wide<BITS, false>);
        case kVarPeer | kVarWide: return reinterpret_cast<void *>(k_gemv_mul1_wide<BITS, true>);
        default: return reinterpret_cast<void *>(k_gemv_mul1<BITS, false>);
    }
}

void * mul1_kernel_for(unsigned bits, int var = kVarDefault) {
    switch (bits) {
        case 2: return mul1_kernel<2>(var);
        case 3: return mul1_kernel<3>(var);
        case 4: return mul1_kernel<4>(var);
        case 5: return mul1_kernel<5>(var);
        case 6: return mul1_kernel<6>(var);
        case 7: return mul1_kernel<7>(var);
        case 8: return mul1_kernel<8>(var);
        default: return nullptr;
    }
}

constexpr size_t kMul1MaxSmem = 200 * 1024;

// Set the kernel's shared-memory and cluster attributes once per (device, bits).
bool mul1_prepare(int device, unsigned bits) {
    static std::mutex mu;
    static bool done[64][9] = {};
    if (device < 0 || device >= 64 || bits > 8) return false;
    std::lock_guard<std::mutex> g(mu);
    if (done[device][bits]) return true;
    for (const int var : {kVarDefault, kVarPeer, kVarWide, kVarPeer | kVarWide}) {
        const void * k = mul1_kernel_for(bits, var);
        if (!k) return false;
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMul1MaxSmem)) != cudaSuccess)
            return false;
        if (cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) return false;
    }
    done[device][bits] = true;
    return true;
}

// Clusters of `cs` CTAs with `smem` bytes each that the device holds at once
// (0 when such a cluster cannot be scheduled at all); cached per key.
int mul1_active_clusters(int device, unsigned bits, int cs, size_t smem, int var) {
    static std::mutex mu;
    static std::map<std::tuple<int, unsigned, int, size_t, int>, int> cache;
    const auto key = std::make_tuple(device, bits, cs, (smem + 1023) / 1024, var);
    {
        std::lock_guard<std::mutex> g(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(cs), 1, 1);
    cfg.blockDim = dim3(kMThreads, 1, 1);
    cfg.dynamicSmemBytes = ((smem + 1023) / 1024) * 1024;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = unsigned(cs);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, mul1_kernel_for(bits, var), &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        n = 0;
    }
    std::lock_guard<std::mutex> g(mu);
    cache[key] = n;
    return n;
}

}  // namespace

// Weight ring depth in stages of kMW chunks: EXL3CU_MUL1_STAGES (tuning
// experiments), else kMStages.
int mul1_stages(unsigned bits) {
    const char * env = std::getenv("EXL3CU_MUL1_STAGES");
    int ns = env ? std::atoi(env) : 0;
    if (ns <= 0) ns = kMStages;
    (void)bits;
    return std::min(ns, kMStagesMax);
}

bool mul1_supported(unsigned bits, int rows) { return bits >= 2 && bits <= 8 && rows >= 1 && rows <= kMRows; }

// Picks the cluster size (K split) so the grid fills the device in one wave:
// the largest S in 1..16 with nunits*S <= resident CTAs and at least one
// chunk per consumer warp for the smallest problem.
cudaError_t launch_gemv_mul1(GemvBatch & b, int nunits, int sms, int device, unsigned bits, bool pdl,
                             cudaStream_t st) {
    if (!mul1_prepare(device, bits)) return cudaErrorInvalidValue;
    int min_nchunks = 1 << 30, max_nchunks = 0, max_rows = 1;
    bool nw_smem = false;
    for (int i = 0; i < b.count; ++i) {
        nw_smem = nw_smem || b.prob[i].x_mode == kXRmsNorm;
        min_nchunks = std::min(min_nchunks, b.prob[i].nchunks);
        max_nchunks = std::max(max_nchunks, b.prob[i].nchunks);
        max_rows = std::max(max_rows, b.prob[i].rows);
    }
    // Long K (k >= 8192, every problem): many chunks per CTA, where the wide build's decode pays for its
    // lower occupancy (14336x4096 at 1 row: 21.4 -> 18.2 us); shorter K keeps the default build,
    // which the wide one slows by up to 20 % on the 2048-wide layer shapes.  EXL3CU_MUL1_WIDE=0/1
    // forces either (tuning experiments).
    const char * wenv = std::getenv("EXL3CU_MUL1_WIDE");
    const bool wide = wenv && wenv[0] ? wenv[0] == '1' : min_nchunks >= kWideMinChunks;
    const int var = (b.peer_on ? kVarPeer : 0) | (wide ? kVarWide : 0);
    const char * env = std::getenv("EXL3CU_CLUSTER_SPLITS");  // tuning experiments only
    const int NS = mul1_stages(bits);
    int S = 0;
    if (env && std::atoi(env) > 0) {
        S = std::min(16, std::atoi(env));
        nw_smem = false;
    } else {
        // largest cluster size whose grid is one wave; else the largest that can run at all.
        // EXL3CU_MUL1_CTAS_PER_SM (tuning experiments) caps the grid at that many CTAs per SM, leaving
        // room for the next launch's CTAs to start under programmatic dependent launch.
        const char * cap_env = std::getenv("EXL3CU_MUL1_CTAS_PER_SM");
        const int cap = cap_env && std::atoi(cap_env) > 0 ? std::atoi(cap_env) * sms : 1 << 30;
        auto choose = [&](bool staged, int & fit_out) {
            int feasible = 0, feasible_fit = 0;
            for (int cand = 16; cand >= 1; --cand) {
                if (cand > 1 && min_nchunks / cand < kMW) continue;
                const int cps = (max_nchunks + cand - 1) / cand;
                const Mul1Layout L = mul1_layout(int(bits), cps, max_rows, cand, NS, staged);
                if (L.bytes > kMul1MaxSmem) break;  // fewer splits only grow the per-CTA range
                const int fit = std::min(mul1_active_clusters(device, bits, cand, L.bytes, var), cap / cand);
                if (fit <= 0) continue;
                if (!feasible) {
                    feasible = cand;
                    feasible_fit = fit;
                }
                if (nunits <= fit) {
                    fit_out = fit;
                    return cand;
                }
            }
            fit_out = feasible_fit;
            return feasible;
        };
        int fit0 = 0, fit1 = 0;
        S = choose(false, fit0);
        // stage the RMSNorm weights only where that costs no occupancy: same split, same wave
        if (nw_smem) nw_smem = choose(true, fit1) == S && (fit1 >= nunits || fit1 == fit0);
    }
    if (S <= 0) return cudaErrorInvalidConfiguration;
    b.splits = S;
    int max_cps = 1;
    for (int i = 0; i < b.count; ++i) {
        b.prob[i].cps = (b.prob[i].nchunks + S - 1) / S;
        max_cps = std::max(max_cps, b.prob[i].cps);
    }
    const Mul1Layout L = mul1_layout(int(bits), max_cps, max_rows, S, NS, nw_smem);
    if (L.bytes > kMul1MaxSmem) return cudaErrorInvalidConfiguration;
    b.stages = NS;
    b.nw_smem = nw_smem ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(nunits * S), 1, 1);
    cfg.blockDim = dim3(kMThreads, 1, 1);
    cfg.dynamicSmemBytes = L.bytes;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = unsigned(S);
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = pdl ? 2 : 1;
    void * args[] = {&b};
    return cudaLaunchKernelExC(&cfg, mul1_kernel_for(bits, var), args);
}

cudaError_t mul1_read_status(unsigned * out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_mul1_status, sizeof(unsigned));
    if (e == cudaSuccess && clear && *out) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(g_mul1_status, &zero, sizeof(unsigned));
    }
    return e;
}

}  // namespace exl3cu
