// Persistent mul1 GEMV over a sequence of problems in dependency groups: one
// cooperative launch runs, e.g., a decode step's q,k,v | o | gate,up | down
// of every layer, instead of one launch per group.
//
// Per-problem math and numerics are those of k_gemv_mul1 (exl3cu_gemv_mul1.cu,
// after src/exl3-ggml.cpp:51-92): rotated activations as 15-bit fixed point per
// CTA, byte sums and products on the integer tensor cores, fp32 partials.
//
// Work units are (problem, column block, K split), numbered in group order and
// dealt round robin to the resident CTAs (grid = what the GPU holds at once,
// checked by the cooperative launch).  Each CTA's producer warp streams the
// trellis of all its units, one after another, through a 4-stage bulk-copy
// ring; the weights of later units do not depend on anything, so they stream
// while earlier groups are still being computed elsewhere.  Consumers wait for
// group g-1 to be complete before reading a group-g unit's activations (a
// counter raised with release semantics by the CTA that finishes each column
// block; read here with acquire semantics, activations then read through L2).
// The K split is reduced without cluster barriers, so that the producer never
// has to stop: every split writes its fp32 partial to a global slot, takes a
// ticket, and the last of a column block's splits sums the slots in split
// order (deterministic), applies H128 and sv and stores y.
//
// Deadlock freedom: a CTA waits only for strictly earlier groups, and every
// unit of an earlier group belongs to a resident CTA that reaches it before
// any later-group wait of its own (units are taken in increasing order).
// Every wait is bounded; a timeout sets the status word and skips the work.
#include "exl3cu_async.cuh"
#include "exl3cu_internal.h"
#include "exl3cu_mul1.cuh"

#include <mutex>

namespace exl3cu {

static __device__ unsigned g_seq_status;

constexpr unsigned kDepWaitRounds = 1u << 24;  // group-counter polls (each sleeps >= 64 ns): about a second or more

struct SeqLayout {
    int ring_off, xq_off, acc_off, part_off, gmax_off, bar_off;
    size_t bytes;
};

__host__ __device__ inline SeqLayout seq_layout(int bits, int cps_max) {
    SeqLayout L;
    const int ng = cps_max / 8 + 1;
    const size_t ring = size_t(kMStages) * kMW * 256 * bits;
    const size_t xq = size_t(cps_max) * 128 * kMRows;
    L.ring_off = 0;
    L.xq_off = int(ring);
    L.acc_off = int((ring + xq + 15) & ~size_t(15));
    L.part_off = L.acc_off + kMRows * 128 * 2 * 4;
    L.gmax_off = L.part_off + kMRows * 128 * 4;
    L.bar_off = int((L.gmax_off + kMRows * ng * 4 + 15) & ~15);
    L.bytes = L.bar_off + 2 * kMStages * 8 + 2 * 4 * kMRows + 16;  // + flag and abort words
    return L;
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned * p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Unit u -> (problem, column block, split).
__device__ __forceinline__ void seq_unit(const SeqArgs & a, int u, int & p, int & nb, int & split) {
    int lo = 0, hi = a.nprob - 1;  // last problem with unit_base <= u
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.prob[mid].unit_base <= u) lo = mid; else hi = mid - 1;
    }
    p = lo;
    const int local = u - a.prob[lo].unit_base;
    nb = local / a.prob[lo].splits;
    split = local - nb * a.prob[lo].splits;
}

template <int BITS>
__global__ void __launch_bounds__(kMThreads) k_gemv_persist(const __grid_constant__ SeqArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int CHUNKB = 256 * BITS;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    const SeqLayout L = seq_layout(BITS, a.cps_max);
    unsigned char * ring = smem + L.ring_off;
    unsigned char * xq = smem + L.xq_off;
    int * acc = reinterpret_cast<int *>(smem + L.acc_off);        // [rows][128][2]
    float * part = reinterpret_cast<float *>(smem + L.part_off);  // [rows][128]
    float * gmax = reinterpret_cast<float *>(smem + L.gmax_off);  // [rows][ng]
    uint64_t * full = reinterpret_cast<uint64_t *>(smem + L.bar_off);
    uint64_t * empty = full + kMStages;
    float * scale_s = reinterpret_cast<float *>(empty + kMStages);
    int * xsum_s = reinterpret_cast<int *>(scale_s + kMRows);
    int * flag_s = xsum_s + kMRows;  // "this CTA finishes the column block"
    int * abort_s = flag_s + 1;      // a wait of this launch ran out: stop at the next unit

    if (threadIdx.x == 0) {
        for (int s = 0; s < kMStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kMW);
        }
        mbar_init_fence();
    }
    __syncthreads();

    if (warp == kMW) {
        // ---- producer: the trellis of every unit of this CTA, in order ----
        if (lane == 0) {
            int j = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < a.nunits && ok; u += gridDim.x) {
                int p, nb, split;
                seq_unit(a, u, p, nb, split);
                const SeqProblem & P = a.prob[p];
                const int c0 = split * P.cps, c1 = min(c0 + P.cps, P.nchunks);
                const int nch = c1 - c0;
                const unsigned char * src = reinterpret_cast<const unsigned char *>(P.lsc) +
                                            (size_t(nb) * P.nchunks + c0) * CHUNKB;
                for (int jl = 0; jl * kMW < nch; ++jl, ++j) {
                    const int s = j % kMStages;
                    if (j >= kMStages && !mbar_wait_sleep(&empty[s], ((j / kMStages) - 1) & 1)) {
                        atomicOr(&g_seq_status, kStatusWaitTimeout);
                        atomicOr(a.abort, 1u);
                        ok = false;
                        break;
                    }
                    const int nc = min(kMW, nch - jl * kMW);
                    mbar_arrive_expect_tx(&full[s], uint32_t(nc * CHUNKB));
                    bulk_g2s(ring + size_t(s) * kMW * CHUNKB, src + size_t(jl) * kMW * CHUNKB, uint32_t(nc * CHUNKB),
                             &full[s]);
                }
            }
        }
        __syncwarp();
        return;  // the producer takes part in no barrier below (consumers use named barrier 1)
    }

    // ---- consumers ----
    const int src = (lane + 31) & 31;
    constexpr uint32_t C = 0x83dcd12du;
    int j = 0;  // ring stage, in step with the producer
    for (int u = blockIdx.x; u < a.nunits; u += gridDim.x) {
        int p, nb, split;
        seq_unit(a, u, p, nb, split);
        const SeqProblem & P = a.prob[p];
        const int rows = P.rows;
        const int c0 = split * P.cps, c1 = min(c0 + P.cps, P.nchunks);
        const int nch = c1 - c0;
        const int nstage = (nch + kMW - 1) / kMW;

        consumer_sync();  // the previous unit's readers of acc / part / xq are done
        for (int e = threadIdx.x; e < rows * 256; e += kMW * 32) acc[e] = 0;
        if (threadIdx.x < kMRows) {
            xsum_s[threadIdx.x] = 0;
            scale_s[threadIdx.x] = 1.0f;
        }
        if (threadIdx.x == 0) {
            if (a.depend && P.group > 0) {
                // group g reads what group g-1 wrote: wait until every column block of g-1 is stored
                const unsigned need = unsigned(a.group_need[P.group - 1]);
                unsigned r = 0;
                while (ld_acquire_gpu(&a.group_done[P.group - 1]) < need) {
                    if (++r >= kDepWaitRounds || ld_acquire_gpu(a.abort) != 0u) {
                        atomicOr(&g_seq_status, kStatusWaitTimeout);
                        atomicOr(a.abort, 1u);
                        break;
                    }
                    __nanosleep(64);
                }
            }
            *abort_s = ld_acquire_gpu(a.abort) != 0u;
        }
        consumer_sync();
        if (*abort_s) break;  // uniform across the consumer warps

        // (1)+(2) rotate, then quantize with the CTA's per-row scale (as k_gemv_mul1)
        const int g0 = c0 >> 3;
        const int ng = ((c1 - 1) >> 3) - g0 + 1;
        const int kbeg = c0 * 16, kend = c1 * 16;
        auto rotate = [&](int item, float (&o)[4]) {
            const int gi = item / rows;
            const int r = item - gi * rows;
            const int kcol = (g0 + gi) * 128 + lane * 4;
            if (P.x_f16) {
                const uint2 raw = __ldcg(reinterpret_cast<const uint2 *>(static_cast<const __half *>(P.x) +
                                                                         size_t(r) * P.x_stride + kcol));
                const __half2 lo = bits_half2(raw.x), hi = bits_half2(raw.y);
                o[0] = __low2float(lo); o[1] = __high2float(lo); o[2] = __low2float(hi); o[3] = __high2float(hi);
            } else {
                const float4 f = __ldcg(reinterpret_cast<const float4 *>(static_cast<const float *>(P.x) +
                                                                         size_t(r) * P.x_stride + kcol));
                o[0] = f.x; o[1] = f.y; o[2] = f.z; o[3] = f.w;
            }
            const uint2 sraw = *reinterpret_cast<const uint2 *>(P.su + kcol);
            const __half2 s01 = bits_half2(sraw.x), s23 = bits_half2(sraw.y);
            o[0] = __fmul_rn(o[0], __low2float(s01));
            o[1] = __fmul_rn(o[1], __high2float(s01));
            o[2] = __fmul_rn(o[2], __low2float(s23));
            o[3] = __fmul_rn(o[3], __high2float(s23));
            h128_warp4(o);
            float m = fmaxf(fmaxf(fabsf(o[0]), fabsf(o[1])), fmaxf(fabsf(o[2]), fabsf(o[3])));
#pragma unroll
            for (int sh = 16; sh; sh >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, sh));
            if (lane == 0) gmax[r * ng + gi] = m;
        };
        constexpr int kItems = 4;
        float v[kItems][4];
        const int nitems = ng * rows;
#pragma unroll
        for (int ii = 0; ii < kItems; ++ii) {
            const int item = warp + ii * kMW;
            if (item < nitems) rotate(item, v[ii]);
        }
        for (int item = warp + kItems * kMW; item < nitems; item += kMW) {
            float o[4];
            rotate(item, o);
        }
        consumer_sync();
        auto quantize = [&](int item, const float (&o)[4]) {
            const int gi = item / rows;
            const int r = item - gi * rows;
            float amax = 0.f;
            for (int q = 0; q < ng; ++q) amax = fmaxf(amax, gmax[r * ng + q]);
            const float scale = amax > 0.f ? amax / kQMax : 1.0f;
            const float inv = 1.0f / scale;
            int qsum = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int k = (g0 + gi) * 128 + lane * 4 + e;
                if (k < kbeg || k >= kend) continue;
                int q = __float2int_rn(o[e] * inv);
                q = max(-16000, min(16000, q));
                qsum += q;
                const int lo = ((q + 64) & 127) - 64;
                const int hi = (q - lo) >> 7;
                const int kl = k - kbeg;
                const int cl = kl >> 4, kk = kl & 15;
                unsigned char * base = xq + size_t(cl) * 128 * rows + ((kk & 7) >> 1) * 16 +
                                       ((kk & 1) + 2 * (kk >> 3)) * 4;
                *reinterpret_cast<uint32_t *>(base + (2 * r) * 64) = uint32_t(uint8_t(int8_t(hi))) * 0x01010101u;
                *reinterpret_cast<uint32_t *>(base + (2 * r + 1) * 64) = uint32_t(uint8_t(int8_t(lo))) * 0x01010101u;
            }
#pragma unroll
            for (int sh = 16; sh; sh >>= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, sh);
            if (lane == 0) {
                atomicAdd(&xsum_s[r], qsum);
                if (gi == 0) scale_s[r] = scale;
            }
        };
#pragma unroll
        for (int ii = 0; ii < kItems; ++ii) {
            const int item = warp + ii * kMW;
            if (item < nitems) quantize(item, v[ii]);
        }
        for (int item = warp + kItems * kMW; item < nitems; item += kMW) {
            float o[4];
            rotate(item, o);
            quantize(item, o);
        }
        consumer_sync();

        // (3) decode + integer tensor-core products.  Every warp waits on and releases every
        //     stage (the ring runs across units), computing only when it has a chunk in it.
        const bool b_live = lane < 8 * rows;
        int D[8][4];
#pragma unroll
        for (int c = 0; c < 8; ++c) D[c][0] = D[c][1] = D[c][2] = D[c][3] = 0;
        // stages in which this warp has a chunk (cl = warp + 8*jl < nch) first, as in k_gemv_mul1 ...
        const int mine = nch > warp ? (nch - warp + kMW - 1) / kMW : 0;
        int jl = 0;
        for (; jl < mine; ++jl, ++j) {
            const int cl = warp + jl * kMW;
            const int s = j % kMStages;
            uint4 bq = make_uint4(0, 0, 0, 0);
            if (b_live) bq = *reinterpret_cast<const uint4 *>(xq + size_t(cl) * 128 * rows + lane * 16);
            if (!mbar_wait_sleep(&full[s], (j / kMStages) & 1)) {
                atomicOr(&g_seq_status, kStatusWaitTimeout);
                atomicOr(a.abort, 1u);
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
        // ... then the unit's last stage if it holds no chunk of this warp: wait for it and release it,
        //     so that every stage's empty barrier sees all eight consumer warps (the ring runs on)
        for (; jl < nstage; ++jl, ++j) {
            const int s = j % kMStages;
            if (!mbar_wait_sleep(&full[s], (j / kMStages) & 1)) {
                atomicOr(&g_seq_status, kStatusWaitTimeout);
                atomicOr(a.abort, 1u);
                break;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // (4) integer sums meet in shared memory; the CTA's fp32 partial goes to `part`
        {
            const int g = lane >> 2, t = lane & 3;
            if (t < rows) {
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    int * a0 = acc + (t * 128 + c * 16 + g) * 2;
                    atomicAdd(a0, D[c][0]);
                    atomicAdd(a0 + 1, D[c][1]);
                    atomicAdd(a0 + 16, D[c][2]);
                    atomicAdd(a0 + 17, D[c][3]);
                }
            }
        }
        consumer_sync();
        const int cu = P.cu_base + nb;
        float * myslot = a.slots + P.slot_base + (size_t(nb) * P.splits + split) * rows * 128;
        for (int e = threadIdx.x; e < rows * 128; e += kMW * 32) {
            const int r = e >> 7;
            const float sq = fmaf(float(acc[2 * e]), 128.f, float(acc[2 * e + 1]));
            const float val = scale_s[r] * fmaf(kCodeA, sq, kCodeC * float(xsum_s[r]));
            if (P.splits > 1) __stcg(myslot + e, val); else part[e] = val;
        }
        bool last = true;
        if (P.splits > 1) {
            __threadfence();  // the partial is visible before the ticket
            consumer_sync();
            if (threadIdx.x == 0) *flag_s = atomicAdd(&a.tickets[cu], 1u) == unsigned(P.splits - 1);
            consumer_sync();
            last = *flag_s != 0;
            if (last) __threadfence();  // every other split's partial is visible
        }
        if (!last) continue;
        // (5) the column block's last split: sum the partials in split order, H128, sv, store y
        for (int r = warp; r < rows; r += kMW) {
            float o[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int e = r * 128 + lane * 4 + q;
                if (P.splits == 1) {
                    o[q] = part[e];
                } else {
                    // all slots in flight at once (one L2 round trip), then summed in split order
                    const float * base = a.slots + P.slot_base + size_t(nb) * P.splits * rows * 128 + e;
                    float pv[kSeqMaxSplits];
#pragma unroll
                    for (int s2 = 0; s2 < kSeqMaxSplits; ++s2)
                        pv[s2] = s2 < P.splits ? __ldcg(base + size_t(s2) * rows * 128) : 0.f;
                    float acc_v = pv[0];
#pragma unroll
                    for (int s2 = 1; s2 < kSeqMaxSplits; ++s2)
                        if (s2 < P.splits) acc_v = __fadd_rn(acc_v, pv[s2]);
                    o[q] = acc_v;
                }
            }
            h128_warp4(o);
            const uint2 sraw = *reinterpret_cast<const uint2 *>(P.sv + nb * 128 + lane * 4);
            const __half2 s01 = bits_half2(sraw.x), s23 = bits_half2(sraw.y);
            float4 out;
            out.x = __fmul_rn(o[0], __low2float(s01));
            out.y = __fmul_rn(o[1], __high2float(s01));
            out.z = __fmul_rn(o[2], __low2float(s23));
            out.w = __fmul_rn(o[3], __high2float(s23));
            *reinterpret_cast<float4 *>(P.y + size_t(r) * P.y_stride + nb * 128 + lane * 4) = out;
        }
        __threadfence();  // y is visible before the group counter moves
        consumer_sync();
        if (threadIdx.x == 0) atomicAdd(&a.group_done[P.group], 1u);
    }
}

// ---------------------------------------------------------------------------

namespace {

void * seq_kernel_for(unsigned bits) {
    switch (bits) {
        case 2: return reinterpret_cast<void *>(k_gemv_persist<2>);
        case 3: return reinterpret_cast<void *>(k_gemv_persist<3>);
        case 4: return reinterpret_cast<void *>(k_gemv_persist<4>);
        case 5: return reinterpret_cast<void *>(k_gemv_persist<5>);
        case 6: return reinterpret_cast<void *>(k_gemv_persist<6>);
        case 7: return reinterpret_cast<void *>(k_gemv_persist<7>);
        case 8: return reinterpret_cast<void *>(k_gemv_persist<8>);
        default: return nullptr;
    }
}

constexpr size_t kSeqMaxSmem = 200 * 1024;

}  // namespace

size_t seq_smem_bytes(unsigned bits, int cps_max) { return seq_layout(int(bits), cps_max).bytes; }

// CTAs of the persistent kernel that fit the device at once with this shared memory (0 if none).
int seq_resident_ctas(int device, unsigned bits, size_t smem, int sms) {
    static std::mutex mu;
    std::lock_guard<std::mutex> g(mu);
    const void * k = seq_kernel_for(bits);
    if (!k || smem > kSeqMaxSmem) return 0;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSeqMaxSmem)) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kMThreads, smem) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    (void)device;
    if (per_sm > 2) per_sm = 2;
    return per_sm * sms;
}

cudaError_t launch_gemv_persist(const SeqArgs & a, unsigned bits, int grid, size_t smem, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(grid), 1, 1);
    cfg.blockDim = dim3(kMThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeCooperative;  // every CTA resident: the group waits rely on it
    attr.val.cooperative = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    void * args[] = {const_cast<SeqArgs *>(&a)};
    return cudaLaunchKernelExC(&cfg, seq_kernel_for(bits), args);
}

cudaError_t seq_read_status(unsigned * out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_seq_status, sizeof(unsigned));
    if (e == cudaSuccess && clear && *out) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(g_seq_status, &zero, sizeof(unsigned));
    }
    return e;
}

}  // namespace exl3cu
