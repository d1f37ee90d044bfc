// EXL3 GEMM on the 5th-generation tensor cores (tcgen05, accumulators in
// TMEM) for batches of rows -- the ragged continuous-batching path.
//
// y = sv * H128( sum_kb H128(x * su)_kb . W_inner(kb) ) per 128-column block,
// as ggml_exl3_mul_mat computes it (src/exl3-ggml.cpp:51-92).  Per MMA:
//   A = rotated activations, M = 128 tokens x K = 16, fp16, K-major;
//   B = W_inner^T, N = 128 output columns (one column block) x K = 16, fp16;
//   D = fp32 in TMEM, 128 lanes (tokens) x 128 columns.
// The decoded weights are the reference's fp16 values bit for bit (the same
// decode_chunk the codec kernels use); the products accumulate in fp32.
//
// Shared-memory operands use the canonical no-swizzle K-major layout: 8x16-byte
// core matrices, LBO = stride between the two 8-element K halves, SBO = stride
// between 8-row groups.  A decode lane's four mma-fragment registers of a
// 16x16 tile fall on exactly four core matrices, one 32-bit store each, with
// the 32 lanes of a warp covering a core matrix's 128 contiguous bytes.
//
// A CTA owns one column block, T <= 4 token tiles of 128 and one K range: it
// decodes each 16-row chunk of W once and issues T MMAs on it, one per token
// tile, into T TMEM accumulators (T*128 columns).  Warp roles (320 threads):
// warp 0 owns TMEM and issues the activation bulk copies; warp 1's elected
// thread issues tcgen05.mma and the commits that recycle the rings; warps
// 2-9 stream the CTA's trellis chunks from HBM and decode them into a ring of
// B tiles, then run the epilogue.  The K split runs across a thread-block
// cluster: every rank parks its fp32 partial tile in shared memory and rank r
// reduces rows [r*128/S, (r+1)*128/S) over all ranks in rank order through
// distributed shared memory, applies H128 and sv and stores y.  Every mbarrier
// wait is bounded.
#include "exl3cu_async.cuh"
#include "exl3cu_internal.h"

#include <cooperative_groups.h>

#include <mutex>

namespace cg = cooperative_groups;

namespace exl3cu {

static __device__ unsigned g_gemm_status;

constexpr int kDecodeWarps = 8;
constexpr int kFirstDecodeWarp = 3;  // warps 0-2: weight copies + TMEM, MMA issue, activation copies
constexpr int kTThreads = 32 * (kFirstDecodeWarp + kDecodeWarps);
constexpr int kBGroups = 3;          // decoded W groups of 4 chunks (4 KB B tiles) in the ring
constexpr int kBTileBytes = 4096;
constexpr int kBRingBytes = kBGroups * 4 * kBTileBytes;
constexpr int kWRingBytes = 32768;   // trellis stages of 4 chunks in flight (>= 4 stages at 8 bits)
constexpr int kMaxWStages = 16;
constexpr int kMaxXStages = 3;       // activation stages of 64 K (4 chunks): 3 for T <= 2, else 2
constexpr int kXTileBytes = 16384;   // 64 K x 128 tokens fp16: one token tile of a stage
constexpr int kMaxTiles = 4;         // token tiles per CTA (T*128 TMEM columns <= 512)
constexpr int kPartStride = 132;     // floats per row of the parked partial tile
constexpr size_t kBarBytes = 512;
// Shared memory is padded to at least this, so that one CTA fits an SM: two
// CTAs could otherwise ask for more than the SM's 512 TMEM columns together,
// and tcgen05.alloc would wait for columns that a cluster peer never frees.
constexpr size_t kMinSmem = 120 * 1024;
// kind::f16: D fp32 (bit 4), A/B fp16, both K-major, N = 128 (>>3 at bit 17), M = 128 (>>4 at bit 24)
constexpr uint32_t kIdescF16 = (1u << 4) | (16u << 17) | (8u << 24);

struct GemmArgs {
    const uint32_t * lsc;  // device-layout weights of the handle's column blocks
    const __half * sv;     // [nblocks * 128]
    const __half * xt;     // tiled rotated activations, see k_tile_x
    float * y;             // [M][y_stride]
    long long y_stride;
    int M;                 // valid rows
    int T;                 // token tiles per CTA
    int tgroups;           // groups of T token tiles
    int nchunks;           // k / 16
    int nblocks;
    int cps;               // chunks per cluster rank, a multiple of 4
    int splits;
    int tmem_cols;
    int xstages;           // activation stages in the ring (2 or 3)
};

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= uint64_t((saddr >> 4) & 0x3fffu);
    d |= uint64_t((lbo >> 4) & 0x3fffu) << 16;
    d |= uint64_t((sbo >> 4) & 0x3fffu) << 32;
    d |= uint64_t(1) << 46;  // descriptor version for sm_100
    return d;                // base offset 0, relative LBO, layout type 0 = no swizzle
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(kIdescF16), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive fp32 TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------------------
// Activation prologue: xh = H128(x * su) per (row, 128-group), rounded to fp16
// (src/exl3-ggml.cpp:60-70 forms the same rotated row), written in the A
// operand's tiled order: element (token, kk) of token tile `tile` at half
//   tile*128*k + (kk/16)*2048 + ((token%128)/8)*128 + ((kk/8)%2)*64 + (token%8)*8 + kk%8,
// i.e. per 16 columns of K a 4 KB block of 8x16-byte core matrices, row group
// r and K half h at r*256 + h*128 bytes (the B tile's arrangement, which the
// tensor cores read at full rate), so a group of 4 chunks of one token tile is
// 16 contiguous KB.  Rows at or beyond M are zero.  One warp per (row, group).
__global__ void k_tile_x(const void * __restrict__ x, int x_f16, long long x_stride, const __half * __restrict__ su,
                         int M, int k, int ntiles, __half * __restrict__ xt) {
    pdl_trigger();
    pdl_wait_primary();  // x comes from the previous kernel; xt may still be read by the previous GEMM
    const int warp = int((blockIdx.x * size_t(blockDim.x) + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    const int groups = k / 128;
    if (warp >= ntiles * 128 * groups) return;  // whole warps only: the count is a multiple of 8
    const int tok = warp / groups, gi = warp % groups;
    const int kcol = gi * 128 + lane * 4;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (tok < M) {
        if (x_f16) {
            const uint2 raw =
                *reinterpret_cast<const uint2 *>(static_cast<const __half *>(x) + size_t(tok) * x_stride + kcol);
            const __half2 lo = bits_half2(raw.x), hi = bits_half2(raw.y);
            v[0] = __low2float(lo); v[1] = __high2float(lo); v[2] = __low2float(hi); v[3] = __high2float(hi);
        } else {
            const float4 f =
                *reinterpret_cast<const float4 *>(static_cast<const float *>(x) + size_t(tok) * x_stride + kcol);
            v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
        }
        const uint2 sraw = *reinterpret_cast<const uint2 *>(su + kcol);
        const __half2 s01 = bits_half2(sraw.x), s23 = bits_half2(sraw.y);
        v[0] = __fmul_rn(v[0], __low2float(s01));
        v[1] = __fmul_rn(v[1], __high2float(s01));
        v[2] = __fmul_rn(v[2], __low2float(s23));
        v[3] = __fmul_rn(v[3], __high2float(s23));
    }
    h128_warp4(v);
    const int tile = tok >> 7, tr = tok & 127;
    const size_t off = size_t(tile) * 128 * k + size_t(kcol >> 4) * 2048 + (tr >> 3) * 128 + ((kcol >> 3) & 1) * 64 +
                       (tr & 7) * 8 + (kcol & 7);
    const __half2 o01 = __floats2half2_rn(v[0], v[1]);
    const __half2 o23 = __floats2half2_rn(v[2], v[3]);
    *reinterpret_cast<uint2 *>(xt + off) = make_uint2(half2_bits(o01), half2_bits(o23));
}

// ---------------------------------------------------------------------------

template <int BITS, unsigned CB>
__global__ void __launch_bounds__(kTThreads, 1) k_gemm_tc(const GemmArgs a) {
    extern __shared__ __align__(1024) unsigned char smem[];
    constexpr int SEGW = 2 * BITS;                   // words of one lane's segment of a chunk
    constexpr int CHUNKB = 256 * BITS;               // bytes of one chunk
    constexpr int WSTAGEB = 4 * CHUNKB;              // bytes of one weight stage (a group of 4 chunks)
    constexpr int WST = kWRingBytes / WSTAGEB > kMaxWStages ? kMaxWStages : kWRingBytes / WSTAGEB;
    pdl_trigger();

    cg::cluster_group cluster = cg::this_cluster();
    const int S = a.splits;
    const int T = a.T;
    const int XST = a.xstages;
    const int split = int(cluster.block_rank());
    const int unit = blockIdx.x / S;
    const int nb = unit / a.tgroups;
    const int tg = unit - nb * a.tgroups;
    const int c0 = min(split * a.cps, a.nchunks);
    const int c1 = min(c0 + a.cps, a.nchunks);
    const int nch = c1 - c0;  // a multiple of 4: k and cps are
    const int ngr = nch / 4;  // groups of 4 chunks (64 rows of K): the unit of every ring
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int xstage_bytes = T * kXTileBytes;

    unsigned char * bring = smem;                 // kBGroups x 4 decoded B tiles of 4 KB
    unsigned char * wring = bring + kBRingBytes;  // WST x 4 chunks of trellis
    unsigned char * xring = wring + kWRingBytes;  // XST x T x 16 KB activations
    uint64_t * bars = reinterpret_cast<uint64_t *>(xring + XST * xstage_bytes);
    uint64_t * fullB = bars;
    uint64_t * emptyB = fullB + kBGroups;
    uint64_t * fullW = emptyB + kBGroups;
    uint64_t * emptyW = fullW + kMaxWStages;
    uint64_t * fullX = emptyW + kMaxWStages;
    uint64_t * emptyX = fullX + kMaxXStages;
    uint64_t * done = emptyX + kMaxXStages;
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    float * part = reinterpret_cast<float *>(smem);  // epilogue reuse of the rings: [128][kPartStride]

    if (threadIdx.x == 0) {
        for (int i = 0; i < kBGroups; ++i) {
            mbar_init(&fullB[i], 4);   // the four decode warps of the group's chunks
            mbar_init(&emptyB[i], 1);  // the MMA commit
        }
        for (int i = 0; i < WST; ++i) {
            mbar_init(&fullW[i], 1);
            mbar_init(&emptyW[i], 4);
        }
        for (int i = 0; i < XST; ++i) {
            mbar_init(&fullX[i], 1);
            mbar_init(&emptyX[i], 1);
        }
        mbar_init(done, 1);
        mbar_init_fence();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_addr(tmem_slot)), "r"(uint32_t(a.tmem_cols)) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- weight groups: static data, streamed from the first cycle (before the PDL wait) ----
        if (lane == 0) {
            const unsigned char * src =
                reinterpret_cast<const unsigned char *>(a.lsc) + (size_t(nb) * a.nchunks + c0) * CHUNKB;
            for (int g = 0; g < ngr; ++g) {
                const int slot = g % WST;
                if (g >= WST && !mbar_wait_sleep(&emptyW[slot], ((g / WST) - 1) & 1)) {
                    atomicOr(&g_gemm_status, kStatusWaitTimeout);
                    break;
                }
                mbar_arrive_expect_tx(&fullW[slot], uint32_t(WSTAGEB));
                bulk_g2s(wring + slot * WSTAGEB, src + size_t(g) * WSTAGEB, uint32_t(WSTAGEB), &fullW[slot]);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issue: one thread, 4*T MMAs per group of 4 chunks ----
        if (lane == 0) {
            // start-address fields of the first B tile / activation tile; later tiles are constant offsets
            const uint64_t bdesc0 = umma_desc(smem_addr(bring), 128, 256);
            const uint64_t adesc0 = umma_desc(smem_addr(xring), 128, 256);
            for (int g = 0; g < ngr; ++g) {
                const int bs = g % kBGroups, xs = g % XST;
                if (!mbar_wait_sleep(&fullB[bs], (g / kBGroups) & 1) || !mbar_wait_sleep(&fullX[xs], (g / XST) & 1)) {
                    atomicOr(&g_gemm_status, kStatusWaitTimeout);
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint64_t bdesc = bdesc0 + uint64_t(((bs * 4 + c) * kBTileBytes) >> 4);
                    for (int t = 0; t < T; ++t) {
                        const uint64_t adesc = adesc0 + uint64_t(((xs * T + t) * kXTileBytes + c * 4096) >> 4);
                        umma_f16(tmem + uint32_t(t * 128), adesc, bdesc, (g | c) != 0 ? 1u : 0u);
                    }
                }
                umma_commit(&emptyB[bs]);
                umma_commit(&emptyX[xs]);
            }
            if (ngr > 0)
                umma_commit(done);  // arrives once every issued MMA has completed
            else
                mbar_arrive(done);
        }
        __syncwarp();
    } else if (warp == 2) {
        // ---- activation groups (written by the prologue kernel: wait for it first) ----
        if (lane == 0) {
            pdl_wait_primary();
            const size_t tile_halves = size_t(a.nchunks) * 2048;  // one token tile, all of K
            const __half * src = a.xt + size_t(tg) * T * tile_halves + size_t(c0) * 2048;
            for (int g = 0; g < ngr; ++g) {
                const int slot = g % XST;
                if (g >= XST && !mbar_wait_sleep(&emptyX[slot], ((g / XST) - 1) & 1)) {
                    atomicOr(&g_gemm_status, kStatusWaitTimeout);
                    break;
                }
                mbar_arrive_expect_tx(&fullX[slot], uint32_t(xstage_bytes));
                for (int t = 0; t < T; ++t)
                    bulk_g2s(xring + (slot * T + t) * kXTileBytes, src + size_t(t) * tile_halves + size_t(g) * 4 * 2048,
                             kXTileBytes, &fullX[slot]);
            }
        }
        __syncwarp();
    } else {
        // ---- decode warps: chunk j of the CTA's range goes to warp j % 8 ----
        const int dw = warp - kFirstDecodeWarp;
        for (int j = dw; j < nch; j += kDecodeWarps) {
            const int g = j >> 2, ws = g % WST;
            if (!mbar_wait_sleep(&fullW[ws], (g / WST) & 1)) {
                atomicOr(&g_gemm_status, kStatusWaitTimeout);
                break;
            }
            uint32_t w[SEGW];
            const uint32_t * seg = reinterpret_cast<const uint32_t *>(wring + ws * WSTAGEB + (j & 3) * CHUNKB) +
                                   lane * SEGW;
            if constexpr ((BITS & 1) == 0) {
#pragma unroll
                for (int i = 0; i < SEGW; i += 4) {
                    const uint4 v = *reinterpret_cast<const uint4 *>(seg + i);
                    w[i] = v.x; w[i + 1] = v.y; w[i + 2] = v.z; w[i + 3] = v.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < SEGW; i += 2) {
                    const uint2 v = *reinterpret_cast<const uint2 *>(seg + i);
                    w[i] = v.x; w[i + 1] = v.y;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&emptyW[ws]);
            uint32_t frag[8][4];
            decode_chunk<BITS, CB>(w, frag);
            const int bs = g % kBGroups;
            if (g >= kBGroups && !mbar_wait_sleep(&emptyB[bs], ((g / kBGroups) - 1) & 1)) {
                atomicOr(&g_gemm_status, kStatusWaitTimeout);
                break;
            }
            uint32_t * bt = reinterpret_cast<uint32_t *>(bring + (bs * 4 + (j & 3)) * kBTileBytes);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                // core matrix (column group 2c or 2c+1, K half 0 or 1) at group*256 + half*128 bytes;
                // lane (g = lane/4, t = lane%4) holds columns 16c+g / 16c+8+g, K pairs 2t / 2t+8 of tile c
                bt[(c * 512 + 0) / 4 + lane] = frag[c][0];    // column 16c+g,   K 2t..2t+1
                bt[(c * 512 + 256) / 4 + lane] = frag[c][1];  // column 16c+8+g, K 2t..2t+1
                bt[(c * 512 + 128) / 4 + lane] = frag[c][2];  // column 16c+g,   K 2t+8..2t+9
                bt[(c * 512 + 384) / 4 + lane] = frag[c][3];  // column 16c+8+g, K 2t+8..2t+9
            }
            fence_proxy_async();  // the generic-proxy stores become visible to the tensor cores
            __syncwarp();
            if (lane == 0) mbar_arrive(&fullB[bs]);
        }
    }

    // ---- epilogue: per token tile, park the partial, then reduce a row slice over the cluster ----
    const bool epi = warp >= kFirstDecodeWarp;
    if (epi && !mbar_wait_sleep(done, 0)) atomicOr(&g_gemm_status, kStatusWaitTimeout);
    tc_fence_after();
    __syncthreads();  // every MMA has completed: the rings are free for the partial tile
    const int rows_per_rank = 128 / S;
    const int ew = warp - kFirstDecodeWarp;  // epilogue warp 0..7
    for (int t = 0; t < T; ++t) {
        if (epi) {
            const int q = warp & 3;  // TMEM lane quarter this warp may read
            const int h = ew >> 2;   // column half
            const int row = q * 32 + lane;
            float * dst = part + row * kPartStride + h * 64;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float v[32];
                if (nch > 0) {
                    tmem_ld32(tmem + (uint32_t(q * 32) << 16) + uint32_t(t * 128 + h * 64 + c * 32), v);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = 0.f;
                }
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                    *reinterpret_cast<float4 *>(dst + c * 32 + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            }
        }
        cluster.sync();
        if (epi) {
            const uint2 sraw = *reinterpret_cast<const uint2 *>(a.sv + nb * 128 + lane * 4);
            const __half2 s01 = bits_half2(sraw.x), s23 = bits_half2(sraw.y);
            for (int r = split * rows_per_rank + ew; r < (split + 1) * rows_per_rank; r += kDecodeWarps) {
                float v[4] = {0.f, 0.f, 0.f, 0.f};
                for (int s = 0; s < S; ++s) {
                    const float * rp = cluster.map_shared_rank(part, s) + r * kPartStride + lane * 4;
                    const float4 p = *reinterpret_cast<const float4 *>(rp);
                    v[0] = __fadd_rn(v[0], p.x);
                    v[1] = __fadd_rn(v[1], p.y);
                    v[2] = __fadd_rn(v[2], p.z);
                    v[3] = __fadd_rn(v[3], p.w);
                }
                h128_warp4(v);
                const int token = (tg * T + t) * 128 + r;
                if (token < a.M) {
                    float4 o;
                    o.x = __fmul_rn(v[0], __low2float(s01));
                    o.y = __fmul_rn(v[1], __high2float(s01));
                    o.z = __fmul_rn(v[2], __low2float(s23));
                    o.w = __fmul_rn(v[3], __high2float(s23));
                    *reinterpret_cast<float4 *>(a.y + size_t(token) * a.y_stride + nb * 128 + lane * 4) = o;
                }
            }
        }
        cluster.sync();  // the partials stay until every rank has read them
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(uint32_t(a.tmem_cols))
                     : "memory");
    }
}

// ---------------------------------------------------------------------------

namespace {

template <int BITS>
void * gemm_kernel_cb(unsigned cb) {
    switch (cb) {
        case CB_3INST: return reinterpret_cast<void *>(k_gemm_tc<BITS, CB_3INST>);
        case CB_MCG: return reinterpret_cast<void *>(k_gemm_tc<BITS, CB_MCG>);
        case CB_MUL1: return reinterpret_cast<void *>(k_gemm_tc<BITS, CB_MUL1>);
        default: return nullptr;
    }
}

void * gemm_kernel_for(unsigned bits, unsigned cb) {
    switch (bits) {
        case 1: return gemm_kernel_cb<1>(cb);
        case 2: return gemm_kernel_cb<2>(cb);
        case 3: return gemm_kernel_cb<3>(cb);
        case 4: return gemm_kernel_cb<4>(cb);
        case 5: return gemm_kernel_cb<5>(cb);
        case 6: return gemm_kernel_cb<6>(cb);
        case 7: return gemm_kernel_cb<7>(cb);
        case 8: return gemm_kernel_cb<8>(cb);
        default: return nullptr;
    }
}

int xstages_for(int T) { return T <= 2 ? 3 : 2; }

size_t gemm_smem(int T) {
    const size_t s = size_t(kBRingBytes) + kWRingBytes + size_t(xstages_for(T)) * T * kXTileBytes + kBarBytes;
    return s < kMinSmem ? kMinSmem : s;
}

constexpr size_t kGemmMaxSmem = size_t(kBRingBytes) + kWRingBytes + size_t(2) * kMaxTiles * kXTileBytes + kBarBytes;
static_assert(kGemmMaxSmem <= 227 * 1024, "GEMM shared memory above the per-CTA limit");
static_assert(size_t(kBRingBytes) + kWRingBytes + size_t(3) * 2 * kXTileBytes + kBarBytes <= kGemmMaxSmem,
              "T = 2 with three activation stages must fit the same limit");
static_assert(size_t(128) * kPartStride * 4 <= size_t(kBRingBytes) + kWRingBytes + 2 * kXTileBytes,
              "the partial tile must fit in the rings of the smallest plan (T = 1, two activation stages)");
static_assert(2 * kMinSmem > 228 * 1024, "the padding must keep a second CTA off the SM");
static_assert((2 * kBGroups + 2 * kMaxWStages + 2 * kMaxXStages + 1) * 8 + 4 <= kBarBytes, "barrier area");

bool gemm_prepare(int device, unsigned bits, unsigned cb) {
    static std::mutex mu;
    static bool done[64][9][3] = {};
    if (device < 0 || device >= 64 || bits < 1 || bits > 8 || cb > 2) return false;
    std::lock_guard<std::mutex> g(mu);
    if (done[device][bits][cb]) return true;
    const void * k = gemm_kernel_for(bits, cb);
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kGemmMaxSmem)) != cudaSuccess)
        return false;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) return false;
    done[device][bits][cb] = true;
    return true;
}

}  // namespace

GemmPlan plan_gemm(int sms, size_t k, size_t nblocks, int rows, int tiles, int splits) {
    GemmPlan p{};
    const int ntiles = (rows + 127) / 128;
    const int tmax = tiles > 0 ? (tiles < kMaxTiles ? tiles : kMaxTiles) : kMaxTiles;
    p.tgroups = (ntiles + tmax - 1) / tmax;
    p.T = (ntiles + p.tgroups - 1) / p.tgroups;  // balanced: at most tgroups-1 padded tiles
    p.tmem_cols = p.T == 1 ? 128 : p.T == 2 ? 256 : 512;
    const int nchunks = int(k / 16);
    const long long units = (long long)nblocks * p.tgroups;
    // K split over a cluster so that units x S fills the device once; at least 8 chunks per rank
    int S = 1;
    while (S < 8 && units * (S * 2) <= sms && nchunks / (S * 2) >= 8) S *= 2;
    if (splits > 0) S = splits < 16 ? splits : 16;
    p.splits = S;
    const int cps = (nchunks + S - 1) / S;
    p.cps = (cps + 3) / 4 * 4;
    p.smem = gemm_smem(p.T);
    p.xt_bytes = size_t(p.tgroups) * p.T * 128 * k * sizeof(__half);
    return p;
}

// y[rows][n_local] for a handle's weights: tile the activations into `xt`
// (GemmPlan::xt_bytes), then one cluster launch over (column block, token-tile
// group) units x K splits.
cudaError_t launch_gemm_tc(const GemmPlan & p, const uint32_t * lsc, const __half * su, const __half * sv, size_t k,
                           size_t nblocks, unsigned bits, unsigned cb, int device, const void * x, int x_f16,
                           long long x_stride, int rows, float * y, long long y_stride, __half * xt, bool pdl,
                           cudaStream_t st) {
    if (!gemm_prepare(device, bits, cb)) return cudaErrorInvalidValue;
    const int ntiles_pad = p.tgroups * p.T;
    const long long warps = (long long)ntiles_pad * 128 * (long long)(k / 128);
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(unsigned((warps * 32 + 255) / 256), 1, 1);
        cfg.blockDim = dim3(256, 1, 1);
        cfg.stream = st;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr.val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = pdl ? 1 : 0;
        cudaError_t e = cudaLaunchKernelEx(&cfg, k_tile_x, x, x_f16, x_stride, su, rows, int(k), ntiles_pad, xt);
        if (e != cudaSuccess) return e;
    }
    GemmArgs a;
    a.lsc = lsc;
    a.sv = sv;
    a.xt = xt;
    a.y = y;
    a.y_stride = y_stride;
    a.M = rows;
    a.T = p.T;
    a.tgroups = p.tgroups;
    a.nchunks = int(k / 16);
    a.nblocks = int(nblocks);
    a.cps = p.cps;
    a.splits = p.splits;
    a.tmem_cols = p.tmem_cols;
    a.xstages = xstages_for(p.T);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(nblocks * p.tgroups * p.splits), 1, 1);
    cfg.blockDim = dim3(kTThreads, 1, 1);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = unsigned(p.splits);
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = pdl ? 2 : 1;
    void * args[] = {&a};
    return cudaLaunchKernelExC(&cfg, gemm_kernel_for(bits, cb), args);
}

cudaError_t gemm_read_status(unsigned * out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_gemm_status, sizeof(unsigned));
    if (e == cudaSuccess && clear && *out) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(unsigned));
    }
    return e;
}

}  // namespace exl3cu
