// EXL3 GEMM on the 5th-generation tensor cores (tcgen05, accumulators in
// TMEM) for batches of rows -- the ragged continuous-batching path.
//
// y = sv * H128( sum_kb H128(x * su)_kb . W_inner(kb) ) per 128-column block,
// as ggml_exl3_mul_mat computes it (src/exl3-ggml.cpp:51-92), with the
// reference's decoded fp16 weights bit for bit and fp32 accumulation.
//
// Swap-AB form, per MMA (kind::f16, M = 128, N = NTOK tokens, K = 16):
//   A = W_inner^T of one column block (128 output columns x 16 rows of K), in
//       TENSOR MEMORY, written there by the decode warps with tcgen05.st;
//   B = the rotated activations (NTOK tokens x 16), fp16, K-major in shared
//       memory, bulk-copied from a buffer the prologue kernel writes;
//   D = fp32 in TMEM: 128 lanes (output columns) x NTOK columns (tokens).
// The decoded weights never touch shared memory, the MMA reads only the
// activation tile, and its cost scales with the batch's tokens (32..256 per
// CTA), not with a padded 128-token tile.
//
// A in TMEM: lane m = output column, 32-bit column j = a pair of K values.  A
// decode lane (g, t) holds, per 16x16 tile, K pairs {2t, 2t+1} and {2t+8, 2t+9}
// of columns g and g+8 (the mma A-fragment layout of decode_tile_pair), and
// tcgen05.st.16x256b puts thread (g, t)'s four registers at (lane g | g+8,
// column 2t | 2t+1): column 2t holds K (2t, 2t+1), column 2t+1 holds K
// (2t+8, 2t+9).  The activations are stored with the same permutation of K
// inside every 16 (kperm16), so each dot product is an exact re-ordering of
// the unpermuted one.  A warp may only address its own quarter of the TMEM
// lanes, so a chunk's 8 tiles are decoded by a warpgroup: warp quarter q
// decodes tiles 2q and 2q+1 (output columns 32q..32q+31).
//
// Warps (512 threads): 0-11 = three decode warpgroups (group g of 8 chunks
// goes to warpgroup g % 3), later the epilogue; 12 = TMEM owner + trellis bulk
// copies; 13 = MMA issue (one thread); 14 = activation bulk copies.  The K
// split runs across a thread-block cluster: every rank parks its fp32 partial
// [NTOK][128] in shared memory and rank r reduces tokens [r*NTOK/S,
// (r+1)*NTOK/S) over all ranks in rank order through distributed shared
// memory, applies H128 and sv and stores y.  Every mbarrier wait is bounded.
#include "exl3cu_async.cuh"
#include "exl3cu_internal.h"

#include <cooperative_groups.h>

#include <mutex>

namespace cg = cooperative_groups;

namespace exl3cu {

static __device__ unsigned g_gemm_status;

constexpr int kMaxWStages = 16;
constexpr size_t kBarBytes = 512;
// Shared memory is padded to at least this, so that one CTA fits an SM: two
// CTAs could otherwise ask for more than the SM's 512 TMEM columns together,
// and tcgen05.alloc would wait for columns that a cluster peer never frees.
constexpr size_t kMinSmem = 120 * 1024;
static_assert(2 * kMinSmem > 228 * 1024, "the padding must keep a second CTA off the SM");

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= uint64_t((saddr >> 4) & 0x3fffu);
    d |= uint64_t((lbo >> 4) & 0x3fffu) << 16;
    d |= uint64_t((sbo >> 4) & 0x3fffu) << 32;
    d |= uint64_t(1) << 46;  // descriptor version for sm_100
    return d;                // base offset 0, relative LBO, layout type 0 = no swizzle
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

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

constexpr int kDecodeGroups = 3;
constexpr int kGemmThreads = 512;
constexpr int kGroupChunks = 8;    // chunks (16 rows of K each) per pipeline group

// Trellis ring of the swap-AB kernel: `wstages` groups, chosen per launch as
// deep as shared memory allows next to the activation slots (up to ~96 KB, so
// that an SM reading weights held by the other die still keeps enough bytes in
// flight).  The depth is a multiple of the number of decode warpgroups, so that
// each slot is only ever consumed by one warpgroup (group g goes to warpgroup
// g % 3 and to slot g % wstages): a parity wait is only sound when the waiter
// itself saw the barrier's previous phase complete, and bulk copies into
// different slots may complete in any order.
constexpr int kSlots = 3;          // groups in flight: TMEM A (64 columns each) + activations
constexpr int kMaxTok = 256;       // tokens per CTA (the MMA's N)
constexpr uint32_t kTmemCols = 512;
constexpr int kACol0 = 256;        // first TMEM column of the A ring (D uses 0..NTOK-1)

// Position inside a 16-block of K at which the A operand in TMEM holds k.
__host__ __device__ constexpr int kperm16(int k) { return 4 * ((k & 7) >> 1) + 2 * (k >> 3) + (k & 1); }

struct GemmArgs {
    PeerOut peer;       // PEER builds: y goes to every rank's buffer as (epoch, value) words
    const uint32_t * lsc;
    const __half * sv;
    const __half * xt;  // [tgroups][k/16][NTOK/8][2][8][8] fp16, K permuted by kperm16
    float * y;
    long long y_stride;
    int M;                 // rows (capacity when m_dev is set)
    const int32_t * m_dev;  // optional: the live row count, min'd with M (ragged batches)
    int m_base;             // rows of the batch before this launch's first row (m_dev counts from 0)
    int ntok;           // tokens per CTA, multiple of 32, <= 256
    int tgroups;
    int nchunks;
    int cps;            // multiple of kGroupChunks
    int splits;
    int wstages;        // trellis ring depth in groups, a multiple of 3
};

// xh = H128(x * su) per (row, 128-group) in fp16, laid out as the B operand:
// token group tg = token / ntok, tr = token % ntok, element k of chunk kc at half
//   tg*ntok*k_total + kc*ntok*16 + (tr/8)*128 + (p/8)*64 + (tr%8)*8 + p%8,  p = kperm16(k % 16)
// (8-token x 16-byte core matrices, 8-token groups 256 B apart, K halves 128 B apart).
__global__ void k_tile_x(const void * __restrict__ x, int x_f16, long long x_stride,
                         const __half * __restrict__ su, int M, const int32_t * __restrict__ m_dev, int m_base, int k,
                         int ntok, int rows_pad, __half * __restrict__ xt) {
    pdl_trigger();
    pdl_wait_primary();
    if (m_dev) M = min(M, max(0, *m_dev - m_base));  // written by an earlier kernel: read after the wait
    const int warp = int((blockIdx.x * size_t(blockDim.x) + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    const int groups = k / 128;
    if (warp >= rows_pad * groups) return;  // whole warps: rows_pad is a multiple of 32
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
    const int tg = tok / ntok, tr = tok - tg * ntok;
    // Lane L holds k = 4L..4L+3 of its 16-wide chunk, kk = 4t..4t+3 (t = L & 3), which kperm16 sends
    // to p = {0,1,4,5} (t = 0), {8,9,12,13} (t = 1), {2,3,6,7} (t = 2), {10,11,14,15} (t = 3).  So lanes
    // t and t + 2 together hold one 8-half row (p>>3 = t) of the token's core matrix: the t < 2 lane
    // takes its partner's two half2 and stores the whole row as one 16-byte write.
    const int t = lane & 3;
    const uint32_t h01 = half2_bits(__floats2half2_rn(v[0], v[1]));
    const uint32_t h23 = half2_bits(__floats2half2_rn(v[2], v[3]));
    const uint32_t q01 = __shfl_xor_sync(0xffffffffu, h01, 2);
    const uint32_t q23 = __shfl_xor_sync(0xffffffffu, h23, 2);
    if (t < 2) {
        const size_t base = size_t(tg) * ntok * k + size_t(kcol >> 4) * ntok * 16 + (tr >> 3) * 128 + (tr & 7) * 8;
        *reinterpret_cast<uint4 *>(xt + base + t * 64) = make_uint4(h01, q01, h23, q23);
    }
}

__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}


// This lane's part of tiles 2q and 2q+1 of one chunk (trellis at `chunk`):
// bits [16*BITS*q, 16*BITS*(q+1)) of its 8*BITS-byte segment, realigned to
// start at bit 0, so that one code path serves all four warp quarters (the
// decode loop stays small enough for the instruction caches).  The loads may
// run up to two words past the segment; they stay inside the CTA's shared
// memory (the activation slots follow the trellis ring) and those bits are
// never used.
template <int BITS, unsigned CB>
__device__ __forceinline__ void decode_pair_window(const unsigned char * chunk, int q, uint32_t (&f)[2][4]) {
    constexpr int NW = BITS / 2 + 1;  // words holding 16*BITS bits at a 16-bit offset
    const int lane = threadIdx.x & 31;
    const int bq = BITS * q;           // first bit / 16
    const uint32_t * seg = reinterpret_cast<const uint32_t *>(chunk) + lane * (2 * BITS) + (bq >> 1);
    const uint32_t sh = uint32_t(bq & 1) * 16u;
    uint32_t raw[NW + 1];
#pragma unroll
    for (int i = 0; i <= NW; ++i) raw[i] = seg[i];
    uint32_t w[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) w[i] = __funnelshift_l(raw[i + 1], raw[i], sh);
    decode_tile_pair<BITS, CB, 0>(w, f);
}

// 16 TMEM lanes x 8 columns (one chunk of one tile) from its four A-fragment
// registers: (lane g, col 2t) = K 2t..2t+1 of column g, (g, 2t+1) = K 2t+8..2t+9,
// and the same two for column g+8.
__device__ __forceinline__ void tmem_st_tile(uint32_t taddr, const uint32_t (&f)[4]) {
    asm volatile("tcgen05.st.sync.aligned.16x256b.x1.b32 [%0], {%1, %2, %3, %4};"
                 ::"r"(taddr), "r"(f[0]), "r"(f[2]), "r"(f[1]), "r"(f[3]) : "memory");
}

// One CTA = one column block x NTOK tokens x one K range, in groups of 8 chunks
// (128 rows of K).  A group occupies one of kSlots slots: 64 TMEM columns of
// decoded weights plus NTOK x 128 fp16 activations in shared memory, guarded by
// one full barrier (4 decode-warp arrivals + the activation copy's arrival and
// bytes) and one empty barrier (the MMA commit, waited on by both producers).
// The MMA thread's whole loop is: wait full, 8 MMAs, commit empty.
template <int BITS, unsigned CB, bool PEER>
__global__ void __launch_bounds__(kGemmThreads, 1) k_gemm(const GemmArgs a) {
    extern __shared__ __align__(1024) unsigned char smem[];
    constexpr int CHUNKB = 256 * BITS;
    constexpr int WSTAGEB = kGroupChunks * CHUNKB;  // one group of trellis
    const int WST = a.wstages;
    const int WRING = WST * WSTAGEB;
    pdl_trigger();

    cg::cluster_group cluster = cg::this_cluster();
    const int S = a.splits;
    const int NT = a.ntok;
    const int split = int(cluster.block_rank());
    const int unit = blockIdx.x / S;
    const int nb = unit / a.tgroups;
    const int tg = unit - nb * a.tgroups;
    int M = a.M;
    if (a.m_dev) {
        // Ragged batch: the live row count comes from an earlier kernel, so every
        // thread waits for the preceding grids before reading it; token groups
        // wholly past it exit at once (all ranks of a cluster share the group).
        pdl_wait_primary();
        M = min(M, max(0, *a.m_dev - a.m_base));
        if (tg * NT >= M) return;
    }
    const int c0 = min(split * a.cps, a.nchunks);
    const int c1 = min(c0 + a.cps, a.nchunks);
    const int ngr = (c1 - c0) / kGroupChunks;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int xslot_bytes = NT * 16 * 2 * kGroupChunks;  // NT tokens x 128 K fp16

    unsigned char * wring = smem;           // WST groups of trellis
    unsigned char * xring = wring + WRING;  // kSlots groups of activations
    uint64_t * bars = reinterpret_cast<uint64_t *>(xring + kSlots * xslot_bytes);
    uint64_t * fullW = bars;
    uint64_t * emptyW = fullW + kMaxWStages;
    uint64_t * full = emptyW + kMaxWStages;
    uint64_t * empty = full + kSlots;
    uint64_t * done = empty + kSlots;
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    float * part = reinterpret_cast<float *>(smem);  // epilogue reuse: [NT][128] fp32

    if (threadIdx.x == 0) {
        for (int i = 0; i < WST; ++i) {
            mbar_init(&fullW[i], 1);
            mbar_init(&emptyW[i], 4);  // the four warps of the decoding warpgroup
        }
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(&full[i], 5);   // four decode warps + the activation copy
            mbar_init(&empty[i], 1);  // the MMA commit
        }
        mbar_init(done, 1);
        mbar_init_fence();
    }
    if (warp == 12) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_addr(tmem_slot)), "r"(kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 12) {
        // ---- trellis groups: static data, streamed from the first cycle (before the PDL wait) ----
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
    } else if (warp == 13) {
        // ---- MMA issue (one thread): ring position and phase carried incrementally ----
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | (uint32_t(NT >> 3) << 17) | (8u << 24);
            const uint64_t bdesc0 = umma_desc(smem_addr(xring), 128, 256);
            const uint64_t bchunk = uint64_t((NT * 32) >> 4);
            const uint64_t bslot = uint64_t(xslot_bytes >> 4);
            uint32_t slot = 0, phase = 0, acc = 0;
            uint64_t bd = bdesc0;
            uint32_t acol = tmem + uint32_t(kACol0);
            for (int g = 0; g < ngr; ++g) {
                if (!mbar_wait(&full[slot], phase)) {
                    atomicOr(&g_gemm_status, kStatusWaitTimeout);
                    break;
                }
                tc_fence_after();  // A was written to TMEM by other threads' tcgen05.st
#pragma unroll
                for (int c = 0; c < kGroupChunks; ++c) {
                    umma_ts(tmem, acol + uint32_t(c * 8), bd + uint64_t(c) * bchunk, idesc, c == 0 ? acc : 1u);
                }
                acc = 1u;
                umma_commit(&empty[slot]);
                if (++slot == uint32_t(kSlots)) {
                    slot = 0;
                    phase ^= 1u;
                    bd = bdesc0;
                    acol = tmem + uint32_t(kACol0);
                } else {
                    bd += bslot;
                    acol += uint32_t(kGroupChunks * 8);
                }
            }
            if (ngr > 0)
                umma_commit(done);
            else
                mbar_arrive(done);
        }
        __syncwarp();
    } else if (warp == 14) {
        // ---- activation groups (written by the prologue kernel: wait for it first) ----
        if (lane == 0) {
            pdl_wait_primary();
            const __half * src = a.xt + size_t(tg) * NT * (size_t(a.nchunks) * 16) + size_t(c0) * NT * 16;
            for (int g = 0; g < ngr; ++g) {
                const int slot = g % kSlots;
                if (g >= kSlots && !mbar_wait_sleep(&empty[slot], ((g / kSlots) - 1) & 1)) {
                    atomicOr(&g_gemm_status, kStatusWaitTimeout);
                    break;
                }
                mbar_arrive_expect_tx(&full[slot], uint32_t(xslot_bytes));
                bulk_g2s(xring + slot * xslot_bytes, src + size_t(g) * NT * 16 * kGroupChunks, uint32_t(xslot_bytes),
                         &full[slot]);
            }
        }
        __syncwarp();
    } else if (warp < 12) {
        // ---- decode: warpgroup wg takes groups wg, wg+3, ...; warp quarter q its tiles 2q, 2q+1 ----
        const int wg = warp >> 2, q = warp & 3;
        const uint32_t lane0 = tmem + (uint32_t(q * 32) << 16);       // tile 2q:   lanes 32q..+15
        const uint32_t lane1 = tmem + (uint32_t(q * 32 + 16) << 16);  // tile 2q+1: lanes 32q+16..+31
        for (int g = wg; g < ngr; g += kDecodeGroups) {
            const int ws = g % WST;
            const int slot = g % kSlots;
            if (!mbar_wait_sleep(&fullW[ws], (g / WST) & 1) ||
                (g >= kSlots && !mbar_wait_sleep(&empty[slot], ((g / kSlots) - 1) & 1))) {
                atomicOr(&g_gemm_status, kStatusWaitTimeout);
                break;
            }
            tc_fence_after();  // the MMAs that read this slot have completed
            const unsigned char * wst = wring + ws * WSTAGEB;
            const uint32_t col = uint32_t(kACol0 + slot * kGroupChunks * 8);
#pragma unroll 1
            for (int c = 0; c < kGroupChunks; ++c) {
                uint32_t f[2][4];
                decode_pair_window<BITS, CB>(wst + c * CHUNKB, q, f);
                tmem_st_tile(lane0 + col + uint32_t(c * 8), f[0]);
                tmem_st_tile(lane1 + col + uint32_t(c * 8), f[1]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&emptyW[ws]);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[slot]);
        }
    }

    // ---- epilogue: D[col][token] -> part[token][col]; rank r reduces tokens [r*NT/S, (r+1)*NT/S) ----
    const bool epi = warp < 12;
    if (epi && !mbar_wait_sleep(done, 0)) atomicOr(&g_gemm_status, kStatusWaitTimeout);
    tc_fence_after();
    __syncthreads();  // every MMA has completed: the rings are free for the partial tile
    if (epi) {
        const int wg = warp >> 2, q = warp & 3;
        for (int tc = wg; tc < NT / 32; tc += kDecodeGroups) {
            float v[32];
            if (ngr > 0) {
                tmem_ld32(tmem + (uint32_t(q * 32) << 16) + uint32_t(tc * 32), v);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = 0.f;
            }
#pragma unroll
            for (int r = 0; r < 32; ++r) part[(tc * 32 + r) * 128 + q * 32 + lane] = v[r];
        }
    }
    cluster.sync();
    if (epi) {
        const int per = NT / S;
        // column split over GPUs: this call's epoch picks the half of every rank's y buffer
        const unsigned epoch =
            PEER ? *reinterpret_cast<const volatile unsigned *>(a.peer.own_state + kPeerEpochWord) + 1u : 0u;
        const uint2 sraw = *reinterpret_cast<const uint2 *>(a.sv + nb * 128 + lane * 4);
        const __half2 s01 = bits_half2(sraw.x), s23 = bits_half2(sraw.y);
        for (int t = split * per + warp; t < (split + 1) * per; t += 12) {
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            for (int s = 0; s < S; ++s) {
                const float4 p = *reinterpret_cast<const float4 *>(cluster.map_shared_rank(part, s) + t * 128 + lane * 4);
                v[0] = __fadd_rn(v[0], p.x);
                v[1] = __fadd_rn(v[1], p.y);
                v[2] = __fadd_rn(v[2], p.z);
                v[3] = __fadd_rn(v[3], p.w);
            }
            h128_warp4(v);
            const int token = tg * NT + t;
            if (token < M) {
                float4 o;
                o.x = __fmul_rn(v[0], __low2float(s01));
                o.y = __fmul_rn(v[1], __high2float(s01));
                o.z = __fmul_rn(v[2], __low2float(s23));
                o.w = __fmul_rn(v[3], __high2float(s23));
                if constexpr (PEER) {  // NVLink stores of (epoch, value) words into every rank's y
                    const long long off = ((epoch & 1u) ? a.peer.y_half : 0) + token * a.peer.y_stride +
                                          a.peer.y_col0 + nb * 128 + lane * 4;
                    for (int pi = 0; pi < a.peer.npeers; ++pi) store_pairs4(a.peer.y[pi] + off, o, epoch);
                } else {
                    *reinterpret_cast<float4 *>(a.y + size_t(token) * a.y_stride + nb * 128 + lane * 4) = o;
                }
            }
        }
    }
    cluster.sync();  // the partials stay until every rank has read them
    tc_fence_before();
    __syncthreads();
    if (warp == 12) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// ---------------------------------------------------------------------------

namespace {

// The PEER build (output to the peers' buffers, for the column split) exists for mul1 weights.
template <int BITS>
void * gemm_kernel_cb(unsigned cb, bool peer) {
    if (peer) return cb == CB_MUL1 ? reinterpret_cast<void *>(k_gemm<BITS, CB_MUL1, true>) : nullptr;
    switch (cb) {
        case CB_3INST: return reinterpret_cast<void *>(k_gemm<BITS, CB_3INST, false>);
        case CB_MCG: return reinterpret_cast<void *>(k_gemm<BITS, CB_MCG, false>);
        case CB_MUL1: return reinterpret_cast<void *>(k_gemm<BITS, CB_MUL1, false>);
        default: return nullptr;
    }
}

void * gemm_kernel_for(unsigned bits, unsigned cb, bool peer = false) {
    switch (bits) {
        case 1: return gemm_kernel_cb<1>(cb, peer);
        case 2: return gemm_kernel_cb<2>(cb, peer);
        case 3: return gemm_kernel_cb<3>(cb, peer);
        case 4: return gemm_kernel_cb<4>(cb, peer);
        case 5: return gemm_kernel_cb<5>(cb, peer);
        case 6: return gemm_kernel_cb<6>(cb, peer);
        case 7: return gemm_kernel_cb<7>(cb, peer);
        case 8: return gemm_kernel_cb<8>(cb, peer);
        default: return nullptr;
    }
}

constexpr size_t kGemmMaxSmem = 227 * 1024;

size_t group_bytes(unsigned bits) { return size_t(kGroupChunks) * 256 * bits; }
size_t xring_bytes(int ntok) { return size_t(kSlots) * ntok * 32 * kGroupChunks; }

size_t gemm_smem(unsigned bits, int ntok, int wstages) {
    const size_t s = size_t(wstages) * group_bytes(bits) + xring_bytes(ntok) + kBarBytes;
    return s < kMinSmem ? kMinSmem : s;
}

// Most tokens per CTA (a multiple of 32, <= 256) whose rings fit the shared
// memory with the minimum trellis ring of three groups.
int gemm_max_tokens(unsigned bits) {
    const long long room = (long long)kGemmMaxSmem - kBarBytes - 3 * (long long)group_bytes(bits);
    const int t = int(room / (kSlots * 32 * kGroupChunks)) / 32 * 32;
    return t < kMaxTok ? t : kMaxTok;
}

// Deepest trellis ring (a multiple of 3 groups, <= 15 groups and ~96 KB) that fits next to the activation slots.
int gemm_wstages(unsigned bits, int ntok) {
    const long long room = (long long)kGemmMaxSmem - kBarBytes - (long long)xring_bytes(ntok);
    long long by_room = room / (long long)group_bytes(bits);
    long long by_bytes = (96 * 1024) / (long long)group_bytes(bits);
    long long w = by_room < by_bytes ? by_room : by_bytes;
    if (w > kMaxWStages - 1) w = kMaxWStages - 1;
    w = w / 3 * 3;
    return w < 3 ? 3 : int(w);
}
// the partial tile [NTOK][128] fp32 reuses the activation slots: 512 NTOK <= 768 NTOK
static_assert(kSlots * 32 * kGroupChunks >= 128 * 4, "the partial tile must fit in the activation slots");
static_assert((2 * kMaxWStages + 2 * kSlots + 1) * 8 + 4 <= kBarBytes, "barrier area");
static_assert(kACol0 + kSlots * kGroupChunks * 8 <= int(kTmemCols) && kMaxTok <= kACol0, "TMEM columns");

bool gemm_prepare(int device, unsigned bits, unsigned cb) {
    static std::mutex mu;
    static bool done[64][9][3] = {};
    if (device < 0 || device >= 64 || bits < 1 || bits > 8 || cb > 2) return false;
    std::lock_guard<std::mutex> g(mu);
    if (done[device][bits][cb]) return true;
    for (const bool peer : {false, true}) {
        const void * k = gemm_kernel_for(bits, cb, peer);
        if (!k) continue;  // no PEER build for this codebook
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kGemmMaxSmem)) != cudaSuccess)
            return false;
        if (cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) return false;
    }
    done[device][bits][cb] = true;
    return true;
}

// Clusters of `splits` CTAs that can be resident at once (one CTA per SM; the
// GPC layout caps the count below SMs / splits), cached per device.
int max_active_clusters(int device, unsigned bits, unsigned cb, int splits) {
    static std::mutex mu;
    static int cache[64][5] = {};
    int si = 0;
    while ((1 << si) < splits && si < 4) ++si;
    if (device < 0 || device >= 64) return 0;
    std::lock_guard<std::mutex> g(mu);
    if (cache[device][si]) return cache[device][si];
    if (!gemm_prepare(device, bits, cb)) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(splits) * 16, 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = kMinSmem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = unsigned(splits);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_kernel_for(bits, cb), &cfg) != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        return 0;
    }
    cache[device][si] = n;
    return n;
}

}  // namespace

// Tokens per CTA: as many as one CTA takes (<= 256, fewer at 6-8 bits where the
// trellis ring is larger), split evenly over the token groups.  K split: the
// largest S in 1, 2, 4, 8 whose clusters of all units are resident in one wave
// and that leaves every rank at least 2 groups of 8 chunks; a second wave
// costs more than the extra decode parallelism gains.
GemmPlan plan_gemm(int device, int sms, size_t k, size_t nblocks, unsigned bits, unsigned cb, int rows, int tokens,
                   int splits) {
    GemmPlan p{};
    int tmax = gemm_max_tokens(bits);
    if (tokens > 0 && tokens < tmax) tmax = tokens / 32 * 32 > 32 ? tokens / 32 * 32 : 32;
    p.tgroups = (rows + tmax - 1) / tmax;
    const int per = (rows + p.tgroups - 1) / p.tgroups;
    p.ntok = (per + 31) / 32 * 32;
    const int nchunks = int(k / 16);
    const long long units = (long long)nblocks * p.tgroups;
    int S = 1;
    for (int c = 2; c <= 8; c *= 2) {
        if (nchunks / c < 2 * kGroupChunks) break;
        const int fit = max_active_clusters(device, bits, cb, c);
        if (fit <= 0 || units > fit) break;
        S = c;
    }
    if (units > sms) S = 1;
    if (splits > 0) S = splits < 16 ? splits : 16;
    p.splits = S;
    const int cps = (nchunks + S - 1) / S;
    p.cps = (cps + kGroupChunks - 1) / kGroupChunks * kGroupChunks;
    p.wstages = gemm_wstages(bits, p.ntok);
    p.smem = gemm_smem(bits, p.ntok, p.wstages);
    p.xt_bytes = size_t(p.tgroups) * p.ntok * k * sizeof(__half);
    return p;
}

cudaError_t launch_gemm(const GemmPlan & p, const uint32_t * lsc, const __half * su, const __half * sv, size_t k,
                        size_t nblocks, unsigned bits, unsigned cb, int device, const void * x, int x_f16,
                        long long x_stride, int rows, const int32_t * m_dev, int m_base, float * y, long long y_stride,
                        __half * xt, bool pdl, cudaStream_t st, const PeerOut * peer) {
    if (!gemm_prepare(device, bits, cb)) return cudaErrorInvalidValue;
    if (peer && cb != CB_MUL1) return cudaErrorInvalidValue;
    const int rows_pad = p.tgroups * p.ntok;
    const long long warps = (long long)rows_pad * (long long)(k / 128);
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
        cudaError_t e = cudaLaunchKernelEx(&cfg, k_tile_x, x, x_f16, x_stride, su, rows, m_dev, m_base, int(k), p.ntok,
                                           rows_pad, xt);
        if (e != cudaSuccess) return e;
    }
    GemmArgs a{};
    if (peer) a.peer = *peer;
    a.lsc = lsc;
    a.sv = sv;
    a.xt = xt;
    a.y = y;
    a.y_stride = y_stride;
    a.M = rows;
    a.m_dev = m_dev;
    a.m_base = m_base;
    a.ntok = p.ntok;
    a.tgroups = p.tgroups;
    a.nchunks = int(k / 16);
    a.cps = p.cps;
    a.splits = p.splits;
    a.wstages = p.wstages;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(nblocks * p.tgroups * p.splits), 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
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
    return cudaLaunchKernelExC(&cfg, gemm_kernel_for(bits, cb, peer != nullptr), args);
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
