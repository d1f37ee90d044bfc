// Device kernels of the hybrid decoder around the EXL3 operator: the layers a
// Qwen3.5-style 3:1 gated-delta-rule / full-attention decoder runs between its
// packed matmuls (embedding, residual + RMSNorm, SwiGLU, q/k norm + RoPE + FP16
// KV append, GQA attention, the gated delta rule with its short convolution
// and gates, the tied fp16 head with a fused argmax).
//
// Rows are the packed tokens of one scheduler step (exl3cu_pack_ragged's
// output): row r belongs to step sequence row_seq[r] at position row_pos[r];
// step sequence s owns cache slot seq_slot[s] and the rows
// [row_offsets[s], row_offsets[s+1]).  All arithmetic and every activation is
// fp32 (the packed operator takes f32 inputs and quantises them itself, more
// finely than fp16 would); the KV cache and the embedding/head are fp16.
//
// The math is the published one (the reference's own graph code is upstream
// llama.cpp and not part of its tree): gated delta rule (Yang et al., "Gated
// Delta Networks", ICLR 2025) S_t = a_t S_{t-1} (I - b_t k_t k_t^T) +
// b_t v_t k_t^T, o_t = S_t q_t, with a_t = exp(-exp(A_log) softplus(x W_a +
// dt_bias)) and b_t = sigmoid(x W_b) (the exporter's A_log -> -exp(A_log)
// convention, tools/export_native_gguf.py:106-118); causal depthwise conv of
// width 4 with SiLU over the q/k/v channels; L2-normalised q, k with q scaled
// by 1/sqrt(128); per-head RMSNorm of o gated by SiLU(z).  Full attention:
// per-head RMSNorm of q and k, rotary embedding on the two halves of each
// head, softmax(q k^T / sqrt(128)) v over positions 0..pos, 4 q heads per kv
// head.
//
// Every kernel is launched with programmatic dependent launch: it lets the
// next kernel be scheduled at once (griddepcontrol.launch_dependents) and
// reads nothing that a kernel of the step writes, and writes nothing, before
// its own griddepcontrol.wait (layer constants such as the delta rule's conv
// weights may load earlier), which returns when the preceding grid has
// completed and flushed -- so a chain of these
// kernels and the EXL3 operator keeps stream order while each launch's
// latency overlaps the tail of the one before.
#include "exl3cu.h"
#include "exl3cu_async.cuh"
#include "exl3cu_hybrid.h"
#include "exl3cu_internal.h"

#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>

namespace cg = cooperative_groups;

namespace exl3cu {

namespace {

constexpr int kHD = 128;     // head dimension
constexpr int kNH = 16;      // q heads / delta-rule heads
constexpr int kNKV = 4;      // kv heads
constexpr int kConvW = 4;    // short convolution width

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int s = 16; s; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
    return v;
}

// Sum over a CTA of `nwarps` warps; `red` holds nwarps floats.  All threads get the total.
__device__ __forceinline__ float block_sum(float v, float * red, int nwarps) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nwarps; ++i) t += red[i];  // fixed order: deterministic
    return t;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }

// ---------------------------------------------------------------------------

// With h_ss (H a multiple of 128): also the row's sum of squares per 128-block,
// [rows][H/128] (warp w takes blocks w, w + 8, ...; lane 4 values of a block).
__global__ void k_embed(const __half * __restrict__ table, const int32_t * __restrict__ ids, int vocab, int H,
                        float * __restrict__ h, float * __restrict__ h_ss) {
    pdl_trigger();
    pdl_wait_primary();
    const int r = blockIdx.x;
    const int32_t id = ids[r];
    const bool ok = id >= 0 && id < vocab;  // an id outside the table gives a zero row
    if (!h_ss) {
        for (int i = threadIdx.x; i < H; i += blockDim.x)
            h[size_t(r) * H + i] = ok ? __half2float(table[size_t(id) * H + i]) : 0.f;
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int b = warp; b < H / 128; b += nw) {
        const int i = b * 128 + lane * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ok) {
            const uint2 raw = *reinterpret_cast<const uint2 *>(table + size_t(id) * H + i);
            const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
            const float2 c = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
            v = make_float4(a.x, a.y, c.x, c.y);
        }
        *reinterpret_cast<float4 *>(h + size_t(r) * H + i) = v;
        float ss = v.x * v.x;
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
        ss = warp_sum(ss);
        if (lane == 0) h_ss[size_t(r) * (H / 128) + b] = ss;
    }
}

// h += delta (when given), then out = h / sqrt(mean(h^2) + eps) * w.
// One CTA of 256 threads per row; the row (H <= 8192, H % 4 == 0) stays in
// registers between the sum and the scaling.
constexpr int kNormThreads = 256;
constexpr int kNormMaxVec = 8;  // float4 per thread: H <= 8192

__global__ void __launch_bounds__(kNormThreads)
k_rmsnorm(float * __restrict__ h, const float * __restrict__ delta, int delta_stride, const float * __restrict__ w,
          float eps, int H, float * __restrict__ out) {
    __shared__ float red[kNormThreads / 32];
    pdl_trigger();
    pdl_wait_primary();
    const int r = blockIdx.x;
    float4 * hr = reinterpret_cast<float4 *>(h + size_t(r) * H);
    const float4 * dr = delta ? reinterpret_cast<const float4 *>(delta + size_t(r) * delta_stride) : nullptr;
    const int nv = H / 4;
    float4 v[kNormMaxVec];
    float ss = 0.f;
#pragma unroll
    for (int q = 0; q < kNormMaxVec; ++q) {
        const int e = threadIdx.x + q * kNormThreads;
        if (e < nv) {
            float4 x = hr[e];
            if (dr) {
                const float4 d = dr[e];
                x.x += d.x; x.y += d.y; x.z += d.z; x.w += d.w;
                hr[e] = x;
            }
            v[q] = x;
            ss = fmaf(x.x, x.x, ss);
            ss = fmaf(x.y, x.y, ss);
            ss = fmaf(x.z, x.z, ss);
            ss = fmaf(x.w, x.w, ss);
        }
    }
    const float inv = rsqrtf(block_sum(ss, red, kNormThreads / 32) / float(H) + eps);
    const float4 * wr = reinterpret_cast<const float4 *>(w);
    float4 * o4 = reinterpret_cast<float4 *>(out + size_t(r) * H);
#pragma unroll
    for (int q = 0; q < kNormMaxVec; ++q) {
        const int e = threadIdx.x + q * kNormThreads;
        if (e < nv) {
            const float4 wv = wr[e];
            o4[e] = make_float4(v[q].x * inv * wv.x, v[q].y * inv * wv.y, v[q].z * inv * wv.z, v[q].w * inv * wv.w);
        }
    }
}

// out = silu(gate) * up; gu row = [gate (F) | up (F)].
__global__ void k_swiglu(const float * __restrict__ gu, int F, float * __restrict__ out) {
    pdl_trigger();
    pdl_wait_primary();
    const int r = blockIdx.y;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= F) return;
    const float g = gu[size_t(r) * 2 * F + i], u = gu[size_t(r) * 2 * F + F + i];
    out[size_t(r) * F + i] = silu(g) * u;
}

// One head of 128 values x[d] (lane holds d = lane + 32 q, q < 4): RMSNorm
// with weights wn, then the rotary embedding of the pairs (i, i + 64) by
// pos * inv_freq[i].  Shared by k_attn_prep and k_attn_decode, which must
// agree bit for bit.
__device__ __forceinline__ void head_norm_rope(const float * __restrict__ x, const float * __restrict__ wn,
                                               const float * __restrict__ inv_freq, int pos, float eps, int lane,
                                               float (&o)[4]) {
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = x[lane + 32 * q];
    float ss = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) ss = fmaf(v[q], v[q], ss);
    const float inv = rsqrtf(warp_sum(ss) / float(kHD) + eps);
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = v[q] * inv * wn[lane + 32 * q];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const int i = lane + 32 * q;  // first-half index; partner i + 64
        float sn, cs;
        sincosf(float(pos) * inv_freq[i], &sn, &cs);
        o[q] = v[q] * cs - v[q + 2] * sn;
        o[q + 2] = v[q + 2] * cs + v[q] * sn;
    }
}

// Per row: RMSNorm of each q and k head (weights qn_w / kn_w), rotary
// embedding (pairs i, i+64 rotated by pos * inv_freq[i]), k and v appended to
// the fp16 cache at the row's position, q written out (f32).  One CTA of
// (kNH + kNKV) warps per row; warp = head.
__global__ void k_attn_prep(const float * __restrict__ qkv, const int32_t * __restrict__ row_seq,
                            const int32_t * __restrict__ row_pos, const int32_t * __restrict__ seq_slot,
                            const float * __restrict__ qn_w, const float * __restrict__ kn_w,
                            const float * __restrict__ inv_freq, float eps, __half * __restrict__ kc,
                            __half * __restrict__ vc, int max_len, int n_slots, float * __restrict__ q_out) {
    pdl_trigger();
    pdl_wait_primary();
    const int r = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = row_pos[r];
    const int slot = seq_slot[row_seq[r]];
    if (pos < 0 || pos >= max_len || slot < 0 || slot >= n_slots) return;  // outside the cache: nothing written
    constexpr int QKV = (kNH + 2 * kNKV) * kHD;
    const float * src = qkv + size_t(r) * QKV;
    const bool is_q = warp < kNH;
    const int head = is_q ? warp : warp - kNH;
    const float * x = src + (is_q ? head * kHD : kNH * kHD + head * kHD);
    float o[4];
    head_norm_rope(x, is_q ? qn_w : kn_w, inv_freq, pos, eps, lane, o);
    if (is_q) {
#pragma unroll
        for (int q = 0; q < 4; ++q) q_out[size_t(r) * kNH * kHD + head * kHD + lane + 32 * q] = o[q];
    } else {
        const size_t base = ((size_t(slot) * kNKV + head) * max_len + pos) * kHD;
        const float * vs = src + kNH * kHD + kNKV * kHD + head * kHD;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            kc[base + lane + 32 * q] = __float2half_rn(o[q]);
            vc[base + lane + 32 * q] = __float2half_rn(vs[lane + 32 * q]);
        }
    }
}

// softmax(q K^T * scale) V over positions 0..pos of the row's sequence.
// Grid (q head, row, split): the CTA (4 warps) covers split `z` of the
// positions; warp w takes positions w, w+4, ... of that range, lane holds 4
// consecutive dims; online softmax per warp, merged in warp order.  With
// more than one split each CTA stores (max, sum, acc[128]) to `part`, and the
// last CTA of the (row, head) to arrive (ticket) merges the splits in split
// order and resets the ticket.
constexpr int kAttnPart = kHD + 4;  // per split: max, sum, 2 pad, acc[128] (16-byte aligned records)

// PREP (k_attn_decode): a step in which every sequence has exactly one row,
// so a row attends to cached positions plus its own new one.  q points at the
// packed [q | k | v] rows; the CTA computes its q head and the row's new k, v
// (k_attn_prep's math, same rounding) into shared memory and uses them for
// position pos, and one CTA per (row, kv head) appends k, v to the cache.  No
// CTA of the launch reads the cache at pos, so the append needs no ordering.
template <bool PREP>
__global__ void __launch_bounds__(128)
k_attn(const float * __restrict__ q, const int32_t * __restrict__ row_seq, const int32_t * __restrict__ row_pos,
       const int32_t * __restrict__ seq_slot, __half * __restrict__ kc, __half * __restrict__ vc,
       int max_len, int n_slots, float scale, float * __restrict__ part, unsigned * __restrict__ tickets,
       float * __restrict__ out, const float * __restrict__ qn_w, const float * __restrict__ kn_w,
       const float * __restrict__ inv_freq, float eps) {
    __shared__ float sm_m[4], sm_l[4], sm_acc[4][kHD];
    __shared__ __align__(16) float sm_q[PREP ? kHD : 1], sm_k[PREP ? kHD : 1], sm_v[PREP ? kHD : 1];
    __shared__ unsigned sm_last;
    pdl_trigger();
    pdl_wait_primary();
    const int head = blockIdx.x, r = blockIdx.y, z = blockIdx.z, S = gridDim.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slot = seq_slot[row_seq[r]];
    if (slot < 0 || slot >= n_slots) return;
    const int pos = row_pos[r];
    const int npos = min(pos, max_len - 1) + 1;
    const int chunk = (npos + S - 1) / S;
    const int p0 = z * chunk, p1 = min(npos, p0 + chunk);
    const int kvh = head / (kNH / kNKV);
    float4 qv;
    if constexpr (PREP) {
        constexpr int QKV = (kNH + 2 * kNKV) * kHD;
        const float * src = q + size_t(r) * QKV;
        // the CTA of the kv group's first q head and split 0 appends (a position outside the cache: none)
        const bool writer = pos >= 0 && pos < max_len && head % (kNH / kNKV) == 0 && z == 0;
        const size_t base = ((size_t(slot) * kNKV + kvh) * max_len + (writer ? pos : 0)) * kHD;
        if (warp == 0) {
            float o[4];
            head_norm_rope(src + head * kHD, qn_w, inv_freq, pos, eps, lane, o);
#pragma unroll
            for (int q2 = 0; q2 < 4; ++q2) sm_q[lane + 32 * q2] = o[q2];
        } else if (warp == 1) {
            float o[4];
            head_norm_rope(src + kNH * kHD + kvh * kHD, kn_w, inv_freq, pos, eps, lane, o);
#pragma unroll
            for (int q2 = 0; q2 < 4; ++q2) {
                const __half hk = __float2half_rn(o[q2]);
                sm_k[lane + 32 * q2] = __half2float(hk);
                if (writer) kc[base + lane + 32 * q2] = hk;
            }
        } else if (warp == 2) {
            const float * vs = src + kNH * kHD + kNKV * kHD + kvh * kHD;
#pragma unroll
            for (int q2 = 0; q2 < 4; ++q2) {
                const __half hv = __float2half_rn(vs[lane + 32 * q2]);
                sm_v[lane + 32 * q2] = __half2float(hv);
                if (writer) vc[base + lane + 32 * q2] = hv;
            }
        }
        __syncthreads();
        qv = *reinterpret_cast<const float4 *>(sm_q + lane * 4);
    } else {
        qv = *reinterpret_cast<const float4 *>(q + size_t(r) * kNH * kHD + head * kHD + lane * 4);
    }
    const __half * kb = kc + (size_t(slot) * kNKV + kvh) * max_len * kHD;
    const __half * vb = vc + (size_t(slot) * kNKV + kvh) * max_len * kHD;
    float m = -INFINITY, l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
    // warp w takes positions w, w+4, w+8, ... of the range, kU at a time: their k/v loads go out
    // together, then the online-softmax updates run in position order
    constexpr int kU = 8;
    for (int pb = p0 + warp; pb < p1; pb += 4 * kU) {
        float2 k01[kU], k23[kU], v01[kU], v23[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int p = pb + 4 * u;
            if (PREP && p == pos) {  // this step's own position: from shared memory
                const float4 kk = *reinterpret_cast<const float4 *>(sm_k + lane * 4);
                const float4 vv = *reinterpret_cast<const float4 *>(sm_v + lane * 4);
                k01[u] = make_float2(kk.x, kk.y);
                k23[u] = make_float2(kk.z, kk.w);
                v01[u] = make_float2(vv.x, vv.y);
                v23[u] = make_float2(vv.z, vv.w);
            } else {
                uint2 kr = make_uint2(0, 0), vr = make_uint2(0, 0);
                if (p < p1) {
                    kr = *reinterpret_cast<const uint2 *>(kb + size_t(p) * kHD + lane * 4);
                    vr = *reinterpret_cast<const uint2 *>(vb + size_t(p) * kHD + lane * 4);
                }
                k01[u] = __half22float2(*reinterpret_cast<const __half2 *>(&kr.x));
                k23[u] = __half22float2(*reinterpret_cast<const __half2 *>(&kr.y));
                v01[u] = __half22float2(*reinterpret_cast<const __half2 *>(&vr.x));
                v23[u] = __half22float2(*reinterpret_cast<const __half2 *>(&vr.y));
            }
        }
        float sc[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            float s = qv.x * k01[u].x;
            s = fmaf(qv.y, k01[u].y, s);
            s = fmaf(qv.z, k23[u].x, s);
            s = fmaf(qv.w, k23[u].y, s);
            sc[u] = warp_sum(s) * scale;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            if (pb + 4 * u >= p1) break;
            const float s = sc[u];
            const float mn = fmaxf(m, s);
            const float corr = expf(m - mn), e = expf(s - mn);
            l = l * corr + e;
            acc[0] = fmaf(e, v01[u].x, acc[0] * corr);
            acc[1] = fmaf(e, v01[u].y, acc[1] * corr);
            acc[2] = fmaf(e, v23[u].x, acc[2] * corr);
            acc[3] = fmaf(e, v23[u].y, acc[3] * corr);
            m = mn;
        }
    }
    if (lane == 0) {
        sm_m[warp] = m;
        sm_l[warp] = l;
    }
#pragma unroll
    for (int q2 = 0; q2 < 4; ++q2) sm_acc[warp][lane * 4 + q2] = acc[q2];
    __syncthreads();
    // merge the warps (warp 0): M, L, A over this CTA's range
    float M = -INFINITY, L = 0.f, A[4] = {0.f, 0.f, 0.f, 0.f};
    if (warp == 0) {
        for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w]);
        for (int w = 0; w < 4; ++w) {
            if (sm_m[w] == -INFINITY) continue;  // a warp that saw no position
            const float c = expf(sm_m[w] - M);
            L = fmaf(sm_l[w], c, L);
#pragma unroll
            for (int q2 = 0; q2 < 4; ++q2) A[q2] = fmaf(sm_acc[w][lane * 4 + q2], c, A[q2]);
        }
    }
    float * dst = out + size_t(r) * kNH * kHD + head * kHD + lane * 4;
    if (S == 1) {
        if (warp == 0) {
            const float invL = 1.0f / L;
#pragma unroll
            for (int q2 = 0; q2 < 4; ++q2) dst[q2] = A[q2] * invL;
        }
        return;
    }
    float * mine = part + ((size_t(r) * kNH + head) * S + z) * kAttnPart;
    if (warp == 0) {
        if (lane == 0) {
            mine[0] = M;
            mine[1] = L;
        }
        reinterpret_cast<float4 *>(mine + 4)[lane] = make_float4(A[0], A[1], A[2], A[3]);
        __threadfence();
    }
    __syncthreads();
    if (threadIdx.x == 0) sm_last = atomicAdd(tickets + size_t(r) * kNH + head, 1u) == unsigned(S - 1);
    __syncthreads();
    if (!sm_last || warp != 0) return;
    __threadfence();
    // merge the splits (S <= 64): lane j holds the (max, sum) of splits j and j + 32, loaded together;
    // the weights exp(m_z - M) go to every lane by shuffles; the sums run in a fixed order
    const float * all = part + (size_t(r) * kNH + head) * S * kAttnPart;
    float mz[2], lz[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int zz = lane + 32 * i;
        mz[i] = zz < S ? __ldcg(all + zz * kAttnPart) : -INFINITY;
        lz[i] = zz < S ? __ldcg(all + zz * kAttnPart + 1) : 0.f;
    }
    float GM = fmaxf(mz[0], mz[1]);
#pragma unroll
    for (int sh = 16; sh; sh >>= 1) GM = fmaxf(GM, __shfl_xor_sync(0xffffffffu, GM, sh));
    float cz[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) cz[i] = mz[i] == -INFINITY ? 0.f : expf(mz[i] - GM);  // a split that saw nothing: 0
    const float GL = warp_sum(fmaf(lz[1], cz[1], lz[0] * cz[0]));
    float G[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int zz = 0; zz < S; ++zz) {
        const float c = __shfl_sync(0xffffffffu, zz < 32 ? cz[0] : cz[1], zz & 31);
        const float4 a = __ldcg(reinterpret_cast<const float4 *>(all + zz * kAttnPart + 4) + lane);
        G[0] = fmaf(a.x, c, G[0]);
        G[1] = fmaf(a.y, c, G[1]);
        G[2] = fmaf(a.z, c, G[2]);
        G[3] = fmaf(a.w, c, G[3]);
    }
    const float invL = 1.0f / GL;
#pragma unroll
    for (int q2 = 0; q2 < 4; ++q2) dst[q2] = G[q2] * invL;
    if (lane == 0) tickets[size_t(r) * kNH + head] = 0u;  // ready for the next launch
}

// Gated delta rule for one (head, step sequence): the sequence's rows in
// order, in tiles of kGdnTile rows.  A cluster of kGdnSplit CTAs serves one
// head; CTA rank q owns v columns [32 q, 32 q + 32) of the head's 128 x 128
// fp32 state.  Thread t owns column 32 q + (t & 31) for k rows
// [16 (t >> 5), +16): 16 registers, loaded from and stored to HBM coalesced.
// The recurrence of a column needs only that column, so the ranks run it
// independently.  Per tile:
//   A (rows in parallel, every rank): the tile's conv inputs staged in shared
//     memory, causal conv + SiLU of the head's q, k, v channels, L2 norms (q
//     also x 1/sqrt(128)), k.q, the gates a = x.W_a, b = x.W_b -> alpha =
//     exp(-exp(A_log) softplus(a + dt_bias)), beta = sigmoid(b);
//   B (rows in order, the only sequential part, one barrier per row): S^T k
//     and S^T q over the eight k slices, u = beta (v - alpha S^T k),
//     o = alpha S^T q + (k.q) u, S = alpha S + k u^T;
//   C (rows in parallel): each rank's share of sum(o^2) per row goes to its
//     peers through distributed shared memory (one cluster barrier per tile,
//     double-buffered), then RMSNorm(o) * norm_w * SiLU(z) -> out (f32).
// The conv state (last three inputs per channel) is read as it was before the
// step and rewritten at the end by rank 0.
constexpr int kGdnThreads = 256;
constexpr int kGdnTile = 16;
constexpr int kGdnSplit = 4;                  // CTAs (v-column slices) per head
constexpr int kGdnCols = kHD / kGdnSplit;     // 32 columns per CTA
constexpr int kGdnKParts = kGdnThreads / kGdnCols;  // 8 k slices
constexpr int kGdnKRows = kHD / kGdnKParts;   // 16 k rows per thread

static __device__ unsigned g_hyb_status;  // reserved: sticky error bits of these kernels (none raised today)

// Shared-memory layout of k_gdn (floats unless noted).
struct GdnSmem {
    static constexpr int Q = 0;                               // [T][128] conv+norm q
    static constexpr int K = Q + kGdnTile * kHD;              // [T][128] k
    static constexpr int V = K + kGdnTile * kHD;              // [T][128] v
    static constexpr int O = V + kGdnTile * kHD;              // [T][32] o of this rank's columns
    static constexpr int RED = O + kGdnTile * kGdnCols;       // [2 buffers][2][8][32]
    static constexpr int PSUM = RED + 2 * 2 * kGdnKParts * kGdnCols;  // [2 tiles][rank][T] sum(o^2) of every rank
    static constexpr int CW = PSUM + 2 * kGdnSplit * kGdnTile;  // [384][4] conv weights of the head
    static constexpr int GATE = CW + 3 * kHD * kConvW;        // [T][4]: alpha, beta, k.q
    static constexpr int CX = GATE + kGdnTile * 4;            // [T+3][384] conv inputs of the tile
    static constexpr int WAB = CX + (kGdnTile + kConvW - 1) * 3 * kHD;  // fp16 [2][H] gate rows (H <= 8192)
    static constexpr int floats_without_wab = WAB;
};

// MINB CTAs per SM: 1 (no register cap) for steps of one or two sequences, whose
// few CTAs fit the GPU anyway; 2 (at most 128 registers) for more, so that the
// clusters of a many-sequence step run in half the waves.
template <int MINB>
__global__ void __launch_bounds__(kGdnThreads, MINB)
k_gdn(const float * __restrict__ qkvz, const float * __restrict__ xn, const float * __restrict__ xn_norm_w,
      const __half * __restrict__ wab, int H, const float * __restrict__ conv_w, float * __restrict__ conv_state,
      const float * __restrict__ A_log, const float * __restrict__ dt_bias, const float * __restrict__ norm_w,
      float eps, float * __restrict__ S, const int32_t * __restrict__ row_offsets,
      const int32_t * __restrict__ seq_slot, int n_slots, float * __restrict__ out) {
    extern __shared__ __align__(128) float sm[];
    float * tq = sm + GdnSmem::Q;
    float * tk = sm + GdnSmem::K;
    float * tv = sm + GdnSmem::V;
    float * to = sm + GdnSmem::O;
    float * red = sm + GdnSmem::RED;
    float * psum = sm + GdnSmem::PSUM;
    float * cw = sm + GdnSmem::CW;
    float * gate = sm + GdnSmem::GATE;
    float * cx = sm + GdnSmem::CX;
    __half * wab_s = reinterpret_cast<__half *>(sm + GdnSmem::WAB);
    cg::cluster_group cluster = cg::this_cluster();
    pdl_trigger();
    const int h = blockIdx.x / kGdnSplit, s = blockIdx.y;
    const int rank = int(cluster.block_rank());
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    constexpr int QKVZ = 4 * kNH * kHD;
    constexpr int CH = 3 * kNH * kHD;  // convolved channels (q, k, v)
    constexpr int C3 = 3 * kHD;
    // the head's conv weights, gate rows and scalars are layer constants that no kernel
    // writes: they load while the previous kernel is still running
    for (int c = t; c < C3; c += kGdnThreads) {
        const int ch = (c / kHD) * kNH * kHD + h * kHD + c % kHD;
#pragma unroll
        for (int w = 0; w < kConvW; ++w) cw[c * kConvW + w] = conv_w[size_t(ch) * kConvW + w];
    }
    for (int i = t; i < H; i += kGdnThreads) {
        wab_s[i] = wab[size_t(h) * H + i];
        wab_s[H + i] = wab[size_t(kNH + h) * H + i];
    }
    const float A = -expf(A_log[h]);
    const float dtb = dt_bias[h];
    const float qscale = rsqrtf(float(kHD));
    pdl_wait_primary();
    const int slot = seq_slot[s];
    const int r0 = row_offsets[s], r1 = row_offsets[s + 1];
    // every CTA of the cluster takes the same early exit, so no cluster barrier is left waiting
    if (slot < 0 || slot >= n_slots || r1 <= r0) return;
    const int jj = t & (kGdnCols - 1), kp = t >> 5;   // column in the slice, k slice
    const int j = rank * kGdnCols + jj;               // column in the head
    const int i0 = kp * kGdnKRows;
    float * Sg = S + (size_t(slot) * kNH + h) * kHD * kHD;
    float Sr[kGdnKRows];  // S[i0 + i][j]
#pragma unroll
    for (int i = 0; i < kGdnKRows; ++i) Sr[i] = Sg[(i0 + i) * kHD + j];
    int rb = 0;    // reduction buffer of the current row
    int tpar = 0;  // psum buffer of the current tile
    __syncthreads();
    for (int tr0 = r0; tr0 < r1; tr0 += kGdnTile, tpar ^= 1) {
        const int nt = min(kGdnTile, r1 - tr0);
        // gate projections: every warp takes the 128-element blocks warp, warp + 8, ... of each
        // row (a decode row is one round trip of 16-byte loads, not one per block), and the
        // eight partial sums of a row meet in shared memory in warp order.  With xn_norm_w the
        // rows are the residual stream h and the layer's RMSNorm is folded in:
        // x . W = rsqrt(mean(h^2) + eps) * sum h * w * W.
        constexpr int kGW = kGdnThreads / 32;
        float * gpart = red;  // [T][kGW][3]: free until the recurrence
#pragma unroll 2
        for (int rr = 0; rr < nt; ++rr) {
            const float * xr = xn + size_t(tr0 + rr) * H;
            float pa = 0.f, pb = 0.f, ss = 0.f;
            for (int ib0 = warp * 128 + lane * 4; ib0 < H; ib0 += kGW * 128 * 2) {
                float4 raw[2];
#pragma unroll
                for (int u = 0; u < 2; ++u)
                    raw[u] = ib0 + u * kGW * 128 < H ? *reinterpret_cast<const float4 *>(xr + ib0 + u * kGW * 128)
                                                     : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int ib = ib0 + u * kGW * 128;
                    if (ib >= H) break;
                    float xv[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
                    if (xn_norm_w) {
                        const float4 wv = *reinterpret_cast<const float4 *>(xn_norm_w + ib);
#pragma unroll
                        for (int q = 0; q < 4; ++q) ss = fmaf(xv[q], xv[q], ss);
                        xv[0] *= wv.x;
                        xv[1] *= wv.y;
                        xv[2] *= wv.z;
                        xv[3] *= wv.w;
                    }
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        pa = fmaf(xv[q], __half2float(wab_s[ib + q]), pa);
                        pb = fmaf(xv[q], __half2float(wab_s[H + ib + q]), pb);
                    }
                }
            }
            pa = warp_sum(pa);
            pb = warp_sum(pb);
            ss = warp_sum(ss);
            if (lane == 0) {
                float * gp = gpart + (rr * kGW + warp) * 3;
                gp[0] = pa;
                gp[1] = pb;
                gp[2] = ss;
            }
        }
        // ---- stage the conv inputs x[tr0-3 .. tr0+nt-1] of the head's 384 channels ----
        // (rows before the sequence's first come from the conv state); these loads are
        // independent of the gate rows' and go out before the barrier
        for (int e = t; e < (nt + kConvW - 1) * (C3 / 4); e += kGdnThreads) {
            const int rr = e / (C3 / 4), c4 = (e % (C3 / 4)) * 4;  // row tr0 - 3 + rr, channels c4..c4+3
            const int ri = tr0 - (kConvW - 1) + rr;
            const int part = c4 / kHD, d = c4 % kHD;
            const int ch = part * kNH * kHD + h * kHD + d;
            float4 x;
            if (ri >= r0) {
                x = *reinterpret_cast<const float4 *>(qkvz + size_t(ri) * QKVZ + ch);
            } else {
                const float * st = conv_state + (size_t(slot) * CH + ch) * (kConvW - 1) + (ri - r0 + kConvW - 1);
                x = make_float4(st[0], st[kConvW - 1], st[2 * (kConvW - 1)], st[3 * (kConvW - 1)]);
            }
            *reinterpret_cast<float4 *>(cx + rr * C3 + c4) = x;
        }
        __syncthreads();
        if (t < nt) {
            float pa = 0.f, pb = 0.f, ss = 0.f;
#pragma unroll
            for (int w = 0; w < kGW; ++w) {  // warp order
                const float * gp = gpart + (t * kGW + w) * 3;
                pa += gp[0];
                pb += gp[1];
                ss += gp[2];
            }
            if (xn_norm_w) {
                const float inv = rsqrtf(ss / float(H) + eps);
                pa *= inv;
                pb *= inv;
            }
            gate[t * 4 + 0] = expf(A * softplus(pa + dtb));  // alpha
            gate[t * 4 + 1] = 1.0f / (1.0f + expf(-pb));     // beta
        }
        // conv + SiLU for every (row, channel) of the tile, from shared memory
        for (int e = t; e < nt * C3; e += kGdnThreads) {
            const int rr = e / C3, c = e % C3;
            float acc = 0.f;
#pragma unroll
            for (int w = 0; w < kConvW; ++w) acc = fmaf(cx[(rr + w) * C3 + c], cw[c * kConvW + w], acc);
            const int part = c / kHD, d = c % kHD;
            (part == 0 ? tq : part == 1 ? tk : tv)[rr * kHD + d] = silu(acc);
        }
        __syncthreads();
        // L2 norms and k.q: warp per row
        for (int rr = warp; rr < nt; rr += kGdnThreads / 32) {
            float * qv = tq + rr * kHD;
            float * kv = tk + rr * kHD;
            float sq = 0.f, sk = 0.f;
            for (int d = lane; d < kHD; d += 32) {
                sq = fmaf(qv[d], qv[d], sq);
                sk = fmaf(kv[d], kv[d], sk);
            }
            const float iq = rsqrtf(warp_sum(sq) + 1e-6f) * qscale;
            const float ik = rsqrtf(warp_sum(sk) + 1e-6f);
            float kq = 0.f;
            for (int d = lane; d < kHD; d += 32) {
                qv[d] *= iq;
                kv[d] *= ik;
                kq = fmaf(kv[d], qv[d], kq);
            }
            kq = warp_sum(kq);
            if (lane == 0) gate[rr * 4 + 2] = kq;
        }
        __syncthreads();
        // ---- B: the recurrence, row by row (state slice in registers) ----
        for (int rr = 0; rr < nt; ++rr) {
            const float4 * kv4 = reinterpret_cast<const float4 *>(tk + rr * kHD + i0);
            const float4 * qv4 = reinterpret_cast<const float4 *>(tq + rr * kHD + i0);
            float a4[2] = {0.f, 0.f}, c4[2] = {0.f, 0.f};
#pragma unroll
            for (int i = 0; i < kGdnKRows / 4; ++i) {
                const float4 kk = kv4[i], qq = qv4[i];
                a4[0] = fmaf(Sr[4 * i], kk.x, a4[0]);
                a4[1] = fmaf(Sr[4 * i + 1], kk.y, a4[1]);
                a4[0] = fmaf(Sr[4 * i + 2], kk.z, a4[0]);
                a4[1] = fmaf(Sr[4 * i + 3], kk.w, a4[1]);
                c4[0] = fmaf(Sr[4 * i], qq.x, c4[0]);
                c4[1] = fmaf(Sr[4 * i + 1], qq.y, c4[1]);
                c4[0] = fmaf(Sr[4 * i + 2], qq.z, c4[0]);
                c4[1] = fmaf(Sr[4 * i + 3], qq.w, c4[1]);
            }
            float * rd = red + rb * 2 * kGdnKParts * kGdnCols;
            rd[kp * kGdnCols + jj] = a4[0] + a4[1];
            rd[kGdnKParts * kGdnCols + kp * kGdnCols + jj] = c4[0] + c4[1];
            __syncthreads();
            float a_j = 0.f, c_j = 0.f;
#pragma unroll
            for (int p = 0; p < kGdnKParts; ++p) {  // fixed order: every thread of column j agrees
                a_j += rd[p * kGdnCols + jj];
                c_j += rd[kGdnKParts * kGdnCols + p * kGdnCols + jj];
            }
            const float alpha = gate[rr * 4 + 0], beta = gate[rr * 4 + 1], kq = gate[rr * 4 + 2];
            const float u_j = beta * (tv[rr * kHD + j] - alpha * a_j);
            if (kp == 0) to[rr * kGdnCols + jj] = fmaf(kq, u_j, alpha * c_j);
#pragma unroll
            for (int i = 0; i < kGdnKRows / 4; ++i) {
                const float4 kk = kv4[i];
                Sr[4 * i] = fmaf(kk.x, u_j, alpha * Sr[4 * i]);
                Sr[4 * i + 1] = fmaf(kk.y, u_j, alpha * Sr[4 * i + 1]);
                Sr[4 * i + 2] = fmaf(kk.z, u_j, alpha * Sr[4 * i + 2]);
                Sr[4 * i + 3] = fmaf(kk.w, u_j, alpha * Sr[4 * i + 3]);
            }
            rb ^= 1;  // the next row writes the other buffer: no second barrier needed
        }
        __syncthreads();  // every row's o slice is in `to`
        // ---- C: this rank's sum(o^2) per row, exchanged across the cluster ----
        float * ps = psum + tpar * kGdnSplit * kGdnTile;  // [rank][T]
        constexpr int kZRows = kGdnTile / (kGdnThreads / 32);  // rows per warp
        const int d = rank * kGdnCols + lane;
        float zr[kZRows];  // the gate inputs z, loaded ahead of the exchange
#pragma unroll
        for (int q = 0; q < kZRows; ++q) {
            const int rr = warp + q * (kGdnThreads / 32);
            zr[q] = rr < nt ? qkvz[size_t(tr0 + rr) * QKVZ + 3 * kNH * kHD + h * kHD + d] : 0.f;
        }
        // this rank's partial goes into every rank's shared memory (its own included), so that after
        // the barrier each rank reads only its own: no remote access follows the last barrier, and a
        // CTA may exit without waiting for its peers
        for (int rr = warp; rr < nt; rr += kGdnThreads / 32) {
            const float o = to[rr * kGdnCols + lane];
            const float ss = warp_sum(o * o);
            if (lane < kGdnSplit) cluster.map_shared_rank(ps, lane)[rank * kGdnTile + rr] = ss;
        }
        cluster.sync();  // every rank's partial sums are in place
#pragma unroll
        for (int q = 0; q < kZRows; ++q) {
            const int rr = warp + q * (kGdnThreads / 32);
            if (rr >= nt) break;
            float ss = 0.f;
#pragma unroll
            for (int p = 0; p < kGdnSplit; ++p) ss += ps[p * kGdnTile + rr];  // rank order
            const float inv = rsqrtf(ss / float(kHD) + eps);
            const size_t r = size_t(tr0 + rr);
            out[r * kNH * kHD + h * kHD + d] = to[rr * kGdnCols + lane] * inv * norm_w[d] * silu(zr[q]);
        }
        if (tr0 + kGdnTile >= r1) break;  // the last tile's cx stays for the conv state below
        __syncthreads();  // the next tile overwrites tq, tk, tv, to, gate, cx (psum is double-buffered)
    }
    // No closing cluster barrier: peers only ever wrote into this CTA's shared memory before the
    // last tile's barrier, and every rank staged (read) the old conv state before arriving there.
    // The conv state: the last three inputs of the sequence so far (rank 0), which are
    // rows nt .. nt+2 of the last tile's staged inputs (those before the sequence's first
    // row were staged from the old conv state)
    if (rank == 0) {
        const int nt_last = (r1 - r0 - 1) % kGdnTile + 1;
        for (int c = t; c < C3; c += kGdnThreads) {
            const int ch = (c / kHD) * kNH * kHD + h * kHD + c % kHD;
            float * st = conv_state + (size_t(slot) * CH + ch) * (kConvW - 1);
#pragma unroll
            for (int w = 0; w < kConvW - 1; ++w) st[w] = cx[(nt_last + w) * C3 + c];
        }
    }
#pragma unroll
    for (int i = 0; i < kGdnKRows; ++i) Sg[(i0 + i) * kHD + j] = Sr[i];
}

// D += A B for one m16n8k16 tile (f16 x f16 -> f32): A row-major fragments a0..a3, B column
// fragments b0, b1 (the PTX ISA's layout for mma.m16n8k16).
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              __half2 b0, __half2 b1) {
    const uint32_t rb0 = *reinterpret_cast<const uint32_t *>(&b0), rb1 = *reinterpret_cast<const uint32_t *>(&b1);
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(rb0), "r"(rb1));
}

// Order-preserving key of a float (larger float, larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// logits[o][v] = sum_i xn[rows[o]][i] * E[v][i] (f32 x, fp16 E, fp32 sums) for
// nout <= 8 rows; best[o] = max over v of (key(logit) << 32 | ~v) (the first
// index wins ties).  Activations staged in shared memory.  One row: warp per
// vocab row, ITER = H / 256 16-byte loads per lane per vocab row issued
// together.  2..8 rows: 16 vocab rows per warp on the tensor cores (fp16 MMA
// with the activations split into fp16 hi + lo).
// With norm_w the rows are the residual stream h and the final RMSNorm is
// applied while staging, with k_rmsnorm's arithmetic (thread t sums the
// squares of float4s t, t + 256, ... in order; warps add in order), so the
// logits equal those of k_rmsnorm + this kernel bit for bit.  The last CTA to
// finish (a ticket in best[kHeadMaxRows]) turns best[] into tokens[] and
// leaves best[] zero for the next launch.
constexpr int kHeadMaxRows = 8;
constexpr int kHeadThreads = 256;

// Optional device-side token feedback for replayed decode steps (tokens NULL: none): the last CTA
// also writes row o's token into next_tokens[o], increments next_pos[o], appends it to
// log[counter * nout + o] (clamped to log_cap - 1) and increments counter.
struct HeadFeedback {
    int32_t * next_tokens;
    int32_t * next_pos;
    int32_t * log;
    long long * counter;
    long long log_cap;
};

// At most 64 registers: four CTAs per SM, the occupancy the one-row form is
// tuned for (a build at 40 registers measured slower within the decode step).
template <int ITER>
__global__ void __launch_bounds__(kHeadThreads, 4)
k_head(const float * __restrict__ xn, const int32_t * __restrict__ rows, int nout, int H,
       const __half * __restrict__ E, int V, float * __restrict__ logits, unsigned long long * __restrict__ best,
       const float * __restrict__ norm_w, float eps, int32_t * __restrict__ tokens, const HeadFeedback fb) {
    extern __shared__ __align__(16) float xs[];  // [nout][H]
    __shared__ float red[kHeadThreads / 32][kHeadMaxRows];
    __shared__ float inv_s[kHeadMaxRows];
    __shared__ unsigned last_s;
    pdl_trigger();
    pdl_wait_primary();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (norm_w) {
        const int nv = H / 4;
        float ss[kHeadMaxRows];
#pragma unroll
        for (int o = 0; o < kHeadMaxRows; ++o) {
            ss[o] = 0.f;
            if (o >= nout) continue;
            const float4 * hr = reinterpret_cast<const float4 *>(xn + size_t(rows[o]) * H);
            for (int e = threadIdx.x; e < nv; e += kHeadThreads) {
                const float4 x = hr[e];
                reinterpret_cast<float4 *>(xs)[o * nv + e] = x;
                ss[o] = fmaf(x.x, x.x, ss[o]);
                ss[o] = fmaf(x.y, x.y, ss[o]);
                ss[o] = fmaf(x.z, x.z, ss[o]);
                ss[o] = fmaf(x.w, x.w, ss[o]);
            }
        }
#pragma unroll
        for (int o = 0; o < kHeadMaxRows; ++o) {
            const float w = warp_sum(ss[o]);
            if (lane == 0) red[warp][o] = w;
        }
        __syncthreads();
        if (threadIdx.x < nout) {
            float t = 0.f;
            for (int w = 0; w < kHeadThreads / 32; ++w) t += red[w][threadIdx.x];  // warp order
            inv_s[threadIdx.x] = rsqrtf(t / float(H) + eps);
        }
        __syncthreads();
        const float4 * w4 = reinterpret_cast<const float4 *>(norm_w);
        for (int e = threadIdx.x; e < nout * nv; e += kHeadThreads) {
            const int o = e / nv;
            const float inv = inv_s[o];
            const float4 x = reinterpret_cast<float4 *>(xs)[e], wv = w4[e - o * nv];
            reinterpret_cast<float4 *>(xs)[e] = make_float4(x.x * inv * wv.x, x.y * inv * wv.y, x.z * inv * wv.z,
                                                            x.w * inv * wv.w);
        }
    } else {
        for (int e = threadIdx.x; e < nout * H / 4; e += kHeadThreads) {
            const int o = (e * 4) / H, i = (e * 4) % H;
            reinterpret_cast<float4 *>(xs)[e] = *reinterpret_cast<const float4 *>(xn + size_t(rows[o]) * H + i);
        }
    }
    __syncthreads();
    unsigned long long mine[kHeadMaxRows];
#pragma unroll
    for (int o = 0; o < kHeadMaxRows; ++o) mine[o] = 0ull;
    const int nwarps = gridDim.x * (kHeadThreads / 32);
    // one activation row: all of a vocab row's 16-byte loads in flight together
    if (nout == 1) {
        for (int v = blockIdx.x * (kHeadThreads / 32) + warp; v < V; v += nwarps) {
            const __half * er = E + size_t(v) * H + lane * 8;
            uint4 raw[ITER];
#pragma unroll
            for (int it = 0; it < ITER; ++it) raw[it] = __ldcs(reinterpret_cast<const uint4 *>(er + it * 256));
            float acc = 0.f;
#pragma unroll
            for (int it = 0; it < ITER; ++it) {
                const __half2 * e2 = reinterpret_cast<const __half2 *>(&raw[it]);
                const float4 * xr = reinterpret_cast<const float4 *>(xs + it * 256 + lane * 8);
                const float4 x0 = xr[0], x1 = xr[1];
                const float2 e0 = __half22float2(e2[0]), e1 = __half22float2(e2[1]);
                const float2 e2v = __half22float2(e2[2]), e3 = __half22float2(e2[3]);
                acc = fmaf(x0.x, e0.x, acc);
                acc = fmaf(x0.y, e0.y, acc);
                acc = fmaf(x0.z, e1.x, acc);
                acc = fmaf(x0.w, e1.y, acc);
                acc = fmaf(x1.x, e2v.x, acc);
                acc = fmaf(x1.y, e2v.y, acc);
                acc = fmaf(x1.z, e3.x, acc);
                acc = fmaf(x1.w, e3.y, acc);
            }
            const float s = warp_sum(acc);
            if (lane == 0) {
                if (logits) logits[v] = s;
                const unsigned long long key = (uint64_t(float_key(s)) << 32) | uint32_t(~uint32_t(v));
                mine[0] = key > mine[0] ? key : mine[0];
            }
        }
    } else {
        // 2..8 activation rows on the tensor cores: mma.m16n8k16, A = 16 vocab rows of E (fp16),
        // B = the activation rows as fp16 hi + lo (x - hi - lo is about 2^-22 x), fp32 sums.  A warp
        // takes 16 vocab rows at a time; per 64-wide k-block lane (g, t) loads k [8t, 8t + 8) and
        // [32 + 8t, 32 + 8t + 8) of vocab rows g and g + 8 (each load instruction reads whole 64-byte
        // row pieces), and k-step s pairs registers 2s, 2s+1 of those with activation row g at the
        // same k: the MMA sums over a permutation of the real k order, the same for A and B.  Lanes
        // of activation rows >= nout supply zeros.
        const int g = lane >> 2, t = lane & 3;
        unsigned long long cand[2] = {0ull, 0ull};  // best (key, ~v) of activation rows 2t, 2t + 1
        const int ngroups = (V + 15) / 16;
        for (int grp = blockIdx.x * (kHeadThreads / 32) + warp; grp < ngroups; grp += nwarps) {
            const int va = grp * 16 + g, vb = va + 8;
            const __half * ea = E + size_t(min(va, V - 1)) * H + 8 * t;
            const __half * eb = E + size_t(min(vb, V - 1)) * H + 8 * t;
            const float * xr = xs + size_t(g < nout ? g : 0) * H + 8 * t;
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            // double-buffered: the next k-block's table rows are in flight while this one's MMAs run
            auto load_kb = [&](int kb, uint4 (&r)[4]) {
                r[0] = __ldcs(reinterpret_cast<const uint4 *>(ea + kb * 64));
                r[1] = __ldcs(reinterpret_cast<const uint4 *>(ea + kb * 64 + 32));
                r[2] = __ldcs(reinterpret_cast<const uint4 *>(eb + kb * 64));
                r[3] = __ldcs(reinterpret_cast<const uint4 *>(eb + kb * 64 + 32));
            };
            const int nkb = H / 64;
            uint4 cur[4], nxt[4];
            load_kb(0, cur);
#pragma unroll 1
            for (int kb = 0; kb < nkb; ++kb) {
                if (kb + 1 < nkb) load_kb(kb + 1, nxt);
                const uint4 a0 = cur[0], a1 = cur[1], b0 = cur[2], b1 = cur[3];
                const uint32_t ra[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                const uint32_t rb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int st = 0; st < 4; ++st) {
                    float4 x = *reinterpret_cast<const float4 *>(xr + kb * 64 + 32 * (st >> 1) + 4 * (st & 1));
                    if (g >= nout) x = make_float4(0.f, 0.f, 0.f, 0.f);
                    const __half2 h01 = __floats2half2_rn(x.x, x.y), h23 = __floats2half2_rn(x.z, x.w);
                    const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
                    const __half2 l01 = __floats2half2_rn(x.x - f01.x, x.y - f01.y);
                    const __half2 l23 = __floats2half2_rn(x.z - f23.x, x.w - f23.y);
                    mma_f16_16816(d, ra[2 * st], rb[2 * st], ra[2 * st + 1], rb[2 * st + 1], h01, h23);
                    mma_f16_16816(d, ra[2 * st], rb[2 * st], ra[2 * st + 1], rb[2 * st + 1], l01, l23);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) cur[i] = nxt[i];
            }
            // d: (va, row 2t), (va, 2t + 1), (vb, 2t), (vb, 2t + 1)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int v = j < 2 ? va : vb, o = 2 * t + (j & 1);
                if (v >= V || o >= nout) continue;
                if (logits) logits[size_t(o) * V + v] = d[j];
                const unsigned long long key = (uint64_t(float_key(d[j])) << 32) | uint32_t(~uint32_t(v));
                cand[j & 1] = key > cand[j & 1] ? key : cand[j & 1];
            }
        }
        // the warp's best per activation row, into lane 0's mine[]
#pragma unroll
        for (int o = 0; o < kHeadMaxRows; ++o) {
            unsigned long long k = (o >> 1) == t ? cand[o & 1] : 0ull;
#pragma unroll
            for (int sh = 16; sh; sh >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, sh);
                k = other > k ? other : k;
            }
            if (lane == 0) mine[o] = k;
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int o = 0; o < kHeadMaxRows; ++o)
            if (o < nout) atomicMax(best + o, mine[o]);
        __threadfence();
    }
    __syncthreads();
    if (threadIdx.x == 0) last_s = atomicAdd(best + kHeadMaxRows, 1ull) == gridDim.x - 1;
    __syncthreads();
    if (!last_s) return;
    // the last CTA: every other CTA's maxima are in; read and clear them atomically
    __threadfence();
    if (threadIdx.x < nout) {
        const unsigned long long b = atomicExch(best + threadIdx.x, 0ull);
        const int32_t tok = int32_t(~uint32_t(b & 0xffffffffull));
        tokens[threadIdx.x] = tok;
        if (fb.next_tokens) {
            fb.next_tokens[threadIdx.x] = tok;
            fb.next_pos[threadIdx.x] += 1;
            fb.log[min(*fb.counter * nout + threadIdx.x, fb.log_cap - 1)] = tok;
        }
    }
    if (threadIdx.x == 0) atomicExch(best + kHeadMaxRows, 0ull);
    if (fb.next_tokens) {
        __syncthreads();  // every row has read the counter
        if (threadIdx.x == 0) *fb.counter += 1;
    }
}

}  // namespace

}  // namespace exl3cu

using namespace exl3cu;

namespace {

int status_of(cudaError_t e) {
    if (e == cudaSuccess) return EXL3CU_OK;
    (void)cudaGetLastError();
    return api_cuda_fail(e, "hybrid decoder kernel");
}

int bad(const char * what) { return api_fail(EXL3CU_INVALID_ARGUMENT, what); }

// Launch with programmatic stream serialization (the kernels wait for their
// predecessor with griddepcontrol.wait before touching memory).
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, void * stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    return status_of(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

// The same with a cluster of `cluster_x` CTAs along x.
template <typename... KArgs, typename... Args>
int launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, int cluster_x, void * stream,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = unsigned(cluster_x);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return status_of(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

// Per-device one-time kernel attributes.
bool set_smem_attr_once(const void * fn, int bytes, std::atomic<unsigned long long> & done_mask) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    const unsigned long long bit = 1ull << dev;
    if (done_mask.load() & bit) return true;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
    done_mask.fetch_or(bit);
    return true;
}

std::atomic<unsigned long long> g_gdn_attr{0}, g_gdn2_attr{0}, g_head_attr_4{0}, g_head_attr_8{0}, g_head_attr_16{0},
    g_head_attr_32{0};
constexpr int kHeadSmemMax = 200 * 1024;

}  // namespace

extern "C" {

int exl3cu_hyb_embed(const uint16_t * d_table, int vocab, const int32_t * d_ids, int rows, int hidden, float * d_h,
                     float * d_h_sumsq, void * stream) {
    if (!d_table || !d_ids || !d_h || rows < 0 || hidden <= 0 || vocab <= 0) return bad("embed: bad arguments");
    if (d_h_sumsq && (hidden % 128 || reinterpret_cast<uintptr_t>(d_h) % 16 || reinterpret_cast<uintptr_t>(d_table) % 8))
        return bad("embed: sums of squares need hidden a multiple of 128 and aligned rows");
    if (!rows) return EXL3CU_OK;
    return launch_pdl(k_embed, dim3(unsigned(rows)), dim3(256), 0, stream,
                      reinterpret_cast<const __half *>(d_table), d_ids, vocab, hidden, d_h, d_h_sumsq);
}

int exl3cu_hyb_rmsnorm(float * d_h, const float * d_delta, int delta_stride, const float * d_w, float eps, int rows,
                       int hidden, float * d_out, void * stream) {
    if (!d_h || !d_w || !d_out || rows < 0 || hidden <= 0 || hidden % 4 || hidden > 4 * kNormThreads * kNormMaxVec ||
        (d_delta && (delta_stride < hidden || delta_stride % 4)))
        return bad("rmsnorm: bad arguments (hidden a multiple of 4 up to 8192)");
    if (!rows) return EXL3CU_OK;
    return launch_pdl(k_rmsnorm, dim3(unsigned(rows)), dim3(kNormThreads), 0, stream, d_h, d_delta, delta_stride, d_w,
                      eps, hidden, d_out);
}

int exl3cu_hyb_swiglu(const float * d_gu, int rows, int ffn, float * d_out, void * stream) {
    if (!d_gu || !d_out || rows < 0 || ffn <= 0) return bad("swiglu: bad arguments");
    if (!rows) return EXL3CU_OK;
    return launch_pdl(k_swiglu, dim3(unsigned((ffn + 255) / 256), unsigned(rows)), dim3(256), 0, stream, d_gu, ffn,
                      d_out);
}

int exl3cu_hyb_attn_prep(const float * d_qkv, int rows, const int32_t * d_row_seq, const int32_t * d_row_pos,
                         const int32_t * d_seq_slot, const float * d_qn_w, const float * d_kn_w,
                         const float * d_inv_freq, float eps, uint16_t * d_kcache, uint16_t * d_vcache, int max_len,
                         int n_slots, float * d_q, void * stream) {
    if (!d_qkv || !d_row_seq || !d_row_pos || !d_seq_slot || !d_qn_w || !d_kn_w || !d_inv_freq || !d_kcache ||
        !d_vcache || !d_q || rows < 0 || max_len <= 0 || n_slots <= 0)
        return bad("attn_prep: bad arguments");
    if (!rows) return EXL3CU_OK;
    return launch_pdl(k_attn_prep, dim3(unsigned(rows)), dim3((kNH + kNKV) * 32), 0, stream, d_qkv, d_row_seq,
                      d_row_pos, d_seq_slot, d_qn_w, d_kn_w, d_inv_freq, eps, reinterpret_cast<__half *>(d_kcache),
                      reinterpret_cast<__half *>(d_vcache), max_len, n_slots, d_q);
}

size_t exl3cu_hyb_attn_scratch_bytes(int rows, int splits) {
    return rows <= 0 || splits <= 1 ? 0 : size_t(rows) * kNH * splits * kAttnPart * sizeof(float);
}

int exl3cu_hyb_attn(const float * d_q, int rows, const int32_t * d_row_seq, const int32_t * d_row_pos,
                    const int32_t * d_seq_slot, const uint16_t * d_kcache, const uint16_t * d_vcache, int max_len,
                    int n_slots, float scale, int splits, float * d_part, size_t part_bytes, unsigned * d_tickets,
                    float * d_out, void * stream) {
    if (!d_q || !d_row_seq || !d_row_pos || !d_seq_slot || !d_kcache || !d_vcache || !d_out || rows < 0 ||
        max_len <= 0 || n_slots <= 0 || splits < 1 || splits > 64)
        return bad("attn: bad arguments");
    if (!rows) return EXL3CU_OK;
    if (rows > 65535) return bad("attn: at most 65535 rows");
    if (splits > 1 && (!d_part || !d_tickets || part_bytes < exl3cu_hyb_attn_scratch_bytes(rows, splits)))
        return bad("attn: split scratch missing or too small (exl3cu_hyb_attn_scratch_bytes; tickets rows*16, zeroed)");
    if (reinterpret_cast<uintptr_t>(d_part) % 16) return bad("attn: split scratch must be 16-byte aligned");
    // the plain kernel only reads the caches
    __half * kc = reinterpret_cast<__half *>(const_cast<uint16_t *>(d_kcache));
    __half * vc = reinterpret_cast<__half *>(const_cast<uint16_t *>(d_vcache));
    return launch_pdl(k_attn<false>, dim3(kNH, unsigned(rows), unsigned(splits)), dim3(128), 0, stream, d_q,
                      d_row_seq, d_row_pos, d_seq_slot, kc, vc, max_len, n_slots, scale, d_part, d_tickets, d_out,
                      static_cast<const float *>(nullptr), static_cast<const float *>(nullptr),
                      static_cast<const float *>(nullptr), 0.f);
}

int exl3cu_hyb_attn_decode(const float * d_qkv, int rows, const int32_t * d_row_seq, const int32_t * d_row_pos,
                           const int32_t * d_seq_slot, const float * d_qn_w, const float * d_kn_w,
                           const float * d_inv_freq, float eps, uint16_t * d_kcache, uint16_t * d_vcache, int max_len,
                           int n_slots, float scale, int splits, float * d_part, size_t part_bytes,
                           unsigned * d_tickets, float * d_out, void * stream) {
    if (!d_qkv || !d_row_seq || !d_row_pos || !d_seq_slot || !d_qn_w || !d_kn_w || !d_inv_freq || !d_kcache ||
        !d_vcache || !d_out || rows < 0 || max_len <= 0 || n_slots <= 0 || splits < 1 || splits > 64)
        return bad("attn_decode: bad arguments");
    if (!rows) return EXL3CU_OK;
    if (rows > 65535) return bad("attn_decode: at most 65535 rows");
    if (splits > 1 && (!d_part || !d_tickets || part_bytes < exl3cu_hyb_attn_scratch_bytes(rows, splits)))
        return bad("attn_decode: split scratch missing or too small (exl3cu_hyb_attn_scratch_bytes; tickets rows*16, zeroed)");
    if (reinterpret_cast<uintptr_t>(d_part) % 16) return bad("attn_decode: split scratch must be 16-byte aligned");
    return launch_pdl(k_attn<true>, dim3(kNH, unsigned(rows), unsigned(splits)), dim3(128), 0, stream, d_qkv,
                      d_row_seq, d_row_pos, d_seq_slot, reinterpret_cast<__half *>(d_kcache),
                      reinterpret_cast<__half *>(d_vcache), max_len, n_slots, scale, d_part, d_tickets, d_out, d_qn_w,
                      d_kn_w, d_inv_freq, eps);
}

size_t exl3cu_hyb_gdn_smem_bytes_for(int hidden) {
    // fixed part and the fp16 gate rows (2 x hidden)
    return size_t(GdnSmem::floats_without_wab) * sizeof(float) + size_t(2 * hidden) * 2;
}

size_t exl3cu_hyb_gdn_smem_bytes(void) { return exl3cu_hyb_gdn_smem_bytes_for(8192); }

int exl3cu_hyb_gdn(const float * d_qkvz, const float * d_xn, const float * d_xn_norm_w, const uint16_t * d_wab,
                   int hidden,
                   const float * d_conv_w, float * d_conv_state, const float * d_A_log, const float * d_dt_bias,
                   const float * d_norm_w, float eps, float * d_state, const int32_t * d_row_offsets,
                   const int32_t * d_seq_slot, int n_seq, int n_slots, float * d_out, void * stream) {
    if (!d_qkvz || !d_xn || !d_wab || !d_conv_w || !d_conv_state || !d_A_log || !d_dt_bias || !d_norm_w ||
        !d_state || !d_row_offsets || !d_seq_slot || !d_out || hidden <= 0 || n_seq < 0 || n_seq > 65535 ||
        n_slots <= 0)
        return bad("gdn: bad arguments");
    if (reinterpret_cast<uintptr_t>(d_state) % 16) return bad("gdn: state must be 16-byte aligned");
    if (hidden > 8192 || hidden % 8) return bad("gdn: hidden must be a multiple of 8 up to 8192");
    if (!n_seq) return EXL3CU_OK;
    const size_t smem = exl3cu_hyb_gdn_smem_bytes_for(hidden);
    const bool few = n_seq <= 2;
    const void * kfn = few ? reinterpret_cast<const void *>(k_gdn<1>) : reinterpret_cast<const void *>(k_gdn<2>);
    if (!set_smem_attr_once(kfn, int(exl3cu_hyb_gdn_smem_bytes()), few ? g_gdn_attr : g_gdn2_attr))
        return status_of(cudaGetLastError());
    return launch_pdl_cluster(few ? k_gdn<1> : k_gdn<2>, dim3(kNH * kGdnSplit, unsigned(n_seq)), dim3(kGdnThreads),
                      smem, kGdnSplit, stream, d_qkvz, d_xn, d_xn_norm_w,
                      reinterpret_cast<const __half *>(d_wab), hidden,
                      d_conv_w, d_conv_state, d_A_log, d_dt_bias, d_norm_w, eps, d_state, d_row_offsets, d_seq_slot,
                      n_slots, d_out);
}

}  // extern "C"

namespace {

int head_launch(const float * d_xn, const int32_t * d_rows, int nout, int hidden, const float * d_norm_w, float eps,
                const uint16_t * d_embed, int vocab, float * d_logits, unsigned long long * d_best, int32_t * d_tokens,
                const HeadFeedback & fb, void * stream) {
    if (!d_xn || !d_rows || !d_embed || !d_best || !d_tokens || nout < 0 || nout > kHeadMaxRows || hidden <= 0 ||
        hidden % 256 || hidden > 8192 || vocab <= 0)
        return bad("head: bad arguments (nout <= 8, hidden a multiple of 256 up to 8192)");
    if (d_norm_w && reinterpret_cast<uintptr_t>(d_norm_w) % 16) return bad("head: norm weights must be 16-byte aligned");
    if (!nout) return EXL3CU_OK;
    const size_t smem = size_t(nout) * hidden * sizeof(float);
    if (smem > size_t(kHeadSmemMax)) return bad("head: activations exceed shared memory");
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int rc = 0;
    // CTAs that are resident together: four per SM, fewer when the staged rows fill shared memory
    const int per_sm = std::max(1, std::min(4, int((200 * 1024) / std::max<size_t>(smem, 1))));
    const dim3 grid(unsigned(sms * per_sm)), block(kHeadThreads);
    const float * xn = d_xn;
    const auto * E = reinterpret_cast<const __half *>(d_embed);
    switch (hidden / 256) {
#define EXL3CU_HEAD_CASE(N)                                                                                        \
    case N:                                                                                                        \
        if (!set_smem_attr_once(reinterpret_cast<const void *>(k_head<N>), kHeadSmemMax, g_head_attr_##N))        \
            return status_of(cudaGetLastError());                                                                  \
        rc = launch_pdl(k_head<N>, grid, block, smem, stream, xn, d_rows, nout, hidden, E, vocab, d_logits, d_best, \
                        d_norm_w, eps, d_tokens, fb);                                                              \
        break;
        EXL3CU_HEAD_CASE(4)
        EXL3CU_HEAD_CASE(8)
        EXL3CU_HEAD_CASE(16)
        EXL3CU_HEAD_CASE(32)
#undef EXL3CU_HEAD_CASE
        default:
            return bad("head: hidden must be 1024, 2048, 4096 or 8192");
    }
    return rc;
}

}  // namespace

extern "C" {

int exl3cu_hyb_head(const float * d_xn, const int32_t * d_rows, int nout, int hidden, const float * d_norm_w,
                    float eps, const uint16_t * d_embed, int vocab, float * d_logits, unsigned long long * d_best,
                    int32_t * d_tokens, void * stream) {
    return head_launch(d_xn, d_rows, nout, hidden, d_norm_w, eps, d_embed, vocab, d_logits, d_best, d_tokens,
                       HeadFeedback{nullptr, nullptr, nullptr, nullptr, 0}, stream);
}

int exl3cu_hyb_head_feedback(const float * d_xn, const int32_t * d_rows, int nout, int hidden, const float * d_norm_w,
                             float eps, const uint16_t * d_embed, int vocab, unsigned long long * d_best,
                             int32_t * d_tokens, int32_t * d_next_tokens, int32_t * d_next_pos, int32_t * d_log,
                             int64_t * d_counter, size_t log_capacity, void * stream) {
    if (!d_next_tokens || !d_next_pos || !d_log || !d_counter || log_capacity == 0)
        return bad("head_feedback: the feedback buffers must be given (log_capacity >= 1)");
    return head_launch(d_xn, d_rows, nout, hidden, d_norm_w, eps, d_embed, vocab, nullptr, d_best, d_tokens,
                       HeadFeedback{d_next_tokens, d_next_pos, d_log, reinterpret_cast<long long *>(d_counter),
                                    static_cast<long long>(log_capacity)},
                       stream);
}

int exl3cu_hyb_status(int clear, unsigned * status) {
    if (!status) return bad("status is NULL");
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(status, g_hyb_status, sizeof(unsigned));
    if (e == cudaSuccess && clear && *status) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(g_hyb_status, &zero, sizeof(unsigned));
    }
    return status_of(e);
}

}  // extern "C"
