// Device kernels of the hybrid decoder around the EXL3 operator: the layers a
// Qwen3.5-style 3:1 gated-delta-rule / full-attention decoder runs between its
// packed matmuls (embedding, residual + RMSNorm, SwiGLU, q/k norm + RoPE + FP16
// KV append, GQA attention, the gated delta rule with its short convolution
// and gates, the tied fp16 head with a fused argmax).
//
// Rows are the packed tokens of one scheduler step (exl3cu_pack_ragged's
// output): row r belongs to step sequence row_seq[r] at position row_pos[r];
// step sequence s owns cache slot seq_slot[s] and the rows
// [row_offsets[s], row_offsets[s+1]).  All arithmetic is fp32; activations
// that feed a packed matmul are rounded to fp16 (the operator's input type),
// the KV cache is fp16, the residual stream and recurrent state are fp32.
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
#include "exl3cu.h"
#include "exl3cu_hybrid.h"
#include "exl3cu_internal.h"

#include <cuda_fp16.h>

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

__global__ void k_embed(const __half * __restrict__ table, const int32_t * __restrict__ ids, int vocab, int H,
                        float * __restrict__ h) {
    const int r = blockIdx.x;
    const int32_t id = ids[r];
    const bool ok = id >= 0 && id < vocab;  // an id outside the table gives a zero row
    for (int i = threadIdx.x; i < H; i += blockDim.x)
        h[size_t(r) * H + i] = ok ? __half2float(table[size_t(id) * H + i]) : 0.f;
}

// h += delta (when given), then out = fp16(h / sqrt(mean(h^2) + eps) * w).  One CTA per row.
__global__ void k_rmsnorm(float * __restrict__ h, const float * __restrict__ delta, int delta_stride,
                          const float * __restrict__ w, float eps, int H, __half * __restrict__ out) {
    __shared__ float red[32];
    const int r = blockIdx.x;
    float * hr = h + size_t(r) * H;
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        float v = hr[i];
        if (delta) {
            v += delta[size_t(r) * delta_stride + i];
            hr[i] = v;
        }
        ss = fmaf(v, v, ss);
    }
    const float tot = block_sum(ss, red, blockDim.x >> 5);
    const float inv = rsqrtf(tot / float(H) + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x)
        out[size_t(r) * H + i] = __float2half_rn(hr[i] * inv * w[i]);
}

// out = fp16(silu(gate) * up); gu row = [gate (F) | up (F)].
__global__ void k_swiglu(const float * __restrict__ gu, int F, __half * __restrict__ out) {
    const int r = blockIdx.y;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= F) return;
    const float g = gu[size_t(r) * 2 * F + i], u = gu[size_t(r) * 2 * F + F + i];
    out[size_t(r) * F + i] = __float2half_rn(silu(g) * u);
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
    const float * wn = is_q ? qn_w : kn_w;
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = x[lane + 32 * q];  // dims lane, lane+32, lane+64, lane+96
    float ss = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) ss = fmaf(v[q], v[q], ss);
    const float inv = rsqrtf(warp_sum(ss) / float(kHD) + eps);
#pragma unroll
    for (int q = 0; q < 4; ++q) v[q] = v[q] * inv * wn[lane + 32 * q];
    float o[4];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const int i = lane + 32 * q;  // first-half index; partner i + 64
        float sn, cs;
        sincosf(float(pos) * inv_freq[i], &sn, &cs);
        o[q] = v[q] * cs - v[q + 2] * sn;
        o[q + 2] = v[q + 2] * cs + v[q] * sn;
    }
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

// softmax(q K^T * scale) V over positions 0..pos of the row's sequence, one
// CTA (4 warps) per (q head, row); warp w takes positions w, w+4, ...; lane
// holds 4 consecutive dims.  Online softmax per warp, merged in fixed order.
__global__ void k_attn(const float * __restrict__ q, const int32_t * __restrict__ row_seq,
                       const int32_t * __restrict__ row_pos, const int32_t * __restrict__ seq_slot,
                       const __half * __restrict__ kc, const __half * __restrict__ vc, int max_len, int n_slots,
                       float scale, __half * __restrict__ out) {
    __shared__ float sm_m[4], sm_l[4], sm_acc[4][kHD];
    const int head = blockIdx.x, r = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slot = seq_slot[row_seq[r]];
    if (slot < 0 || slot >= n_slots) return;
    const int pos = min(row_pos[r], max_len - 1);
    const int kvh = head / (kNH / kNKV);
    const float4 qv = *reinterpret_cast<const float4 *>(q + size_t(r) * kNH * kHD + head * kHD + lane * 4);
    const __half * kb = kc + (size_t(slot) * kNKV + kvh) * max_len * kHD;
    const __half * vb = vc + (size_t(slot) * kNKV + kvh) * max_len * kHD;
    float m = -INFINITY, l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int p = warp; p <= pos; p += 4) {
        const uint2 kr = *reinterpret_cast<const uint2 *>(kb + size_t(p) * kHD + lane * 4);
        const float2 k01 = __half22float2(*reinterpret_cast<const __half2 *>(&kr.x));
        const float2 k23 = __half22float2(*reinterpret_cast<const __half2 *>(&kr.y));
        float s = qv.x * k01.x;
        s = fmaf(qv.y, k01.y, s);
        s = fmaf(qv.z, k23.x, s);
        s = fmaf(qv.w, k23.y, s);
        s = warp_sum(s) * scale;
        const float mn = fmaxf(m, s);
        const float corr = expf(m - mn), e = expf(s - mn);
        const uint2 vr = *reinterpret_cast<const uint2 *>(vb + size_t(p) * kHD + lane * 4);
        const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vr.x));
        const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vr.y));
        l = l * corr + e;
        acc[0] = fmaf(e, v01.x, acc[0] * corr);
        acc[1] = fmaf(e, v01.y, acc[1] * corr);
        acc[2] = fmaf(e, v23.x, acc[2] * corr);
        acc[3] = fmaf(e, v23.y, acc[3] * corr);
        m = mn;
    }
    if (lane == 0) {
        sm_m[warp] = m;
        sm_l[warp] = l;
    }
#pragma unroll
    for (int q2 = 0; q2 < 4; ++q2) sm_acc[warp][lane * 4 + q2] = acc[q2];
    __syncthreads();
    if (warp == 0) {
        float M = -INFINITY;
        for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_m[w]);
        float L = 0.f, a[4] = {0.f, 0.f, 0.f, 0.f};
        for (int w = 0; w < 4; ++w) {
            if (sm_m[w] == -INFINITY) continue;  // a warp that saw no position
            const float c = expf(sm_m[w] - M);
            L = fmaf(sm_l[w], c, L);
#pragma unroll
            for (int q2 = 0; q2 < 4; ++q2) a[q2] = fmaf(sm_acc[w][lane * 4 + q2], c, a[q2]);
        }
        const float invL = 1.0f / L;
#pragma unroll
        for (int q2 = 0; q2 < 4; ++q2)
            out[size_t(r) * kNH * kHD + head * kHD + lane * 4 + q2] = __float2half_rn(a[q2] * invL);
    }
}

// Gated delta rule for one (head, step sequence): the sequence's rows in
// order.  256 threads; the head's 128 x 128 fp32 state lives in shared memory
// for the CTA's lifetime (loaded from and stored back to S).  Thread t: v
// column j = t & 127, k half = t >> 7.
constexpr int kGdnThreads = 256;

__global__ void __launch_bounds__(kGdnThreads)
k_gdn(const float * __restrict__ qkvz, const __half * __restrict__ xn, const __half * __restrict__ wab, int H,
      const float * __restrict__ conv_w, float * __restrict__ conv_state, const float * __restrict__ A_log,
      const float * __restrict__ dt_bias, const float * __restrict__ norm_w, float eps, float * __restrict__ S,
      const int32_t * __restrict__ row_offsets, const int32_t * __restrict__ seq_slot, int n_slots,
      __half * __restrict__ out) {
    extern __shared__ __align__(16) float sm[];
    float * St = sm;                          // [128 k][128 v]
    float * cq = St + kHD * kHD;              // conv outputs q, k, v of the current row
    float * ck = cq + kHD;
    float * cv = ck + kHD;
    float * red = cv + kHD;                   // [4][128]: k-half sums of S^T k and S^T q; then o
    float * scal = red + 4 * kHD;             // [32]: per-warp gate sums, alpha, beta
    const int h = blockIdx.x, s = blockIdx.y;
    const int slot = seq_slot[s];
    if (slot < 0 || slot >= n_slots) return;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int j = t & (kHD - 1), half = t >> 7;
    float * Sg = S + (size_t(slot) * kNH + h) * kHD * kHD;
    for (int e = t; e < kHD * kHD / 4; e += kGdnThreads)
        reinterpret_cast<float4 *>(St)[e] = reinterpret_cast<const float4 *>(Sg)[e];
    const int r0 = row_offsets[s], r1 = row_offsets[s + 1];
    constexpr int QKVZ = 4 * kNH * kHD;
    constexpr int CH = 3 * kNH * kHD;  // convolved channels (q, k, v)
    const float A = -expf(A_log[h]);
    const float qscale = rsqrtf(float(kHD));
    __syncthreads();
    for (int r = r0; r < r1; ++r) {
        // (1) causal conv + SiLU on this head's 384 channels; the conv state keeps the last 3 inputs
        for (int c = t; c < 3 * kHD; c += kGdnThreads) {
            const int part = c / kHD, d = c % kHD;                // 0 q, 1 k, 2 v
            const int ch = part * kNH * kHD + h * kHD + d;        // channel in [0, CH)
            const float x = qkvz[size_t(r) * QKVZ + ch];
            float * st = conv_state + (size_t(slot) * CH + ch) * (kConvW - 1);
            const float * wc = conv_w + size_t(ch) * kConvW;
            float acc = st[0] * wc[0];
            acc = fmaf(st[1], wc[1], acc);
            acc = fmaf(st[2], wc[2], acc);
            acc = fmaf(x, wc[3], acc);
            st[0] = st[1];
            st[1] = st[2];
            st[2] = x;
            (part == 0 ? cq : part == 1 ? ck : cv)[d] = silu(acc);
        }
        // (2) the gates' projections a = x . W_a[h], b = x . W_b[h] (fp16 x and weights, fp32 sums)
        float pa = 0.f, pb = 0.f;
        for (int i = t; i < H; i += kGdnThreads) {
            const float x = __half2float(xn[size_t(r) * H + i]);
            pa = fmaf(x, __half2float(wab[size_t(h) * H + i]), pa);
            pb = fmaf(x, __half2float(wab[size_t(kNH + h) * H + i]), pb);
        }
        pa = warp_sum(pa);
        pb = warp_sum(pb);
        __syncthreads();  // conv outputs complete; scal free
        if (lane == 0) {
            scal[warp] = pa;
            scal[8 + warp] = pb;
        }
        __syncthreads();
        // (3) L2 norms of q and k (warp 0: q, warp 1: k), gates (thread 64)
        if (warp < 2) {
            float * vec = warp == 0 ? cq : ck;
            float ss = 0.f;
            for (int d = lane; d < kHD; d += 32) ss = fmaf(vec[d], vec[d], ss);
            const float inv = rsqrtf(warp_sum(ss) + 1e-6f) * (warp == 0 ? qscale : 1.0f);
            for (int d = lane; d < kHD; d += 32) vec[d] *= inv;
        } else if (t == 64) {
            float a = 0.f, b = 0.f;
            for (int w = 0; w < 8; ++w) {
                a += scal[w];
                b += scal[8 + w];
            }
            scal[16] = expf(A * softplus(a + dt_bias[h]));  // alpha
            scal[17] = 1.0f / (1.0f + expf(-b));              // beta
        }
        __syncthreads();
        const float alpha = scal[16], beta = scal[17];
        // (4) a_j = sum_i S[i][j] k[i], c_j = sum_i S[i][j] q[i] over this thread's k half
        float ak = 0.f, cqs = 0.f;
        const int i0 = half * (kHD / 2);
#pragma unroll 8
        for (int i = i0; i < i0 + kHD / 2; ++i) {
            const float sv = St[i * kHD + j];
            ak = fmaf(sv, ck[i], ak);
            cqs = fmaf(sv, cq[i], cqs);
        }
        red[half * kHD + j] = ak;
        red[2 * kHD + half * kHD + j] = cqs;
        __syncthreads();
        float kq = 0.f;
        for (int i = 0; i < kHD; ++i) kq = fmaf(ck[i], cq[i], kq);  // every thread, same order
        const float a_j = red[j] + red[kHD + j];
        const float c_j = red[2 * kHD + j] + red[3 * kHD + j];
        const float u_j = beta * (cv[j] - alpha * a_j);
        const float o_j = fmaf(kq, u_j, alpha * c_j);
        // (5) S = alpha S + k u^T on this thread's half
#pragma unroll 8
        for (int i = i0; i < i0 + kHD / 2; ++i) St[i * kHD + j] = fmaf(ck[i], u_j, alpha * St[i * kHD + j]);
        // (6) RMSNorm of o over the head, times norm_w, gated by SiLU(z)
        __syncthreads();  // red reused
        if (half == 0) red[j] = o_j;
        __syncthreads();
        if (warp == 0) {
            float ss = 0.f;
            for (int d = lane; d < kHD; d += 32) ss = fmaf(red[d], red[d], ss);
            const float inv = rsqrtf(warp_sum(ss) / float(kHD) + eps);
            for (int d = lane; d < kHD; d += 32) {
                const float z = qkvz[size_t(r) * QKVZ + 3 * kNH * kHD + h * kHD + d];
                out[size_t(r) * kNH * kHD + h * kHD + d] = __float2half_rn(red[d] * inv * norm_w[d] * silu(z));
            }
        }
        __syncthreads();
    }
    for (int e = t; e < kHD * kHD / 4; e += kGdnThreads)
        reinterpret_cast<float4 *>(Sg)[e] = reinterpret_cast<const float4 *>(St)[e];
}

// Order-preserving key of a float (larger float, larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// logits[o][v] = sum_i xn[rows[o]][i] * E[v][i] (fp16 inputs, fp32 sums) for
// nout <= 8 rows; best[o] = max over v of (key(logit) << 32 | ~v) (the first
// index wins ties).  Warp per vocab row, activations staged in shared memory.
constexpr int kHeadMaxRows = 8;
constexpr int kHeadThreads = 256;

__global__ void __launch_bounds__(kHeadThreads)
k_head(const __half * __restrict__ xn, const int32_t * __restrict__ rows, int nout, int H,
       const __half * __restrict__ E, int V, float * __restrict__ logits, unsigned long long * __restrict__ best) {
    extern __shared__ __align__(16) __half xs[];  // [nout][H]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < nout * H / 8; e += kHeadThreads) {
        const int o = (e * 8) / H, i = (e * 8) % H;
        reinterpret_cast<uint4 *>(xs)[e] = *reinterpret_cast<const uint4 *>(xn + size_t(rows[o]) * H + i);
    }
    __syncthreads();
    unsigned long long mine[kHeadMaxRows];
#pragma unroll
    for (int o = 0; o < kHeadMaxRows; ++o) mine[o] = 0ull;
    const int nwarps = gridDim.x * (kHeadThreads / 32);
    for (int v = blockIdx.x * (kHeadThreads / 32) + warp; v < V; v += nwarps) {
        float acc[kHeadMaxRows];
#pragma unroll
        for (int o = 0; o < kHeadMaxRows; ++o) acc[o] = 0.f;
        const __half * er = E + size_t(v) * H;
        for (int i = lane * 8; i < H; i += 256) {
            const uint4 raw = *reinterpret_cast<const uint4 *>(er + i);
            const __half2 * e2 = reinterpret_cast<const __half2 *>(&raw);
            float2 ef[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) ef[q] = __half22float2(e2[q]);
#pragma unroll
            for (int o = 0; o < kHeadMaxRows; ++o) {
                if (o >= nout) break;
                const uint4 xr = *reinterpret_cast<const uint4 *>(xs + o * H + i);
                const __half2 * x2 = reinterpret_cast<const __half2 *>(&xr);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 xf = __half22float2(x2[q]);
                    acc[o] = fmaf(xf.x, ef[q].x, acc[o]);
                    acc[o] = fmaf(xf.y, ef[q].y, acc[o]);
                }
            }
        }
#pragma unroll
        for (int o = 0; o < kHeadMaxRows; ++o) {
            if (o >= nout) break;
            const float s = warp_sum(acc[o]);
            if (lane == 0) {
                if (logits) logits[size_t(o) * V + v] = s;
                const unsigned long long key = (uint64_t(float_key(s)) << 32) | uint32_t(~uint32_t(v));
                mine[o] = key > mine[o] ? key : mine[o];
            }
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int o = 0; o < kHeadMaxRows; ++o)
            if (o < nout) atomicMax(best + o, mine[o]);
    }
}

__global__ void k_head_tokens(const unsigned long long * __restrict__ best, int nout, int32_t * __restrict__ tokens) {
    const int o = threadIdx.x;
    if (o < nout) tokens[o] = int32_t(~uint32_t(best[o] & 0xffffffffull));
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

}  // namespace

extern "C" {

int exl3cu_hyb_embed(const uint16_t * d_table, int vocab, const int32_t * d_ids, int rows, int hidden, float * d_h,
                     void * stream) {
    if (!d_table || !d_ids || !d_h || rows < 0 || hidden <= 0 || vocab <= 0) return bad("embed: bad arguments");
    if (!rows) return EXL3CU_OK;
    k_embed<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(reinterpret_cast<const __half *>(d_table), d_ids,
                                                                  vocab, hidden, d_h);
    return status_of(cudaGetLastError());
}

int exl3cu_hyb_rmsnorm(float * d_h, const float * d_delta, int delta_stride, const float * d_w, float eps, int rows,
                       int hidden, uint16_t * d_out, void * stream) {
    if (!d_h || !d_w || !d_out || rows < 0 || hidden <= 0 || (d_delta && delta_stride < hidden))
        return bad("rmsnorm: bad arguments");
    if (!rows) return EXL3CU_OK;
    k_rmsnorm<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(d_h, d_delta, delta_stride, d_w, eps, hidden,
                                                                    reinterpret_cast<__half *>(d_out));
    return status_of(cudaGetLastError());
}

int exl3cu_hyb_swiglu(const float * d_gu, int rows, int ffn, uint16_t * d_out, void * stream) {
    if (!d_gu || !d_out || rows < 0 || ffn <= 0) return bad("swiglu: bad arguments");
    if (!rows) return EXL3CU_OK;
    const dim3 grid(unsigned((ffn + 255) / 256), unsigned(rows));
    k_swiglu<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(d_gu, ffn, reinterpret_cast<__half *>(d_out));
    return status_of(cudaGetLastError());
}

int exl3cu_hyb_attn_prep(const float * d_qkv, int rows, const int32_t * d_row_seq, const int32_t * d_row_pos,
                         const int32_t * d_seq_slot, const float * d_qn_w, const float * d_kn_w,
                         const float * d_inv_freq, float eps, uint16_t * d_kcache, uint16_t * d_vcache, int max_len,
                         int n_slots, float * d_q, void * stream) {
    if (!d_qkv || !d_row_seq || !d_row_pos || !d_seq_slot || !d_qn_w || !d_kn_w || !d_inv_freq || !d_kcache ||
        !d_vcache || !d_q || rows < 0 || max_len <= 0 || n_slots <= 0)
        return bad("attn_prep: bad arguments");
    if (!rows) return EXL3CU_OK;
    k_attn_prep<<<rows, (kNH + kNKV) * 32, 0, static_cast<cudaStream_t>(stream)>>>(
        d_qkv, d_row_seq, d_row_pos, d_seq_slot, d_qn_w, d_kn_w, d_inv_freq, eps, reinterpret_cast<__half *>(d_kcache),
        reinterpret_cast<__half *>(d_vcache), max_len, n_slots, d_q);
    return status_of(cudaGetLastError());
}

int exl3cu_hyb_attn(const float * d_q, int rows, const int32_t * d_row_seq, const int32_t * d_row_pos,
                    const int32_t * d_seq_slot, const uint16_t * d_kcache, const uint16_t * d_vcache, int max_len,
                    int n_slots, float scale, uint16_t * d_out, void * stream) {
    if (!d_q || !d_row_seq || !d_row_pos || !d_seq_slot || !d_kcache || !d_vcache || !d_out || rows < 0 ||
        max_len <= 0 || n_slots <= 0)
        return bad("attn: bad arguments");
    if (!rows) return EXL3CU_OK;
    if (rows > 65535) return bad("attn: at most 65535 rows");
    const dim3 grid(kNH, unsigned(rows));
    k_attn<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(d_q, d_row_seq, d_row_pos, d_seq_slot,
                                                                 reinterpret_cast<const __half *>(d_kcache),
                                                                 reinterpret_cast<const __half *>(d_vcache), max_len,
                                                                 n_slots, scale, reinterpret_cast<__half *>(d_out));
    return status_of(cudaGetLastError());
}

size_t exl3cu_hyb_gdn_smem_bytes(void) { return size_t(kHD * kHD + 3 * kHD + 4 * kHD + 32) * sizeof(float); }

int exl3cu_hyb_gdn(const float * d_qkvz, const uint16_t * d_xn, const uint16_t * d_wab, int hidden,
                   const float * d_conv_w, float * d_conv_state, const float * d_A_log, const float * d_dt_bias,
                   const float * d_norm_w, float eps, float * d_state, const int32_t * d_row_offsets,
                   const int32_t * d_seq_slot, int n_seq, int n_slots, uint16_t * d_out, void * stream) {
    if (!d_qkvz || !d_xn || !d_wab || !d_conv_w || !d_conv_state || !d_A_log || !d_dt_bias || !d_norm_w ||
        !d_state || !d_row_offsets || !d_seq_slot || !d_out || hidden <= 0 || n_seq < 0 || n_seq > 65535 ||
        n_slots <= 0)
        return bad("gdn: bad arguments");
    if (!n_seq) return EXL3CU_OK;
    static bool attr_set = false;
    const size_t smem = exl3cu_hyb_gdn_smem_bytes();
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(k_gdn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return status_of(e);
        attr_set = true;
    }
    const dim3 grid(kNH, unsigned(n_seq));
    k_gdn<<<grid, kGdnThreads, smem, static_cast<cudaStream_t>(stream)>>>(
        d_qkvz, reinterpret_cast<const __half *>(d_xn), reinterpret_cast<const __half *>(d_wab), hidden, d_conv_w,
        d_conv_state, d_A_log, d_dt_bias, d_norm_w, eps, d_state, d_row_offsets, d_seq_slot, n_slots,
        reinterpret_cast<__half *>(d_out));
    return status_of(cudaGetLastError());
}

int exl3cu_hyb_head(const uint16_t * d_xn, const int32_t * d_rows, int nout, int hidden, const uint16_t * d_embed,
                    int vocab, float * d_logits, unsigned long long * d_best, int32_t * d_tokens, void * stream) {
    if (!d_xn || !d_rows || !d_embed || !d_best || !d_tokens || nout < 0 || nout > kHeadMaxRows || hidden <= 0 ||
        hidden % 256 || vocab <= 0)
        return bad("head: bad arguments (nout <= 8, hidden a multiple of 256)");
    if (!nout) return EXL3CU_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(d_best, 0, sizeof(unsigned long long) * size_t(nout), st);
    if (e != cudaSuccess) return status_of(e);
    const size_t smem = size_t(nout) * hidden * sizeof(__half);
    static bool attr_set = false;
    if (!attr_set) {
        e = cudaFuncSetAttribute(k_head, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return status_of(e);
        attr_set = true;
    }
    if (smem > 200 * 1024) return bad("head: activations exceed shared memory");
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    k_head<<<sms * 4, kHeadThreads, smem, st>>>(reinterpret_cast<const __half *>(d_xn), d_rows, nout, hidden,
                                                reinterpret_cast<const __half *>(d_embed), vocab, d_logits, d_best);
    e = cudaGetLastError();
    if (e != cudaSuccess) return status_of(e);
    k_head_tokens<<<1, 32, 0, st>>>(d_best, nout, d_tokens);
    return status_of(cudaGetLastError());
}

}  // extern "C"
