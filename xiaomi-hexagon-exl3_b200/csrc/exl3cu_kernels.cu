// Codec kernels: codebook evaluation, ring-layout tile decode (decode_inner),
// device-layout conversion (runtime records / upstream trellis -> LSC), LSC
// decode, Hadamard-128 and original-basis reconstruction.
//
// These back the exl3_codec.h host API (reference include/exl3_codec.h:10-29)
// and the weight upload path; the GEMV hot loop lives in exl3cu_gemv.cu.
#include "exl3cu_async.cuh"
#include "exl3cu_internal.h"

namespace exl3cu {

// ---------------------------------------------------------------------------
// Codebook over an arbitrary state list (exhaustive-test entry; the same
// decode_pair code the GEMV uses).  Reference: src/exl3_codec.cpp:68-86.
__global__ void k_codebook(const uint16_t * __restrict__ states, size_t count, unsigned cb,
                           uint16_t * __restrict__ out) {
    const size_t i = (size_t(blockIdx.x) * blockDim.x + threadIdx.x) * 2;
    if (i >= count) return;
    const uint32_t s0 = states[i];
    const uint32_t s1 = (i + 1 < count) ? states[i + 1] : 0u;
    const uint32_t r = decode_pair_rt(s0, s1, cb);
    out[i] = uint16_t(r & 0xffffu);
    if (i + 1 < count) out[i + 1] = uint16_t(r >> 16);
}

// ---------------------------------------------------------------------------
// decode_inner on the upstream ring layout trellis[k/16][n/16][16*bits]
// (src/exl3_codec.cpp:92-145).  One warp per 16x16 tile: lane L decodes
// positions 8L..8L+7, whose windows cover ring bits
// [8*bits*L + bits - 16, 8*bits*L + 8*bits) -- at most 72 bits, so four ring
// words starting at the word of the first bit always hold them.
__device__ __forceinline__ uint32_t ring_word(const uint16_t * tile, unsigned i) {
    const uint32_t lo = tile[2 * i], hi = tile[2 * i + 1];
    return lo | (hi << 16);
}

__device__ __forceinline__ void decode_ring_tile_lane(const uint16_t * __restrict__ tile, unsigned bits, unsigned cb,
                                                      uint32_t (&frag)[4]) {
    const unsigned lane = threadIdx.x & 31u;
    const unsigned ring = 256u * bits;
    const unsigned nwords = 8u * bits;
    const unsigned first = (8u * bits * lane + bits + ring - 16u) % ring;  // first window's start bit
    const unsigned w0 = first >> 5;
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = ring_word(tile, (w0 + i) % nwords);
    uint32_t s[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const unsigned start = (first + unsigned(e) * bits) % ring;
        const unsigned rel = (start + ring - 32u * w0) % ring;  // 0..~103 inside w[]
        const unsigned i = rel >> 5, o = rel & 31u;  // i is 0, 1 or 2
        const uint32_t a = i == 0 ? w[0] : (i == 1 ? w[1] : w[2]);
        const uint32_t b = i == 0 ? w[1] : (i == 1 ? w[2] : w[3]);
        s[e] = (o <= 16u) ? ((a >> (16u - o)) & 0xffffu) : (__funnelshift_l(b, a, o - 16u) & 0xffffu);
    }
    frag[0] = decode_pair_rt(s[0], s[1], cb);
    frag[1] = decode_pair_rt(s[4], s[5], cb);
    frag[2] = decode_pair_rt(s[2], s[3], cb);
    frag[3] = decode_pair_rt(s[6], s[7], cb);
}

// Write one warp's tile (mma A-fragment of W^T) as rows of a row-major fp16
// matrix: transpose through shared memory so each lane stores 16 bytes.
__device__ __forceinline__ void store_tile_rowmajor(const uint32_t (&frag)[4], uint16_t * smem_tile,
                                                    uint16_t * __restrict__ out, size_t ld) {
    const unsigned lane = threadIdx.x & 31u;
    const unsigned g = lane >> 2, t = lane & 3u;
    // frag[0] = {e0,e1}: rows 2t,2t+1 col g; frag[2] = {e2,e3}: rows 2t+8,2t+9 col g;
    // frag[1] = {e4,e5}: rows 2t,2t+1 col g+8; frag[3] = {e6,e7}: rows 2t+8,2t+9 col g+8.
    const unsigned r0 = 2u * t;
    smem_tile[(r0 + 0) * 16 + g] = uint16_t(frag[0]);
    smem_tile[(r0 + 1) * 16 + g] = uint16_t(frag[0] >> 16);
    smem_tile[(r0 + 8) * 16 + g] = uint16_t(frag[2]);
    smem_tile[(r0 + 9) * 16 + g] = uint16_t(frag[2] >> 16);
    smem_tile[(r0 + 0) * 16 + g + 8] = uint16_t(frag[1]);
    smem_tile[(r0 + 1) * 16 + g + 8] = uint16_t(frag[1] >> 16);
    smem_tile[(r0 + 8) * 16 + g + 8] = uint16_t(frag[3]);
    smem_tile[(r0 + 9) * 16 + g + 8] = uint16_t(frag[3] >> 16);
    __syncwarp();
    const unsigned row = lane >> 1, half = lane & 1u;
    const uint4 v = *reinterpret_cast<const uint4 *>(smem_tile + row * 16 + half * 8);
    *reinterpret_cast<uint4 *>(out + size_t(row) * ld + half * 8) = v;
    __syncwarp();
}

__global__ void k_decode_inner_ring(const uint16_t * __restrict__ packed, size_t k, size_t n, size_t first_column,
                                    size_t column_count, unsigned bits, unsigned cb, uint16_t * __restrict__ out) {
    __shared__ __align__(16) uint16_t stage[8][256];
    const unsigned warp = threadIdx.x >> 5;
    const size_t tiles_c = column_count / 16;
    const size_t tile = size_t(blockIdx.x) * 8 + warp;
    if (tile >= (k / 16) * tiles_c) return;
    const size_t rk = tile / tiles_c, cn = tile % tiles_c;
    const uint16_t * src = packed + (rk * (n / 16) + first_column / 16 + cn) * 16u * bits;
    uint32_t frag[4];
    decode_ring_tile_lane(src, bits, cb, frag);
    store_tile_rowmajor(frag, stage[warp], out + rk * 16 * column_count + cn * 16, column_count);
}

// ---------------------------------------------------------------------------
// Device layout conversion.  Output word `ow` of a chunk belongs to lane
// L = ow / (2*bits), segment word sw = ow % (2*bits).  Segment memory byte S
// holds ring-order byte S ^ 3 = bits*c + j of the lane segment, i.e. ring byte
// bits*L + j of tile c, found at tile memory byte (bits*L + j) ^ 3.
__device__ __forceinline__ uint32_t gather_lsc_word(const uint8_t * const tile_ptr[8], unsigned bits, unsigned lane,
                                                    unsigned sw) {
    uint32_t word = 0;
#pragma unroll
    for (unsigned q = 0; q < 4; ++q) {
        const unsigned S = 4u * sw + q;
        const unsigned ro = S ^ 3u;
        const unsigned c = ro / bits, j = ro % bits;
        const unsigned tb = (bits * lane + j) ^ 3u;
        word |= uint32_t(tile_ptr[c][tb]) << (8u * q);
    }
    return word;
}

// records: [n/128][k/128] groups of 2048*bits+512 bytes (record (nb,kb), tiles r*8+c).
__global__ void k_records_to_lsc(const uint8_t * __restrict__ records, size_t k, unsigned bits, size_t nb0,
                                 size_t nbc, uint32_t * __restrict__ lsc) {
    const size_t words_per_chunk = 64u * bits;
    const size_t nchunks = k / 16;
    const size_t total = nbc * nchunks * words_per_chunk;
    const size_t group_bytes = 2048u * bits + 512u;
    for (size_t idx = size_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total; idx += size_t(gridDim.x) * blockDim.x) {
        const size_t chunk = idx / words_per_chunk;
        const unsigned ow = unsigned(idx % words_per_chunk);
        const size_t nbl = chunk / nchunks, rk = chunk % nchunks;
        const size_t kb = rk / 8, r = rk % 8;
        const uint8_t * rec = records + ((nb0 + nbl) * (k / 128) + kb) * group_bytes;
        const uint8_t * tp[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) tp[c] = rec + (r * 8 + c) * 32u * bits;
        lsc[idx] = gather_lsc_word(tp, bits, ow / (2u * bits), ow % (2u * bits));
    }
}

// trellis: upstream [k/16][n/16][16*bits] uint16.
__global__ void k_trellis_to_lsc(const uint16_t * __restrict__ trellis, size_t k, size_t n, unsigned bits, size_t nb0,
                                 size_t nbc, uint32_t * __restrict__ lsc) {
    const size_t words_per_chunk = 64u * bits;
    const size_t nchunks = k / 16;
    const size_t total = nbc * nchunks * words_per_chunk;
    const uint8_t * base = reinterpret_cast<const uint8_t *>(trellis);
    for (size_t idx = size_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total; idx += size_t(gridDim.x) * blockDim.x) {
        const size_t chunk = idx / words_per_chunk;
        const unsigned ow = unsigned(idx % words_per_chunk);
        const size_t nbl = chunk / nchunks, rk = chunk % nchunks;
        const uint8_t * tp[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) tp[c] = base + (rk * (n / 16) + (nb0 + nbl) * 8 + c) * 32u * bits;
        lsc[idx] = gather_lsc_word(tp, bits, ow / (2u * bits), ow % (2u * bits));
    }
}

// LSC -> row-major inner weights for column blocks [0, nbc) of the handle.
template <int BITS>
__global__ void k_lsc_decode(const uint32_t * __restrict__ lsc, size_t k, size_t nbc, unsigned cb,
                             uint16_t * __restrict__ out) {
    __shared__ __align__(16) uint16_t stage[4][256];
    const unsigned warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const size_t nchunks = k / 16;
    const size_t chunk = size_t(blockIdx.x) * 4 + warp;
    if (chunk >= nbc * nchunks) return;
    const size_t nb = chunk / nchunks, rk = chunk % nchunks;
    uint32_t w[2 * BITS];
    load_segment<BITS>(lsc + chunk * 64u * BITS + lane * 2u * BITS, w);
    uint32_t frag[8][4];
    if (cb == CB_MUL1) decode_chunk<BITS, CB_MUL1>(w, frag);
    else if (cb == CB_MCG) decode_chunk<BITS, CB_MCG>(w, frag);
    else decode_chunk<BITS, CB_3INST>(w, frag);
    const size_t ld = nbc * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) store_tile_rowmajor(frag[c], stage[warp], out + rk * 16 * ld + nb * 128 + c * 16, ld);
}

// ---------------------------------------------------------------------------
// In-place H128 on count/128 groups, one warp per group.
__global__ void k_hadamard128(float * __restrict__ v, size_t groups) {
    const size_t g = size_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (g >= groups) return;
    const unsigned lane = threadIdx.x & 31u;
    float4 x = *reinterpret_cast<float4 *>(v + g * 128 + lane * 4);
    float r[4] = {x.x, x.y, x.z, x.w};
    h128_warp4(r);
    *reinterpret_cast<float4 *>(v + g * 128 + lane * 4) = make_float4(r[0], r[1], r[2], r[3]);
}

// Original basis (src/exl3_codec.cpp:169-204): for each 128x128 block of the
// decoded inner matrix (already in `io` as fp16, row stride ld), rotate every
// row, then every column, then scale by suh[row]*svh[col] and round to fp16.
// One CTA (8 warps) per block; the block lives in shared memory as fp32.
__global__ void k_reconstruct_blocks(uint16_t * __restrict__ io, size_t ld, size_t first_column,
                                     const uint16_t * __restrict__ suh, const uint16_t * __restrict__ svh) {
    extern __shared__ __align__(16) float blk[];  // 128 x 129 (padded)
    const unsigned warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const size_t rk = size_t(blockIdx.y) * 128, cn = size_t(blockIdx.x) * 128;
    constexpr int LD = 129;
    for (int r = warp; r < 128; r += 8) {
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
            v[q] = __half2float(__ushort_as_half(io[(rk + r) * ld + cn + lane * 4 + q]));
        h128_warp4(v);
#pragma unroll
        for (int q = 0; q < 4; ++q) blk[r * LD + lane * 4 + q] = v[q];
    }
    __syncthreads();
    for (int c = warp; c < 128; c += 8) {
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = blk[(lane * 4 + q) * LD + c];
        h128_warp4(v);
        const float sv = __half2float(__ushort_as_half(svh[first_column + cn + c]));
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const unsigned r = lane * 4 + q;
            const float su = __half2float(__ushort_as_half(suh[rk + r]));
            const float val = __fmul_rn(__fmul_rn(v[q], su), sv);
            io[(rk + r) * ld + cn + c] = __half_as_ushort(__float2half_rn(val));
        }
    }
}

// ---------------------------------------------------------------------------
// get_rows (src/exl3-ggml.cpp:19-49): for token id, the original-basis column
// W[:, id] over all k rows as f32.  One CTA per (id, 128-row group kb), as the
// reference reconstructs one 128x128 group per (id, kb): the group is decoded
// into shared memory (fp16 -> fp32 exact), every row is rotated (H128 along
// the row, the reference's butterfly), the id's column is kept, rotated along
// the k direction, scaled by suh[row] then svh[id] and rounded to fp16 -- the
// operations of exl3::reconstruct (src/exl3_codec.cpp:169-204) in its order.
// ids are local to the handle's column range; an id outside it yields a row
// of NaN and raises kStatusBadIndex.
static __device__ unsigned g_rows_status;

template <int BITS, unsigned CB>
__global__ void __launch_bounds__(256) k_get_rows(const uint32_t * __restrict__ lsc, const uint16_t * __restrict__ suh,
                                                  const uint16_t * __restrict__ svh, size_t k, size_t ncols,
                                                  const int32_t * __restrict__ ids, void * __restrict__ out,
                                                  size_t out_stride, bool out_f16) {
    __shared__ uint16_t blk[128 * 130];  // decoded fp16 bits (exact), row pitch 65 words
    __shared__ float col[128];
    const unsigned warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const size_t kb = blockIdx.x, r_out = blockIdx.y;
    const int32_t id = ids[r_out];
    const size_t dst_off = r_out * out_stride + kb * 128;
    float * dst = static_cast<float *>(out) + dst_off;
    uint16_t * dst16 = static_cast<uint16_t *>(out) + dst_off;
    if (id < 0 || size_t(id) >= ncols) {
        if (threadIdx.x < 128) {
            if (out_f16) dst16[threadIdx.x] = 0x7e00u;
            else dst[threadIdx.x] = __int_as_float(0x7fc00000);
        }
        if (threadIdx.x == 0) atomicOr(&g_rows_status, kStatusBadIndex);
        return;
    }
    const size_t nb = size_t(id) / 128, c_in = size_t(id) % 128, nchunks = k / 16;
    {
        // warp w decodes chunk (nb, 8*kb + w): rows 16w..16w+15 of the group, all 128 columns
        const size_t chunk = nb * nchunks + kb * 8 + warp;
        uint32_t w[2 * BITS];
        load_segment<BITS>(lsc + chunk * 64u * BITS + lane * 2u * BITS, w);
        uint32_t frag[8][4];
        decode_chunk<BITS, CB>(w, frag);
        const unsigned g = lane >> 2, t = lane & 3u;
        const unsigned r0 = warp * 16 + 2 * t;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            // A-fragment of W^T: reg0 = rows 2t, 2t+1 of column g; reg1 column g+8; reg2/3 rows +8
            const unsigned cg0 = c * 16 + g, cg8 = cg0 + 8;
            const uint32_t f0 = frag[c][0], f1 = frag[c][1], f2 = frag[c][2], f3 = frag[c][3];
            blk[(r0) * 130 + cg0] = uint16_t(f0 & 0xffffu);
            blk[(r0 + 1) * 130 + cg0] = uint16_t(f0 >> 16);
            blk[(r0) * 130 + cg8] = uint16_t(f1 & 0xffffu);
            blk[(r0 + 1) * 130 + cg8] = uint16_t(f1 >> 16);
            blk[(r0 + 8) * 130 + cg0] = uint16_t(f2 & 0xffffu);
            blk[(r0 + 9) * 130 + cg0] = uint16_t(f2 >> 16);
            blk[(r0 + 8) * 130 + cg8] = uint16_t(f3 & 0xffffu);
            blk[(r0 + 9) * 130 + cg8] = uint16_t(f3 >> 16);
        }
    }
    __syncthreads();
    for (int r = warp; r < 128; r += 8) {
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = __half2float(__ushort_as_half(blk[r * 130 + lane * 4 + q]));
        h128_warp4(v);
        if (lane == c_in / 4) col[r] = v[c_in % 4];
    }
    __syncthreads();
    if (warp == 0) {
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = col[lane * 4 + q];
        h128_warp4(v);
        const float sv = __half2float(__ushort_as_half(svh[id]));
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const size_t row = kb * 128 + lane * 4 + q;
            const float su = __half2float(__ushort_as_half(suh[row]));
            const __half h = __float2half_rn(__fmul_rn(__fmul_rn(v[q], su), sv));
            if (out_f16) dst16[lane * 4 + q] = __half_as_ushort(h);
            else dst[lane * 4 + q] = __half2float(h);
        }
    }
}

template <int BITS>
static cudaError_t get_rows_bits(const uint32_t * lsc, const uint16_t * suh, const uint16_t * svh, size_t k,
                                 size_t ncols, unsigned cb, const int32_t * ids, size_t count, void * out,
                                 size_t out_stride, bool f16, cudaStream_t st) {
    const dim3 grid(unsigned(k / 128), unsigned(count));
    if (cb == CB_MUL1) k_get_rows<BITS, CB_MUL1><<<grid, 256, 0, st>>>(lsc, suh, svh, k, ncols, ids, out, out_stride, f16);
    else if (cb == CB_MCG) k_get_rows<BITS, CB_MCG><<<grid, 256, 0, st>>>(lsc, suh, svh, k, ncols, ids, out, out_stride, f16);
    else k_get_rows<BITS, CB_3INST><<<grid, 256, 0, st>>>(lsc, suh, svh, k, ncols, ids, out, out_stride, f16);
    return cudaGetLastError();
}

cudaError_t launch_get_rows(const uint32_t * lsc, const uint16_t * suh, const uint16_t * svh, size_t k, size_t ncols,
                            unsigned bits, unsigned cb, const int32_t * ids, size_t count, void * out,
                            size_t out_stride, bool out_f16, cudaStream_t st) {
    if (!count) return cudaSuccess;
    switch (bits) {
        case 1: return get_rows_bits<1>(lsc, suh, svh, k, ncols, cb, ids, count, out, out_stride, out_f16, st);
        case 2: return get_rows_bits<2>(lsc, suh, svh, k, ncols, cb, ids, count, out, out_stride, out_f16, st);
        case 3: return get_rows_bits<3>(lsc, suh, svh, k, ncols, cb, ids, count, out, out_stride, out_f16, st);
        case 4: return get_rows_bits<4>(lsc, suh, svh, k, ncols, cb, ids, count, out, out_stride, out_f16, st);
        case 5: return get_rows_bits<5>(lsc, suh, svh, k, ncols, cb, ids, count, out, out_stride, out_f16, st);
        case 6: return get_rows_bits<6>(lsc, suh, svh, k, ncols, cb, ids, count, out, out_stride, out_f16, st);
        case 7: return get_rows_bits<7>(lsc, suh, svh, k, ncols, cb, ids, count, out, out_stride, out_f16, st);
        case 8: return get_rows_bits<8>(lsc, suh, svh, k, ncols, cb, ids, count, out, out_stride, out_f16, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t rows_read_status(unsigned * out, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_rows_status, sizeof(unsigned));
    if (e == cudaSuccess && clear && *out) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(g_rows_status, &zero, sizeof(unsigned));
    }
    return e;
}

// ---------------------------------------------------------------------------
// Host launchers (stream-ordered, no synchronisation).

cudaError_t launch_codebook(const uint16_t * states, size_t count, unsigned cb, uint16_t * out, cudaStream_t st) {
    if (!count) return cudaSuccess;
    const size_t pairs = (count + 1) / 2;
    k_codebook<<<unsigned((pairs + 255) / 256), 256, 0, st>>>(states, count, cb, out);
    return cudaGetLastError();
}

cudaError_t launch_decode_inner(const uint16_t * packed, size_t k, size_t n, size_t first_column,
                                size_t column_count, unsigned bits, unsigned cb, uint16_t * out, cudaStream_t st) {
    const size_t tiles = (k / 16) * (column_count / 16);
    k_decode_inner_ring<<<unsigned((tiles + 7) / 8), 256, 0, st>>>(packed, k, n, first_column, column_count, bits,
                                                                     cb, out);
    return cudaGetLastError();
}

static unsigned grid_for(size_t total, unsigned block) {
    const size_t g = (total + block - 1) / block;
    return unsigned(g < 65535u * 64u ? g : 65535u * 64u);
}

cudaError_t launch_records_to_lsc(const uint8_t * records, size_t k, unsigned bits, size_t nb0, size_t nbc,
                                  uint32_t * lsc, cudaStream_t st) {
    const size_t total = nbc * (k / 16) * 64u * bits;
    k_records_to_lsc<<<grid_for(total, 256), 256, 0, st>>>(records, k, bits, nb0, nbc, lsc);
    return cudaGetLastError();
}

cudaError_t launch_trellis_to_lsc(const uint16_t * trellis, size_t k, size_t n, unsigned bits, size_t nb0,
                                  size_t nbc, uint32_t * lsc, cudaStream_t st) {
    const size_t total = nbc * (k / 16) * 64u * bits;
    k_trellis_to_lsc<<<grid_for(total, 256), 256, 0, st>>>(trellis, k, n, bits, nb0, nbc, lsc);
    return cudaGetLastError();
}

template <int BITS>
static cudaError_t lsc_decode_bits(const uint32_t * lsc, size_t k, size_t nbc, unsigned cb, uint16_t * out,
                                   cudaStream_t st) {
    const size_t chunks = nbc * (k / 16);
    k_lsc_decode<BITS><<<unsigned((chunks + 3) / 4), 128, 0, st>>>(lsc, k, nbc, cb, out);
    return cudaGetLastError();
}

cudaError_t launch_lsc_decode(const uint32_t * lsc, size_t k, size_t nbc, unsigned bits, unsigned cb, uint16_t * out,
                              cudaStream_t st) {
    switch (bits) {
        case 1: return lsc_decode_bits<1>(lsc, k, nbc, cb, out, st);
        case 2: return lsc_decode_bits<2>(lsc, k, nbc, cb, out, st);
        case 3: return lsc_decode_bits<3>(lsc, k, nbc, cb, out, st);
        case 4: return lsc_decode_bits<4>(lsc, k, nbc, cb, out, st);
        case 5: return lsc_decode_bits<5>(lsc, k, nbc, cb, out, st);
        case 6: return lsc_decode_bits<6>(lsc, k, nbc, cb, out, st);
        case 7: return lsc_decode_bits<7>(lsc, k, nbc, cb, out, st);
        case 8: return lsc_decode_bits<8>(lsc, k, nbc, cb, out, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_hadamard128(float * v, size_t count, cudaStream_t st) {
    const size_t groups = count / 128;
    if (!groups) return cudaSuccess;
    k_hadamard128<<<unsigned((groups + 7) / 8), 256, 0, st>>>(v, groups);
    return cudaGetLastError();
}

cudaError_t launch_reconstruct_blocks(uint16_t * io, size_t k, size_t column_count, size_t first_column,
                                      const uint16_t * suh, const uint16_t * svh, cudaStream_t st) {
    const size_t smem = 128 * 129 * sizeof(float);
    // function attributes are per device context: set on every call (cheap, not a hot path)
    cudaError_t e = cudaFuncSetAttribute(k_reconstruct_blocks, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    dim3 grid(unsigned(column_count / 128), unsigned(k / 128));
    k_reconstruct_blocks<<<grid, 256, smem, st>>>(io, column_count, first_column, suh, svh);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Ragged continuous-admission batch packer.  Sequence i asks for want[i] rows
// this step (1 for a decode token, a chunk length for prefill) starting at
// position pos[i]; in the given order each is granted min(want, rows left of
// the max_rows budget), so the caller's order is its admission policy (e.g.
// decode tokens first).  Outputs row_offsets[n_seq + 1] (row_offsets[n_seq] =
// the packed row count) and, per packed row r < max_rows, its sequence and
// position (-1 past the packed rows).  One CTA: a capped exclusive scan in
// 64-bit arithmetic, then a binary search over the offsets per row.
constexpr int kPackThreads = 1024;

__global__ void __launch_bounds__(kPackThreads) k_pack_ragged(int n_seq, const int32_t * __restrict__ want,
                                                              const int32_t * __restrict__ pos, int32_t max_rows,
                                                              int32_t * __restrict__ row_offsets,
                                                              int32_t * __restrict__ row_seq,
                                                              int32_t * __restrict__ row_pos) {
    __shared__ long long part[kPackThreads];
    const int t = threadIdx.x;
    const int per = (n_seq + kPackThreads - 1) / kPackThreads;
    const int i0 = min(t * per, n_seq), i1 = min(i0 + per, n_seq);
    long long sum = 0;
    for (int i = i0; i < i1; ++i) sum += max(want[i], 0);
    part[t] = sum;
    __syncthreads();
    for (int off = 1; off < kPackThreads; off <<= 1) {  // inclusive Hillis-Steele scan
        const long long v = t >= off ? part[t - off] : 0;
        __syncthreads();
        part[t] += v;
        __syncthreads();
    }
    long long run = t > 0 ? part[t - 1] : 0;
    for (int i = i0; i < i1; ++i) {
        row_offsets[i] = int32_t(run < max_rows ? run : max_rows);
        run += max(want[i], 0);
    }
    if (t == kPackThreads - 1) row_offsets[n_seq] = int32_t(part[t] < max_rows ? part[t] : max_rows);
    __syncthreads();  // the offsets are visible to the whole block
    const int rows = row_offsets[n_seq];
    for (int r = t; r < max_rows; r += kPackThreads) {
        if (r >= rows) {
            row_seq[r] = -1;
            row_pos[r] = -1;
            continue;
        }
        int lo = 0, hi = n_seq - 1;  // last i with row_offsets[i] <= r
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (row_offsets[mid] <= r) lo = mid; else hi = mid - 1;
        }
        row_seq[r] = lo;
        row_pos[r] = pos[lo] + (r - row_offsets[lo]);
    }
}

cudaError_t launch_pack_ragged(int n_seq, const int32_t * want, const int32_t * pos, int32_t max_rows,
                               int32_t * row_offsets, int32_t * row_seq, int32_t * row_pos, cudaStream_t st) {
    k_pack_ragged<<<1, kPackThreads, 0, st>>>(n_seq, want, pos, max_rows, row_offsets, row_seq, row_pos);
    return cudaGetLastError();
}

}  // namespace exl3cu
