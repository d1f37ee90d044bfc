// EXL3 codec host API, backed by the B200 kernels of libexl3cu.
//
// Drop-in for the reference's include/exl3_codec.h:1-31: the same namespace,
// enum and signatures, the same layouts (upstream trellis [k/16][n/16][16*bits]
// little-endian uint16, row-major outputs), and the same error contract --
// std::invalid_argument for a bad bitrate, codebook, shape or slice.  Buffers
// are host memory owned by the caller, as in the reference; each call copies to
// the current CUDA device, runs there and copies back (std::runtime_error on a
// CUDA failure).  Decoded inner weights are bit-exact with the reference;
// reconstruct() and hadamard128() follow its fp32 operation order.
#pragma once

#include <cstddef>
#include <cstdint>

namespace exl3 {

enum class Codebook : uint32_t { three_inst = 0, mcg = 1, mul1 = 2 };

float half_to_float(uint16_t value);
uint16_t float_to_half(float value);
uint16_t decode_codebook(uint16_t state, Codebook codebook);

// `packed` is the upstream trellis tensor [k/16][n/16][16*bits] as little-endian
// uint16 words, tiles in the order the upstream CUDA kernels use; outputs are
// row-major fp16 bit patterns.
void decode_tile(const uint16_t * packed, unsigned bits, Codebook codebook, uint16_t * row_major);
void decode_inner(const uint16_t * packed, size_t k, size_t n, unsigned bits, Codebook codebook, uint16_t * output);
void decode_inner_slice(const uint16_t * packed, size_t k, size_t n, size_t first_column, size_t column_count,
                        unsigned bits, Codebook codebook, uint16_t * output);

// Rotates every run of 128 consecutive floats by the normalised 128-point
// Walsh-Hadamard transform, in place; `count` is a multiple of 128.
void hadamard128(float * values, size_t count);

// The weight matrix in its unrotated basis, [k][n] row-major fp16:
// rows scaled by suh, H128 on both sides of the decoded matrix, columns by svh.
void reconstruct(const uint16_t * packed, const uint16_t * suh, const uint16_t * svh, size_t k, size_t n,
                 unsigned bits, Codebook codebook, uint16_t * output);
void reconstruct_slice(const uint16_t * packed, const uint16_t * suh, const uint16_t * svh, size_t k, size_t n,
                       size_t first_column, size_t column_count, unsigned bits, Codebook codebook, uint16_t * output);

}  // namespace exl3
