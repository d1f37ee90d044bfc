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

// Packed tiles use upstream CUDA lane order and little-endian uint16 storage.
void decode_tile(const uint16_t * packed, unsigned bits, Codebook codebook, uint16_t * row_major);
void decode_inner(const uint16_t * packed, size_t k, size_t n, unsigned bits, Codebook codebook, uint16_t * output);
void decode_inner_slice(const uint16_t * packed, size_t k, size_t n, size_t first_column, size_t column_count,
                        unsigned bits, Codebook codebook, uint16_t * output);

// In-place orthonormal H128 on each consecutive group of 128 values.
void hadamard128(float * values, size_t count);

// Original-basis matrix: diag(suh) H128 W_hat H128 diag(svh), laid out as [k,n].
void reconstruct(const uint16_t * packed, const uint16_t * suh, const uint16_t * svh, size_t k, size_t n,
                 unsigned bits, Codebook codebook, uint16_t * output);
void reconstruct_slice(const uint16_t * packed, const uint16_t * suh, const uint16_t * svh, size_t k, size_t n,
                       size_t first_column, size_t column_count, unsigned bits, Codebook codebook, uint16_t * output);

}  // namespace exl3
