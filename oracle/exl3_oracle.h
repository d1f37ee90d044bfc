/*
 * EXL3 CPU oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's EXL3 codec and CPU mul_mat operator
 * (jyohukuchan/xiaomi-hexagon-exl3: src/exl3_codec.cpp, src/exl3-ggml.cpp).
 * It is the checker the parity tests compare the CUDA path against; only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it.
 * The shipped library never links, calls or falls back to it.
 *
 * Pinned: tests/test_oracle.py checks every function here against golden
 * vectors produced by the reference's own sources (oracle/_ref, built by
 * oracle/Makefile) and against the reference's known-answer tests
 * (tests/test_codec.cpp of the reference).
 *
 * All functions return 0 on success, nonzero (1) on invalid arguments -- the
 * cases where the reference throws std::invalid_argument.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_CB_3INST = 0, ORC_CB_MCG = 1, ORC_CB_MUL1 = 2 };

float orc_half_to_float(uint16_t h);
uint16_t orc_float_to_half(float f);
uint16_t orc_decode_codebook(uint16_t state, unsigned codebook);
int orc_decode_tile(const uint16_t * packed, unsigned bits, unsigned codebook, uint16_t * tile256);
int orc_decode_inner(const uint16_t * packed, size_t k, size_t n, size_t first_column, size_t column_count,
                     unsigned bits, unsigned codebook, uint16_t * out);
int orc_hadamard128(float * values, size_t count);
int orc_reconstruct(const uint16_t * packed, const uint16_t * suh, const uint16_t * svh, size_t k, size_t n,
                    size_t first_column, size_t column_count, unsigned bits, unsigned codebook, uint16_t * out);

/* Runtime group records <-> upstream trellis layout. */
size_t orc_group_bytes(unsigned bits);
int orc_pack_records(const uint16_t * packed, const uint16_t * suh, const uint16_t * svh, size_t k, size_t n,
                     unsigned bits, uint8_t * records);

/* ggml_exl3_mul_mat restated over runtime records, any bitrate 1..8 / codebook.
 * x: rows x k (f32 if x_is_f16 == 0, else f16 bits), row stride x_stride elements.
 * y: rows x n f32, row stride y_stride elements.  nth worker threads split output
 * column blocks like the reference's ith/nth. */
int orc_mul_mat(const uint8_t * records, unsigned bits, unsigned codebook, size_t k, size_t n, const void * x,
                int x_is_f16, size_t rows, size_t x_stride, float * y, size_t y_stride, int nth);

/* ggml_exl3_get_rows restated: one original-basis column per id, as f32 rows of k. */
int orc_get_rows(const uint8_t * records, unsigned bits, unsigned codebook, size_t k, size_t n, const int32_t * ids,
                 size_t count, float * out);

#ifdef __cplusplus
}
#endif
