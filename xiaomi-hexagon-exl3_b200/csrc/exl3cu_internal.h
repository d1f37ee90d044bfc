// Internal declarations shared by the CUDA translation units of libexl3cu.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "exl3cu_common.cuh"
#include "exl3cu_decode.cuh"

namespace exl3cu {

struct GemvArgs {
    const uint32_t * lsc;   // device weights, LSC layout, column blocks [0, nblocks)
    const __half * su;      // [k]
    const __half * sv;      // [nblocks * 128]
    const void * x;         // [rows][x_stride], f32 or f16
    float * y;              // [rows][y_stride]
    float * ws_partial;     // [nblocks][splits][8][128] (splits > 1)
    unsigned * ws_count;    // [nblocks], zero between calls
    long long x_stride;     // elements
    long long y_stride;     // elements
    int x_f16;
    int rows;               // 1..8
    int nblocks;
    int nchunks;            // k / 16
    int cps;                // chunks per split
    int splits;
};

struct GemvPlan {
    int cps;
    int splits;
    size_t smem;
};

GemvPlan plan_gemv(int device_sms, size_t k, size_t nblocks, int rows);
size_t gemv_workspace_bytes(size_t nblocks, int splits);
cudaError_t launch_gemv(const GemvArgs & a, const GemvPlan & p, unsigned bits, unsigned cb, cudaStream_t st);

cudaError_t launch_codebook(const uint16_t * states, size_t count, unsigned cb, uint16_t * out, cudaStream_t st);
cudaError_t launch_decode_inner(const uint16_t * packed, size_t k, size_t n, size_t first_column,
                                size_t column_count, unsigned bits, unsigned cb, uint16_t * out, cudaStream_t st);
cudaError_t launch_records_to_lsc(const uint8_t * records, size_t k, unsigned bits, size_t nb0, size_t nbc,
                                  uint32_t * lsc, cudaStream_t st);
cudaError_t launch_trellis_to_lsc(const uint16_t * trellis, size_t k, size_t n, unsigned bits, size_t nb0,
                                  size_t nbc, uint32_t * lsc, cudaStream_t st);
cudaError_t launch_lsc_decode(const uint32_t * lsc, size_t k, size_t nbc, unsigned bits, unsigned cb, uint16_t * out,
                              cudaStream_t st);
cudaError_t launch_hadamard128(float * v, size_t count, cudaStream_t st);
cudaError_t launch_reconstruct_blocks(uint16_t * io, size_t k, size_t column_count, size_t first_column,
                                      const uint16_t * suh, const uint16_t * svh, cudaStream_t st);

}  // namespace exl3cu
