// Internal declarations shared by the CUDA translation units of libexl3cu.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "exl3cu_common.cuh"
#include "exl3cu_decode.cuh"

struct exl3cu_weight;

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

// One problem of a grouped GEMV launch: y[r] = x[r] . W for r < rows (<= 8).
struct GemvProblem {
    const uint32_t * lsc;
    const __half * su;
    const __half * sv;
    const void * x;
    float * y;
    long long x_stride;
    long long y_stride;
    int nchunks;    // k / 16
    int cps;        // chunks per cluster rank
    int rows;       // 1..8
    int x_f16;
    int unit_base;  // first unit (column block) of this problem in the launch
    int x_mode;     // kXPlain; kXGlu: rows [gate (k) | up (k)], input silu(gate) up;
                    // kXRmsNorm: rows h, input h rsqrt(mean(h^2) + eps) nw (mul1 kernel only)
    const float * nw;
    float eps;
    int y_accum;    // 1: y += x . W (one writer per element) instead of y = x . W
    const float * x_ss;  // kXRmsNorm, optional: [rows][k/128] sums of squares of the rows' 128-blocks
    float * y_ss;        // optional: [rows][y_ss_stride] sums of squares of the final y, per column block
    int y_ss_stride;     // column blocks of the item's y row
};

constexpr int kXPlain = 0, kXGlu = 1, kXRmsNorm = 2;

constexpr int kMaxBatch = 8;  // problems per launch, passed by value in the kernel parameters

// Peer-memory exchange of a column split (exl3cu_peers.cu, and the mul1 GEMV's epilogue).  A rank's
// y buffer holds (epoch << 32 | float bits) words, [2][rows_cap][y_stride]; its state words are
// [kPeerTicketWord] the wait kernel's arrival ticket and [kPeerEpochWord] the rank's epoch counter.
constexpr int kMaxPeers = 8;
constexpr int kPeerTicketWord = 8;
constexpr int kPeerEpochWord = 9;

// Where a launch's output also goes: the E-th call (E = counter + 1) stores its y rows as
// (E, value) words into half (E & 1) of every rank's y buffer.
struct PeerOut {
    unsigned long long * y[kMaxPeers];  // every rank's y buffer (this rank's included)
    const unsigned * own_state;         // this rank's state words
    long long y_stride;                 // words between rows of a y buffer
    long long y_half;                   // words between the two halves
    long long y_col0;                   // this rank's first column in the full row
    int npeers;
};

struct GemvBatch {
    GemvProblem prob[kMaxBatch];
    int count;
    int splits;     // cluster size: CTAs per unit along K
    int stages;     // mul1 kernel: weight ring depth (stages of kMW chunks)
    int nw_smem;    // mul1 kernel: RMSNorm weights staged in shared memory before the dependency wait
    int peer_on;    // mul1 kernel, one problem: y goes to the peers' buffers (`peer`) instead of prob[0].y
    PeerOut peer;
};

int choose_cluster_splits(int sms, int nunits, int min_nchunks);
size_t cluster_smem_bytes(int max_cps, int rows);
cudaError_t launch_gemv_cluster(const GemvBatch & b, int nunits, size_t smem, unsigned bits, unsigned cb, bool pdl,
                                cudaStream_t st);

bool mul1_supported(unsigned bits, int rows);
bool pdl_launch_enabled();  // programmatic dependent launch on (EXL3CU_PDL unset or not "0")
cudaError_t launch_gemv_mul1(GemvBatch & b, int nunits, int sms, int device, unsigned bits, bool pdl,
                             cudaStream_t st);
cudaError_t mul1_read_status(unsigned * out, bool clear);

// tcgen05 GEMM for batches of rows (exl3cu_gemm_tc.cu): decoded weights in TMEM
// as the A operand, tokens as N (<= 256 per CTA).
struct GemmPlan {
    int ntok;       // tokens per CTA, multiple of 32
    int tgroups;    // token groups
    int splits;     // cluster size along K
    int cps;        // chunks per cluster rank (multiple of 8)
    int wstages;    // trellis ring depth in groups of 8 chunks (multiple of 3)
    size_t smem;
    size_t xt_bytes;  // tiled activation scratch
};
// tokens / splits > 0 override the automatic tokens per CTA / cluster size.
GemmPlan plan_gemm(int device, int sms, size_t k, size_t nblocks, unsigned bits, unsigned cb, int rows, int tokens = 0,
                   int splits = 0);
// rows = the launch's row capacity; m_dev (nullable) = device-resident live row count of
// the whole batch, of which this launch covers rows [m_base, m_base + rows).
cudaError_t launch_gemm(const GemmPlan & p, const uint32_t * lsc, const __half * su, const __half * sv, size_t k,
                        size_t nblocks, unsigned bits, unsigned cb, int device, const void * x, int x_f16,
                        long long x_stride, int rows, const int32_t * m_dev, int m_base, float * y, long long y_stride,
                        __half * xt, bool pdl, cudaStream_t st, const PeerOut * peer = nullptr);
// Ragged batch packer (exl3cu_kernels.cu): grants each sequence min(want, remaining budget) rows in order.
cudaError_t launch_pack_ragged(int n_seq, const int32_t * want, const int32_t * pos, int32_t max_rows,
                               int32_t * row_offsets, int32_t * row_seq, int32_t * row_pos, cudaStream_t st);
cudaError_t gemm_read_status(unsigned * out, bool clear);

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
// out: f32 rows, or fp16 rows (the bits exl3::reconstruct produces) with out_f16.
cudaError_t launch_get_rows(const uint32_t * lsc, const uint16_t * suh, const uint16_t * svh, size_t k, size_t ncols,
                            unsigned bits, unsigned cb, const int32_t * ids, size_t count, void * out,
                            size_t out_stride, bool out_f16, cudaStream_t st);
cudaError_t rows_read_status(unsigned * out, bool clear);
cudaError_t peer_read_status(unsigned * out, bool clear);
// 0 when p is device (or managed) memory of `device` (-1: any device), else a failure status with the
// thread's error text set (exl3cu_api.cu).
int api_check_device_ptr(const void * p, int device, const char * name);
cudaError_t launch_reconstruct_blocks(uint16_t * io, size_t k, size_t column_count, size_t first_column,
                                      const uint16_t * suh, const uint16_t * svh, cudaStream_t st);

// Shared by the C-ABI translation units (defined in exl3cu_api.cu): record
// the calling thread's last error and return `status`; the CUDA form also
// clears a non-sticky CUDA error.
int api_fail(int status, const char * message);
int api_cuda_fail(cudaError_t e, const char * what);
// Weights owned by a model handle: exl3cu_weight_free refuses them and the
// model frees them with weight_free_owned.
void weight_set_model_owned(struct ::exl3cu_weight * w);
void weight_free_owned(struct ::exl3cu_weight * w);
struct WeightGeometry {
    size_t k, n_local;
    unsigned bits, codebook;
    int device;
    const uint32_t * lsc;
    const uint16_t * su;
    const uint16_t * sv;
};
WeightGeometry weight_geometry(const struct ::exl3cu_weight * w);

}  // namespace exl3cu
