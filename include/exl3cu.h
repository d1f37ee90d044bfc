/*
 * exl3cu -- C ABI of the B200 (sm_100a) EXL3 packed-weight matmul library.
 *
 * Plain pointers and sizes only.  Every entry returns an int status
 * (enum exl3cu_status) and never throws; exl3cu_last_error() gives the
 * detail of the last failure on the calling thread.  Calls taking a
 * `stream` are stream-ordered (a cudaStream_t, NULL = legacy default stream)
 * and do not synchronise unless stated.  Pointers named d_* are device
 * memory of the weight's device; h_* are host memory.
 *
 * Reference interfaces each entry replaces (jyohukuchan/xiaomi-hexagon-exl3):
 *   codec      include/exl3_codec.h:10-29 (exl3::decode_codebook/decode_inner/
 *              hadamard128/reconstruct) -- host-pointer C++ versions of these
 *              are in include/exl3_codec.h of this library.
 *   operator   ggml_exl3_mul_mat, include/exl3-block.h:46 / src/exl3-ggml.cpp:51-92,
 *              and the device operator op_exl3_matmul, src/exl3-htp.c:159-232,
 *              whose HTP_STATUS_* codes the statuses below mirror.
 *   weights    the runtime group records of include/exl3-block.h:14,34-39
 *              (tools/export_native_gguf.py:27-36) or the upstream trellis/suh/svh
 *              tensors (src/exl3_model.cpp:79-157), loaded once into persistent
 *              device buffers (the role the ggml backend buffer plays upstream).
 */
#ifndef EXL3CU_H
#define EXL3CU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EXL3CU_ABI_VERSION 1

/* Mirrors HTP_STATUS_{OK, INVAL_PARAMS, NO_SUPPORT, VTCM_TOO_SMALL, INTERNAL_ERR}
 * of src/exl3-htp.c:159-232 (VTCM_TOO_SMALL's analogue is device memory). */
enum exl3cu_status {
    EXL3CU_OK = 0,
    EXL3CU_INVALID_ARGUMENT = 1,
    EXL3CU_NO_SUPPORT = 2,
    EXL3CU_OUT_OF_MEMORY = 3,
    EXL3CU_CUDA_ERROR = 4
};

/* Activation dtypes: the ggml type ids (GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1). */
enum exl3cu_dtype { EXL3CU_F32 = 0, EXL3CU_F16 = 1 };
/* Input forms of exl3cu_mul_mat_batch_ex (beyond EXL3CU_F32 / EXL3CU_F16). */
enum exl3cu_x_form {
    EXL3CU_X_GLU = 2,     /* f32 rows [gate (k) | up (k)]; the operator's input is silu(gate) * up */
    EXL3CU_X_RMSNORM = 3  /* f32 rows h; the input is h * rsqrt(mean(h^2) + eps) * norm_w (mean over k) */
};

/* exl3::Codebook (include/exl3_codec.h:8). */
enum exl3cu_codebook { EXL3CU_CB_3INST = 0, EXL3CU_CB_MCG = 1, EXL3CU_CB_MUL1 = 2 };

typedef struct exl3cu_weight exl3cu_weight;
typedef struct exl3cu_model exl3cu_model;

/* Storage dtypes of model tensors (the safetensors dtypes exl3::Model accepts,
 * src/exl3_model.cpp:87). */
enum exl3cu_storage_dtype { EXL3CU_ST_F16 = 0, EXL3CU_ST_BF16 = 1, EXL3CU_ST_I16 = 2, EXL3CU_ST_F32 = 3, EXL3CU_ST_I32 = 4 };

/* exl3cu_model_open flags. */
#define EXL3CU_MODEL_VALIDATE_ONLY 1u

int exl3cu_abi_version(void);
const char * exl3cu_status_string(int status);
const char * exl3cu_last_error(void);

/* ---- codec on device buffers ----------------------------------------------------- */

/* d_out[i] = exl3::decode_codebook(d_states[i], codebook)   (src/exl3_codec.cpp:68-86) */
int exl3cu_decode_codebook(const uint16_t * d_states, size_t count, unsigned codebook, uint16_t * d_out,
                           void * stream);

/* exl3::decode_inner_slice: upstream trellis [k/16][n/16][16*bits] -> row-major fp16
 * [k][column_count], bit-exact (src/exl3_codec.cpp:123-145). */
int exl3cu_decode_inner(const uint16_t * d_packed, size_t k, size_t n, size_t first_column, size_t column_count,
                        unsigned bits, unsigned codebook, uint16_t * d_out, void * stream);

/* exl3::hadamard128 in place on count (multiple of 128) fp32 values (src/exl3_codec.cpp:147-167). */
int exl3cu_hadamard128(float * d_values, size_t count, void * stream);

/* exl3::reconstruct_slice: original-basis fp16 [k][column_count] (src/exl3_codec.cpp:169-204). */
int exl3cu_reconstruct(const uint16_t * d_packed, const uint16_t * d_suh, const uint16_t * d_svh, size_t k,
                       size_t n, size_t first_column, size_t column_count, unsigned bits, unsigned codebook,
                       uint16_t * d_out, void * stream);

/* ---- persistent device weights ----------------------------------------------------- */

/* Load column blocks [first_block, first_block + block_count) of a k x n matrix
 * (block_count 0 = all) from runtime group records -- n/128 * k/128 records of
 * 2048*bits + 512 bytes, record (nb,kb) at nb*(k/128)+kb (include/exl3-block.h:14).
 * `records` may be host or device memory.  Synchronises the device. */
int exl3cu_weight_from_records(const void * records, size_t record_bytes, size_t k, size_t n, unsigned bits,
                               unsigned codebook, size_t first_block, size_t block_count, int device,
                               exl3cu_weight ** out);

/* Same from the upstream tensors: trellis [k/16][n/16][16*bits] uint16, suh [k], svh [n] fp16. */
int exl3cu_weight_from_trellis(const uint16_t * trellis, const uint16_t * suh, const uint16_t * svh, size_t k,
                               size_t n, unsigned bits, unsigned codebook, size_t first_block, size_t block_count,
                               int device, exl3cu_weight ** out);

int exl3cu_weight_free(exl3cu_weight * w);

/* n_local = 128 * block_count columns held by this handle. */
int exl3cu_weight_info(const exl3cu_weight * w, size_t * k, size_t * n_local, unsigned * bits, unsigned * codebook,
                       size_t * device_bytes);

/* Decode the handle's device-layout weights back to row-major inner fp16 [k][n_local]. */
int exl3cu_weight_decode_inner(const exl3cu_weight * w, uint16_t * d_out, void * stream);

/* ---- the operator ---------------------------------------------------------------- */

/* y[r][0..n_local) = x[r] . W for r < rows (ggml_exl3_mul_mat semantics,
 * src/exl3-ggml.cpp:51-92): x rows of k f32/f16 values (x_dtype), row stride
 * x_row_stride elements; y rows of n_local f32, stride y_row_stride.  The K split
 * is reduced inside each thread-block cluster, so calls need no workspace and
 * calls on different streams may share a handle. */
int exl3cu_mul_mat(const exl3cu_weight * w, const void * d_x, int x_dtype, size_t rows, size_t x_row_stride,
                   float * d_y, size_t y_row_stride, void * stream);

/* Several independent operator calls in as few launches as possible: item i
 * computes d_y[i] = d_x[i] . weights[i] exactly as exl3cu_mul_mat would.  Items
 * sharing a bitrate and codebook run together (up to 8 per launch), so one
 * launch streams e.g. a layer's q, k and v, or gate and up.  Outputs must not
 * alias inputs of other items.  No counterpart in the reference, whose
 * operator handles one tensor per call. */
int exl3cu_mul_mat_batch(size_t count, const exl3cu_weight * const * weights, const void * const * d_x,
                         const int * x_dtype, const size_t * rows, const size_t * x_row_stride, float * const * d_y,
                         const size_t * y_row_stride, void * stream);

/* No counterpart in the reference.  exl3cu_mul_mat_batch with the layer glue of a
 * decoder folded into the operator: per item an input form (EXL3CU_F32,
 * EXL3CU_F16, EXL3CU_X_GLU: SwiGLU of a [gate | up] row computed on load,
 * EXL3CU_X_RMSNORM: RMSNorm of a residual-stream row with d_norm_w[i] and eps
 * computed on load), and y_accumulate[i] != 0 to add the product into y (the
 * residual add) instead of storing it.  The fused forms and accumulation run on
 * the integer-tensor-core GEMV only: mul1 weights of 2..8 bits and rows below
 * the GEMM threshold (5 by default); other items return EXL3CU_NO_SUPPORT.
 * d_norm_w / y_accumulate may be NULL when no item uses them.
 * Sums of squares for the RMSNorm, per 128-column block (f32 [rows][width/128],
 * dense): with d_y_sumsq[i] the operator also writes those of item i's final y
 * rows (after the accumulation), and an RMSNorm item given d_x_sumsq[i] takes
 * its rows' mean square from them instead of reading every row in full -- so
 * the kernel that updates the residual stream hands its norm to the next.
 * Either array, or entries of it, may be NULL.  As in exl3cu_mul_mat_batch, an
 * output must not alias any item's input, its own included. */
int exl3cu_mul_mat_batch_ex(size_t count, const exl3cu_weight * const * weights, const void * const * d_x,
                            const int * x_form, const size_t * rows, const size_t * x_row_stride,
                            const float * const * d_norm_w, float eps, float * const * d_y,
                            const size_t * y_row_stride, const int * y_accumulate,
                            const float * const * d_x_sumsq, float * const * d_y_sumsq, void * stream);

/* ---- ragged continuous-admission batches ----------------------------------------- */

/* GPU-side batch packer.  Sequence i asks for d_want[i] rows this step (1 for a
 * decode token, a prefill chunk length otherwise) starting at position
 * d_pos[i]; in the given order each is granted min(want, rows left of the
 * max_rows budget), so the caller's order is its admission policy.  Writes
 * d_row_offsets[n_seq + 1] (d_row_offsets[n_seq] = packed rows) and, for each of
 * the max_rows rows, its sequence index and position in d_row_seq / d_row_pos
 * (-1 past the packed rows).  Device int32 arrays of the current device.  No
 * counterpart in the reference (the upstream llama-server slots do this on the
 * host). */
int exl3cu_pack_ragged(size_t n_seq, const int32_t * d_want, const int32_t * d_pos, int32_t max_rows,
                       int32_t * d_row_offsets, int32_t * d_row_seq, int32_t * d_row_pos, void * stream);

/* The operator over a packed ragged batch: y[r] = x[r] . W for the
 * d_row_offsets[n_seq] rows that the packer (or the caller) wrote, a count read
 * on the device, so one captured CUDA graph serves batches of any size up to
 * max_rows; rows of y at or past the count are not written.  Runs on the
 * tensor-core GEMM.  Rows are independent, so the result equals
 * exl3cu_mul_mat over the same rows. */
int exl3cu_mul_mat_ragged(const exl3cu_weight * w, const void * d_x, int x_dtype, size_t x_row_stride,
                          const int32_t * d_row_offsets, size_t n_seq, size_t max_rows, float * d_y,
                          size_t y_row_stride, void * stream);

/* Plan overrides of the batched path, process-wide (for tuning).  Operands of
 * at least `min_rows` rows run on the tensor-core GEMM (tcgen05, decoded
 * weights and accumulators in TMEM; default 5), smaller ones on the decode
 * GEMV.  `tokens_per_cta` (a multiple of 32 up to 256: the MMA's N) and
 * `splits` (1, 2, 4, 8 or 16 CTAs of a cluster along K) replace the automatic
 * plan; 0 leaves a value automatic, min_rows 0 leaves it unchanged.  No
 * counterpart in the reference (its DSP operator fixes its row chunking,
 * src/exl3-htp.c:165-171). */
int exl3cu_gemm_config(size_t min_rows, int tokens_per_cta, int splits);

/* Sticky error bits the kernels of `device` raised since the last clear:
 * bit 0 = a bounded wait on an asynchronous copy ran out (the results of the
 * calls since are unreliable); bit 1 = exl3cu_get_rows read an id outside the
 * handle's columns (that row was filled with NaN).  Synchronises the device.  No counterpart in
 * the reference (its DSP operator returns statuses synchronously). */
int exl3cu_device_status(int device, unsigned * status, int clear);

/* Bytes of split-K workspace exl3cu_mul_mat_ws needs for this handle (any rows). */
size_t exl3cu_mul_mat_workspace_bytes(const exl3cu_weight * w);

/* The operator with its K split reduced through a caller-owned global workspace
 * of at least exl3cu_mul_mat_workspace_bytes(w) bytes, zero-filled once before
 * its first use (the operator leaves it zeroed again): the last CTA of each
 * column block to arrive sums the partials.  Same results as exl3cu_mul_mat
 * within rounding. */
int exl3cu_mul_mat_ws(const exl3cu_weight * w, const void * d_x, int x_dtype, size_t rows, size_t x_row_stride,
                      float * d_y, size_t y_row_stride, void * d_workspace, size_t workspace_bytes, void * stream);

/* Host-buffer form: copies x to the device, runs the operator, copies y back.
 * With synchronize != 0 it returns after y is in h_y (the ggml operator's
 * contract); otherwise the copies are only stream-ordered and h_x/h_y should be
 * pinned.  Staging buffers are owned by the handle. */
int exl3cu_mul_mat_host(exl3cu_weight * w, const void * h_x, int x_dtype, size_t rows, size_t x_row_stride,
                        float * h_y, size_t y_row_stride, int synchronize, void * stream);

/* EXL3 get_rows (replaces ggml_exl3_get_rows, src/exl3-ggml.cpp:19-49; the
 * reference patch dispatches GET_ROWS on an EXL3 src0 to it,
 * patches/llama-exl3.patch:114-121): for each of `count` column ids (local to
 * the handle's column range), writes the original-basis column W[:, id] -- k
 * values, each the fp16 the reference's exl3::reconstruct produces, widened to
 * f32 -- to d_out + i * out_row_stride.  This is the tied-embedding lookup:
 * token id -> hidden vector.  One CTA per (id, 128-row group).  count <= 65535.
 * Stream-ordered; ids are read on the device, and an id out of range yields a
 * NaN row and sets bit 1 of exl3cu_device_status. */
int exl3cu_get_rows(const exl3cu_weight * w, const int32_t * d_ids, size_t count, float * d_out,
                    size_t out_row_stride, void * stream);

/* Host-buffer form of exl3cu_get_rows (the ggml CPU-backend contract): checks
 * every id on the host first (EXL3CU_INVALID_ARGUMENT naming the first bad one,
 * where the reference asserts), stages ids and rows in the handle's buffers. */
int exl3cu_get_rows_host(exl3cu_weight * w, const int32_t * h_ids, size_t count, float * h_out,
                         size_t out_row_stride, int synchronize, void * stream);

/* No counterpart in the reference.  exl3cu_mul_mat for callers that may not
 * allocate device memory: the split-K scratch is a fixed 4 MiB array inside the
 * library (per GPU, for the life of the process) instead of a workspace.  The
 * first call on a device resolves that array's address (make it before any
 * stream capture); every call clears the part it needs first; calls that
 * overlap on the GPU share the array and race, so order them on one stream.
 * The resolved address is cached per device for the life of the process: do
 * not use this entry across a cudaDeviceReset of that device.
 * Returns EXL3CU_NO_SUPPORT when the weight's split-K plan needs more than the
 * array holds. */
int exl3cu_mul_mat_noalloc(const exl3cu_weight * w, const void * d_x, int x_dtype, size_t rows, size_t x_row_stride,
                           float * d_y, size_t y_row_stride, void * stream);

/* ------------------------------------------------------------------------
 * Peer-memory exchange for the column-split operator (2..8 GPUs of one node,
 * one process per GPU).  No counterpart in the reference: its operator splits
 * output column blocks over CPU threads of one process (src/exl3-ggml.cpp:74);
 * here each GPU computes a contiguous range of column blocks and the slices
 * meet over NVLink without a collective library.
 *
 * exl3cu_ipc_alloc: zero-filled device memory on `device` that peers can map;
 *   writes its 64-byte CUDA IPC handle to out_handle.
 * exl3cu_ipc_open / exl3cu_ipc_close: map / unmap a peer's buffer (from
 *   another process) on `device`.
 * Exchange protocol: a rank's y buffer holds 8-byte words (epoch << 32 |
 *   float bits), two halves of rows_cap x y_row_stride words each (y_half
 *   words apart); its state words (16, zero-initialised) hold an arrival
 *   ticket [8] and the rank's epoch counter [9].  The E-th call (E = counter
 *   + 1, read on the device) writes half (E & 1).  Every word is stored with
 *   one single-copy-atomic 8-byte store, so no fence or flag is needed: a
 *   reader waits until each word carries this call's epoch.
 * exl3cu_store_peers: rows x cols floats of this rank's slice (row stride
 *   slice_stride) go as (E, value) words into half (E & 1) of every rank's y
 *   buffer at column y_col0 (row stride y_row_stride).
 * exl3cu_mul_mat_peers: the operator of this rank's slice (handle w) with the
 *   store above, fused for mul1 weights: the GEMV's epilogue (1..4 rows) or
 *   the tensor-core GEMM's epilogue (5..2048 rows) stores its output blocks
 *   to the peers over NVLink.  Other operands run the operator into d_slice
 *   (row stride slice_stride) and then exl3cu_store_peers.
 * exl3cu_wait_peers: on the stream, waits until every word of rows x cols in
 *   half (E & 1) of this rank's y carries epoch E, copies the values into
 *   d_out (row stride out_row_stride; NULL: wait only) and advances the
 *   counter.  Bounded: after about a second it sets bit 0 of
 *   exl3cu_device_status, copies what is there and returns.
 * A rank can be at most one call ahead of another, since its next store
 * follows its wait for this call.  All of them read the epoch on the device,
 * so a call sequence can be captured in a CUDA graph and replayed.  Columns,
 * strides and offsets are multiples of 4; npeers <= 8. */
int exl3cu_ipc_alloc(int device, size_t bytes, void ** out_ptr, void * out_handle);
int exl3cu_ipc_free(int device, void * ptr);
int exl3cu_ipc_open(int device, const void * handle, void ** out_ptr);
int exl3cu_ipc_close(int device, void * ptr);
int exl3cu_store_peers(const float * d_slice, size_t rows, size_t cols, size_t slice_stride, int npeers,
                       void * const * d_y_peers, size_t y_row_stride, size_t y_half, size_t y_col0,
                       const unsigned * d_state, void * stream);
int exl3cu_wait_peers(unsigned * d_state, const void * d_y, size_t y_row_stride, size_t y_half, float * d_out,
                      size_t out_row_stride, size_t rows, size_t cols, void * stream);
int exl3cu_mul_mat_peers(const exl3cu_weight * w, const void * d_x, int x_dtype, size_t rows, size_t x_row_stride,
                         float * d_slice, size_t slice_stride, int npeers, void * const * d_y_peers,
                         size_t y_row_stride, size_t y_half, size_t y_col0, const unsigned * d_state, void * stream);

/* ------------------------------------------------------------------------
 * Model loader (replaces exl3::Model's constructor, src/exl3_model.cpp:79-157,
 * and extends it from the tied head to every EXL3 matrix).
 *
 * exl3cu_model_open reads <directory>/model.safetensors and
 * <directory>/hexagon-exl3.json and applies exl3::Model's checks in its order
 * and with its messages (spans, dtypes, manifest, <= 5.0 bits-per-weight
 * budget, head geometry, codebook markers); any failure returns
 * EXL3CU_INVALID_ARGUMENT with that message.  Then, on `device`:
 *   - every X.trellis (3-D I16, 16*bits last dimension) with F16 X.suh/X.svh
 *     becomes a persistent weight handle at its own bit width (mixed-bit
 *     models), codebook from its X.mul1 / X.mcg marker;
 *   - every other tensor is copied into one device arena.
 * With flags = EXL3CU_MODEL_VALIDATE_ONLY nothing touches a GPU and weight and
 * tensor pointers read back as NULL.  The weight handles belong to the model:
 * exl3cu_weight_free refuses them; exl3cu_model_free releases everything.
 * Matrices and tensors are indexed in name order. */
int exl3cu_model_open(const char * directory, int device, unsigned flags, exl3cu_model ** out);
int exl3cu_model_free(exl3cu_model * m);
/* tensor_count / payload_bytes / hidden_size / vocab_size / bits_per_weight are
 * exl3::Model's accessors (src/exl3_model.cpp:162-166); any pointer may be NULL. */
int exl3cu_model_info(const exl3cu_model * m, size_t * tensor_count, size_t * payload_bytes, size_t * hidden_size,
                      size_t * vocab_size, size_t * parameter_count, double * bits_per_weight);
size_t exl3cu_model_matrix_count(const exl3cu_model * m);
/* Matrix `index`: its name (the X of X.trellis; valid while m lives), shape,
 * bit width, codebook and weight handle. */
int exl3cu_model_matrix(const exl3cu_model * m, size_t index, const char ** name, size_t * k, size_t * n,
                        unsigned * bits, unsigned * codebook, exl3cu_weight ** weight);
int exl3cu_model_find_matrix(const exl3cu_model * m, const char * name, size_t * index);
/* Matrix index of the tied head (input_embedding.source). */
int exl3cu_model_head(const exl3cu_model * m, size_t * index);
/* Tensor `index` (0 .. tensor_count-1): name, storage dtype, shape, bytes, and
 * its device copy (NULL for the parts of an EXL3 matrix, which live in the
 * weight handle, and for validate-only models). */
int exl3cu_model_tensor(const exl3cu_model * m, size_t index, const char ** name, int * dtype, size_t * ndim,
                        const size_t ** shape, size_t * bytes, void ** d_data);
int exl3cu_model_find_tensor(const exl3cu_model * m, const char * name, size_t * index);
/* exl3::Model::embedding (src/exl3_model.cpp:168-187): the hidden_size fp16
 * values of token's original-basis column of the tied head, into host memory.
 * Synchronous.  token >= vocab_size -> EXL3CU_INVALID_ARGUMENT. */
int exl3cu_model_embedding(exl3cu_model * m, uint32_t token, uint16_t * h_out);
/* Batched, stream-ordered form on the device: exl3cu_get_rows on the head. */
int exl3cu_model_embed(const exl3cu_model * m, const int32_t * d_ids, size_t count, float * d_out,
                       size_t out_row_stride, void * stream);

#ifdef __cplusplus
}
#endif

#endif /* EXL3CU_H */
