/* Hybrid-decoder layer kernels around the EXL3 operator (libexl3cu).
 *
 * No counterpart in the reference tree: its model graph (attention, the gated
 * delta net, norms, the head) is upstream llama.cpp's, reached through its
 * patch (patches/llama-exl3.patch:175-183 routes FLASH_ATTN_EXT /
 * GATED_DELTA_NET).  These entries are the B200 side of that graph for a
 * Qwen3.5-style 3:1 gated-delta-rule / full-attention decoder with 16 heads of
 * 128 (4 kv heads), driven by a host scheduler that packs ragged steps with
 * exl3cu_pack_ragged.  All pointers are device pointers on the current device;
 * calls are stream-ordered; fp16 buffers (KV cache, embedding, gate rows) are
 * passed as uint16_t; activations are f32.
 *
 * Row conventions: row r of a step belongs to step sequence row_seq[r] at
 * position row_pos[r]; step sequence s uses cache slot seq_slot[s] (0 ..
 * n_slots-1) and rows [row_offsets[s], row_offsets[s+1]).
 */
#ifndef EXL3CU_HYBRID_H
#define EXL3CU_HYBRID_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* h[r] = fp32(table[ids[r]]) for an fp16 [vocab, hidden] table (ids outside give zeros).
 * With d_h_sumsq (hidden a multiple of 128) also each row's sums of squares per
 * 128-block, f32 [rows][hidden/128], the form exl3cu_mul_mat_batch_ex's
 * RMSNorm input takes. */
int exl3cu_hyb_embed(const uint16_t * d_table, int vocab, const int32_t * d_ids, int rows, int hidden, float * d_h,
                     float * d_h_sumsq, void * stream);

/* h += delta (when d_delta is not NULL, row stride delta_stride), then
 * out = h * rsqrt(mean(h^2) + eps) * w, per row of `hidden` values (f32). */
int exl3cu_hyb_rmsnorm(float * d_h, const float * d_delta, int delta_stride, const float * d_w, float eps, int rows,
                       int hidden, float * d_out, void * stream);

/* out = silu(gate) * up with gu rows [gate (ffn) | up (ffn)] (f32). */
int exl3cu_hyb_swiglu(const float * d_gu, int rows, int ffn, float * d_out, void * stream);

/* Full-attention prologue: qkv rows [q 16x128 | k 4x128 | v 4x128] (f32);
 * per-head RMSNorm of q and k (weights qn_w / kn_w [128], eps), rotary
 * embedding on pairs (i, i+64) at angle row_pos * inv_freq[i] (i < 64), k and
 * v appended to the fp16 caches [n_slots][4][max_len][128] at the row's
 * position, q written to d_q [rows][16*128] (f32).  Rows whose position or
 * slot lies outside the caches are skipped. */
int exl3cu_hyb_attn_prep(const float * d_qkv, int rows, const int32_t * d_row_seq, const int32_t * d_row_pos,
                         const int32_t * d_seq_slot, const float * d_qn_w, const float * d_kn_w,
                         const float * d_inv_freq, float eps, uint16_t * d_kcache, uint16_t * d_vcache, int max_len,
                         int n_slots, float * d_q, void * stream);

/* GQA attention of each row's 16 q heads over positions 0..row_pos of its
 * sequence (4 q heads per kv head), softmax(q.k * scale); out f32 [rows][16*128].
 * splits > 1 divides each row's positions over that many CTAs (flash-decoding);
 * it needs d_part of exl3cu_hyb_attn_scratch_bytes(rows, splits) bytes and
 * d_tickets of rows*16 unsigned, zero before the first call (the kernel leaves
 * them zero). */
size_t exl3cu_hyb_attn_scratch_bytes(int rows, int splits);
int exl3cu_hyb_attn(const float * d_q, int rows, const int32_t * d_row_seq, const int32_t * d_row_pos,
                    const int32_t * d_seq_slot, const uint16_t * d_kcache, const uint16_t * d_vcache, int max_len,
                    int n_slots, float scale, int splits, float * d_part, size_t part_bytes, unsigned * d_tickets,
                    float * d_out, void * stream);

/* exl3cu_hyb_attn_prep and exl3cu_hyb_attn in one launch, for a step in which
 * every sequence has exactly one row (decode): d_qkv holds the packed
 * [q | k | v] rows of exl3cu_hyb_attn_prep, the new k and v are appended to
 * the caches at row_pos and used from on-chip memory, and the result equals the
 * two calls' bit for bit.  With two rows of one sequence in the step, a row
 * would miss the other's new position: use the two calls. */
int exl3cu_hyb_attn_decode(const float * d_qkv, int rows, const int32_t * d_row_seq, const int32_t * d_row_pos,
                           const int32_t * d_seq_slot, const float * d_qn_w, const float * d_kn_w,
                           const float * d_inv_freq, float eps, uint16_t * d_kcache, uint16_t * d_vcache, int max_len,
                           int n_slots, float scale, int splits, float * d_part, size_t part_bytes,
                           unsigned * d_tickets, float * d_out, void * stream);

/* Dynamic shared memory one exl3cu_hyb_gdn CTA uses (the 128x128 state and scratch). */
size_t exl3cu_hyb_gdn_smem_bytes(void);

/* Gated delta rule over each step sequence's rows in order, per head:
 *   qkvz rows [q | k | v | z] (4 x 16 x 128, f32, the projections' outputs);
 *   xn: the layer's normed input rows, f32 (for the gate projections); or,
 *       with xn_norm_w, the residual-stream rows h, normalised here with
 *       weights xn_norm_w [hidden] and eps (RMSNorm folded into the gates);
 *   wab: fp16 [32][hidden], rows 0..15 W_a, 16..31 W_b;
 *   conv_w f32 [3*2048][4], conv_state f32 [n_slots][3*2048][3] (last three inputs);
 *   A_log, dt_bias f32 [16]; norm_w f32 [128]; state f32 [n_slots][16][128 (k)][128 (v)].
 * Writes f32 [rows][16*128] = RMSNorm(o_head) * norm_w * silu(z_head). */
int exl3cu_hyb_gdn(const float * d_qkvz, const float * d_xn, const float * d_xn_norm_w, const uint16_t * d_wab,
                   int hidden,
                   const float * d_conv_w, float * d_conv_state, const float * d_A_log, const float * d_dt_bias,
                   const float * d_norm_w, float eps, float * d_state, const int32_t * d_row_offsets,
                   const int32_t * d_seq_slot, int n_seq, int n_slots, float * d_out, void * stream);

/* Tied fp16 head with greedy choice, one launch: for o < nout (<= 8),
 * logits[o][v] = sum_i x[rows[o]][i] * embed[v][i] (f32 x, fp32 sums; written
 * when d_logits is not NULL), tokens[o] = argmax_v (lowest index on ties).
 * x = d_xn, or with d_norm_w the final RMSNorm of d_xn's rows (weights
 * d_norm_w, eps) computed on load, equal bit for bit to exl3cu_hyb_rmsnorm
 * followed by this call.  d_best: 9 64-bit scratch words, zero before the
 * first call; every call leaves them zero.  hidden is 1024, 2048, 4096 or
 * 8192. */
int exl3cu_hyb_head(const float * d_xn, const int32_t * d_rows, int nout, int hidden, const float * d_norm_w,
                    float eps, const uint16_t * d_embed, int vocab, float * d_logits, unsigned long long * d_best,
                    int32_t * d_tokens, void * stream);

/* exl3cu_hyb_head for replayed decode steps with the token feedback on the
 * device, one launch: besides d_tokens, the last CTA writes row o's token into
 * d_next_tokens[o] (the next step's token ids), adds 1 to d_next_pos[o] (its
 * positions), stores it at d_log[*d_counter * nout + o] (clamped to
 * log_capacity - 1) and adds 1 to *d_counter.  No logits are written. */
int exl3cu_hyb_head_feedback(const float * d_xn, const int32_t * d_rows, int nout, int hidden, const float * d_norm_w,
                             float eps, const uint16_t * d_embed, int vocab, unsigned long long * d_best,
                             int32_t * d_tokens, int32_t * d_next_tokens, int32_t * d_next_pos, int32_t * d_log,
                             int64_t * d_counter, size_t log_capacity, void * stream);

/* Sticky error bits of these kernels on the current device (reserved: the
 * current kernels wait on nothing and raise none).  Synchronises the device. */
int exl3cu_hyb_status(int clear, unsigned * status);

#ifdef __cplusplus
}
#endif

#endif /* EXL3CU_HYBRID_H */
