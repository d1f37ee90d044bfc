/*
 * EXL3 runtime-record format constants and the ggml operator entry points.
 *
 * Same names and values as the reference's include/exl3-block.h:1-50 for the
 * format it defines: ggml type ids 43/44/45 (patches/llama-exl3.patch:10-13),
 * 128-wide groups, group records of 2048*bits + 512 bytes (64 trellis tiles in
 * order r*8+c, then suh[128] and svh[128] fp16), record (nb,kb) at index
 * nb*(k/128)+kb.  The Hexagon VTCM planners of that header have no B200
 * meaning and are not provided.
 *
 * ggml_exl3_mul_mat / ggml_exl3_get_rows keep the reference's signatures
 * (include/exl3-block.h:41-50); this library's implementations run on the GPU
 * through the exl3cu C ABI (include/exl3cu.h).
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#define EXL3_TYPE_4 43
#define EXL3_TYPE_6 44
#define EXL3_TYPE_8 45
#define EXL3_GROUP_DIM 128

static inline unsigned exl3_type_bits(unsigned type) {
    return type == EXL3_TYPE_4 ? 4 : type == EXL3_TYPE_6 ? 6 : type == EXL3_TYPE_8 ? 8 : 0;
}
static inline size_t exl3_group_bytes(unsigned bits) { return 2048u * bits + 512u; }
static inline const uint16_t * exl3_group_su(const void * group, unsigned bits) {
    return (const uint16_t *) ((const unsigned char *) group + 2048u * bits);
}
static inline const uint16_t * exl3_group_sv(const void * group, unsigned bits) {
    return (const uint16_t *) ((const unsigned char *) group + 2048u * bits + 256u);
}

struct ggml_compute_params;
struct ggml_tensor;
#ifdef __cplusplus
extern "C" {
#endif
void ggml_exl3_mul_mat(const struct ggml_compute_params * params, struct ggml_tensor * dst);
void ggml_exl3_get_rows(const struct ggml_compute_params * params, struct ggml_tensor * dst);
/* No counterpart in the reference (whose CPU operator keeps no device state):
 * frees every weight the two operators above uploaded to the GPU.  Call it
 * when a model is unloaded; later calls upload again on first sight. */
void ggml_exl3_release_weights(void);
#ifdef __cplusplus
}
#endif
