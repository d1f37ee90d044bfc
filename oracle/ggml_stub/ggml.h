/*
 * Test-infrastructure stand-in for upstream ggml.h, just large enough to compile
 * the reference's unmodified src/exl3-ggml.cpp (its CPU operator) into the
 * oracle library under oracle/_ref.  Only the members that file touches exist:
 * ggml_tensor::{type, ne, nb, src, data}, ggml_nrows, ggml_nelements and
 * GGML_ASSERT.  The type ids follow upstream ggml (F32=0, F16=1, I32=26) and
 * the llama.cpp patch of the reference (EXL3_4/6/8 = 43/44/45,
 * patches/llama-exl3.patch:10-13).
 *
 * Never linked into the shipped library.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#ifdef __cplusplus
extern "C" {
#endif

enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
    GGML_TYPE_I32 = 26,
    GGML_TYPE_EXL3_4 = 43,
    GGML_TYPE_EXL3_6 = 44,
    GGML_TYPE_EXL3_8 = 45,
};

#define GGML_MAX_DIMS 4
#define GGML_MAX_SRC 10

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[GGML_MAX_DIMS];
    size_t nb[GGML_MAX_DIMS];
    struct ggml_tensor * src[GGML_MAX_SRC];
    void * data;
};
typedef struct ggml_tensor ggml_tensor;

static inline int64_t ggml_nrows(const struct ggml_tensor * t) {
    return t->ne[1] * t->ne[2] * t->ne[3];
}

static inline int64_t ggml_nelements(const struct ggml_tensor * t) {
    return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3];
}

#define GGML_ASSERT(x)                                                          \
    do {                                                                        \
        if (!(x)) {                                                             \
            fprintf(stderr, "GGML_ASSERT(%s) failed at %s:%d\n", #x, __FILE__, \
                    __LINE__);                                                  \
            abort();                                                            \
        }                                                                       \
    } while (0)

#ifdef __cplusplus
}
#endif
