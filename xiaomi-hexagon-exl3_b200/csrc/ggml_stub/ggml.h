/*
 * Minimal stand-in for upstream ggml.h, used only when exl3_ggml_cuda.cpp is
 * built outside a llama.cpp tree (this repository's standalone build and its
 * tests).  Inside llama.cpp the real ggml.h is found first and this file is
 * not used.  It declares just the members the EXL3 operator reads
 * (type, ne, nb, src, data) under upstream's names, with upstream's type ids
 * for F32/F16/I32 and the reference patch's EXL3_4/6/8 = 43/44/45
 * (patches/llama-exl3.patch:10-13).
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

static inline int64_t ggml_nrows(const struct ggml_tensor * t) { return t->ne[1] * t->ne[2] * t->ne[3]; }
static inline int64_t ggml_nelements(const struct ggml_tensor * t) {
    return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3];
}

#define GGML_ASSERT(x)                                                                     \
    do {                                                                                   \
        if (!(x)) {                                                                        \
            fprintf(stderr, "GGML_ASSERT(%s) failed at %s:%d\n", #x, __FILE__, __LINE__); \
            abort();                                                                       \
        }                                                                                  \
    } while (0)

#ifdef __cplusplus
}
#endif
