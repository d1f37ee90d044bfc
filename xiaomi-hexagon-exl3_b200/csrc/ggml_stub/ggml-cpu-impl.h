/* Minimal stand-in for upstream ggml-cpu-impl.h (see ggml.h in this folder):
 * the per-op thread split the EXL3 operator reads. */
#pragma once
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

struct ggml_compute_params {
    int ith;
    int nth;
    size_t wsize;
    void * wdata;
};

#ifdef __cplusplus
}
#endif
