/*
 * Test-infrastructure stand-in for upstream ggml-cpu-impl.h: the CPU thread
 * split (ith of nth) that the reference's src/exl3-ggml.cpp reads.  Never
 * linked into the shipped library.
 */
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
typedef struct ggml_compute_params ggml_compute_params;

#ifdef __cplusplus
}
#endif
