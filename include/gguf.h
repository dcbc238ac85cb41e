/* The GGUF types the vireo-b200 boundary uses.
 *
 * gguf_tensor is ABI-identical to the reference's (vireo src/gguf.h:36-45)
 * and the ggml type ids are the reference's wire enum (src/gguf.h:20-23), so
 * tensors built by the reference's gguf.c loader (or by moe_ffn, which fills
 * only data and ggml_type, src/gguf_run.c:202-204) pass through unchanged.
 * The include guard is the reference's: a translation unit that already
 * includes the reference's full gguf.h (loader API included) gets the same
 * definitions from it. */
#ifndef VIREO_GGUF_H
#define VIREO_GGUF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { GGML_F32=0, GGML_F16=1, GGML_Q4_0=2, GGML_Q4_1=3, GGML_Q5_0=6,
       GGML_Q5_1=7, GGML_Q8_0=8, GGML_Q8_1=9, GGML_Q2_K=10, GGML_Q3_K=11,
       GGML_Q4_K=12, GGML_Q5_K=13, GGML_Q6_K=14, GGML_Q8_K=15 };

typedef struct { const char *ptr; uint64_t len; } gguf_str;

typedef struct {
    gguf_str name;
    uint32_t n_dims;
    uint64_t dims[4];
    uint32_t ggml_type;
    uint64_t offset;       /* from data section start */
    const void *data;      /* host (mmap) or device pointer */
    uint64_t n_elems;
    uint64_t nbytes;
} gguf_tensor;

#ifdef __cplusplus
}
#endif
#endif
