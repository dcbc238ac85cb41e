/* vireo-b200: GGUF dequantisation and quantised mat-vec on B200 (sm_100a).
 *
 * Drop-in for the reference's gguf_compute.h (vireo src/gguf_compute.h:8-10):
 * the three reference functions keep their names and signatures; their
 * pointers may be host or device pointers (host buffers are staged through
 * the device; weights in a range registered with gguf_weights_register are
 * read from their device copy).  The reference functions return nothing;
 * vireo_last_error() reports the status of the calling thread's last call.
 * The *_dev variants take device pointers only and run asynchronously on
 * the given CUDA stream (cudaStream_t passed as void*, NULL = the library's
 * own stream). */
#ifndef VIREO_GGUF_COMPUTE_H
#define VIREO_GGUF_COMPUTE_H
#include <stdint.h>

#include "gguf.h"
#include "vireo_status.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- reference interface -------------------------------------------------- */

/* replaces src/gguf_compute.c:17-36 (exact half -> float, host function) */
float gguf_f16_to_f32(uint16_t h);

/* replaces src/gguf_compute.c:105-124: n values of one row of the given type
 * (F32, F16, Q8_0, Q5_0, Q4_K, Q6_K) into dst, bit-identical to the
 * reference; other types leave dst untouched (status VIREO_ERR_UNSUPPORTED). */
void gguf_dequant_row(uint32_t type, const void *src, float *dst, int n);

/* replaces src/gguf_compute.c:159-214: y[o] = sum_i W[o,i] x[i], o < d, W =
 * w->data, d rows of n values in w->ggml_type.  Q8_0/Q4_K/Q6_K with
 * n % 256 == 0 and d % 16 == 0 run on the tensor-core streaming kernel;
 * every other supported shape/type on the general kernel.  Returns after y
 * is written (synchronous, like the reference). */
void gguf_matmul(float *y, const float *x, const gguf_tensor *w, int n, int d);

/* ---- extensions ------------------------------------------------------------ */

/* status of this thread's last gguf_* call (VIREO_OK or a VIREO_ERR_*) */
int vireo_last_error(void);
const char *vireo_status_string(int status);

/* select the CUDA device before the first call (default: current device) */
int vireo_device_init(int device);

/* device-pointer, stream-ordered variants (no host synchronisation) */
int gguf_matmul_dev(float *y, const float *x, const gguf_tensor *w, int n, int d, void *stream);
int gguf_dequant_row_dev(uint32_t type, const void *src, float *dst, int n, void *stream);

/* Upload a host byte range (e.g. the tensor data section of a mmap'd GGUF)
 * once; later calls whose weight pointer falls inside it use the device
 * copy.  Returns a status. */
int gguf_weights_register(const void *host, uint64_t nbytes);
int gguf_weights_unregister(const void *host);

/* wait for all work queued on stream (NULL = the library's stream) and
 * return the first device-side status recorded since the last call */
int vireo_sync(void *stream);

#ifdef __cplusplus
}
#endif
#endif
