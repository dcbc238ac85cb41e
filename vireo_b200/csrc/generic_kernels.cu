// Element-wise dequantisation and the general (any type, any shape) GEMV.
//
// deq_elem reproduces the reference's per-value arithmetic exactly
// (vireo src/gguf_compute.c:17-124): the same products in the same order,
// each rounded separately (the reference is compiled without FMA
// contraction), so gguf_dequant_row on the device is bit-identical to the
// reference's.  The general GEMV (one warp per output row) serves the
// shapes and types the tensor-core path does not take: F32/F16/Q5_0
// weights, K not a multiple of 256, d not a multiple of 16.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "quant_frag.cuh"
#include "vireo_internal.h"

namespace vireo {

__device__ __forceinline__ float f16_at(const uint8_t* p) {
  uint16_t h = (uint16_t)p[0] | ((uint16_t)p[1] << 8);
  return __half2float(__ushort_as_half(h));
}

// value i of a row stored in the given block format
__device__ __forceinline__ float deq_elem(uint32_t type, const uint8_t* row, int i) {
  switch (type) {
    case T_F32: {
      const uint8_t* p = row + 4 * (size_t)i;
      uint32_t b = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
      return __uint_as_float(b);
    }
    case T_F16:
      return f16_at(row + 2 * (size_t)i);
    case T_Q8_0: {
      const uint8_t* b = row + 34 * (size_t)(i >> 5);
      return __fmul_rn((float)(int8_t)b[2 + (i & 31)], f16_at(b));
    }
    case T_Q5_0: {
      const uint8_t* b = row + 22 * (size_t)(i >> 5);
      const int j = i & 31;
      const uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
      const uint32_t nib = (j < 16) ? (b[6 + j] & 15u) : (b[6 + j - 16] >> 4);
      const int q = (int)(nib | (((qh >> j) & 1u) << 4)) - 16;
      return __fmul_rn((float)q, f16_at(b));
    }
    case T_Q4_K: {
      const uint8_t* b = row + 144 * (size_t)(i >> 8);
      const int r = i & 255, c = r >> 6, hi = (r >> 5) & 1, l = r & 31;
      const uint8_t qb = b[16 + 32 * c + l];
      const uint32_t q = hi ? (qb >> 4) : (qb & 15u);
      const int j = 2 * c + hi;
      const uint8_t* s = b + 4;
      uint32_t sc, mn;
      if (j < 4) {
        sc = s[j] & 63u;
        mn = s[j + 4] & 63u;
      } else {
        sc = (s[j + 4] & 15u) | ((uint32_t)(s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
      }
      const float dl = __fmul_rn(f16_at(b), (float)sc), ml = __fmul_rn(f16_at(b + 2), (float)mn);
      return __fsub_rn(__fmul_rn(dl, (float)q), ml);
    }
    case T_Q6_K: {
      const uint8_t* b = row + 210 * (size_t)(i >> 8);
      const int r = i & 255, h = r >> 7, rr = r & 127, st = rr >> 5, l = rr & 31;
      const uint8_t qlb = b[64 * h + l + 32 * (st & 1)];
      const uint32_t nib = (st >> 1) ? (qlb >> 4) : (qlb & 15u);
      const uint32_t hb = (b[128 + 32 * h + l] >> (2 * st)) & 3u;
      const int q = (int)(nib | (hb << 4)) - 32;
      const int sc = (int)(int8_t)b[192 + 8 * h + 2 * st + (l >> 4)];
      return __fmul_rn(__fmul_rn(f16_at(b + 208), (float)sc), (float)q);
    }
    default:
      return 0.f;
  }
}

__global__ void dequant_kernel(uint32_t type, const uint8_t* src, float* dst, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    dst[i] = deq_elem(type, src, i);
}

// one row of an embedding table, the row index read from device memory
// (a token id another kernel wrote, e.g. the previous step's argmax); an id
// outside [0, vocab) gives zeros and records VIREO_ERR_ARG
__global__ void embed_kernel(uint32_t type, const uint8_t* table, uint64_t rb, const int32_t* token, int vocab,
                             float* dst, int n, int* err) {
  const int t = *token;
  const bool ok = t >= 0 && t < vocab;
  if (!ok && blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(err, 0, VIREO_ERR_ARG);
  const uint8_t* row = table + (ok ? (uint64_t)t * rb : 0);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    dst[i] = ok ? deq_elem(type, row, i) : 0.f;
}

// one warp per row; lanes stride over K, then a fixed xor-tree reduction
__global__ void gemv_generic_kernel(uint32_t type, const uint8_t* w, const float* x, float* y, int n, int d,
                                    uint64_t rb) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= d) return;
  const uint8_t* r = w + (uint64_t)row * rb;
  float acc = 0.f;
  for (int i = lane; i < n; i += 32) acc = fmaf(deq_elem(type, r, i), __ldg(x + i), acc);
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) y[row] = acc;
}

int launch_dequant(uint32_t type, const void* src, float* dst, int n, cudaStream_t s) {
  int be, bb;
  if (type_block(type, &be, &bb) || n < 0 || n % be) return VIREO_ERR_UNSUPPORTED;
  if (n == 0) return VIREO_OK;
  int blocks = (n + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  dequant_kernel<<<blocks, 256, 0, s>>>(type, (const uint8_t*)src, dst, n);
  return cuda_status(cudaGetLastError());
}

int launch_embed(uint32_t type, const void* table, const int32_t* token, int vocab, float* dst, int n, int* err,
                 cudaStream_t s) {
  int be, bb;
  if (type_block(type, &be, &bb) || n <= 0 || n % be) return VIREO_ERR_UNSUPPORTED;
  embed_kernel<<<(n + 255) / 256, 256, 0, s>>>(type, (const uint8_t*)table, row_bytes(type, n), token, vocab, dst, n,
                                               err);
  return cuda_status(cudaGetLastError());
}

int launch_gemv_generic(uint32_t type, const void* w, const float* x, float* y, int n, int d, cudaStream_t s) {
  int be, bb;
  if (type_block(type, &be, &bb) || n <= 0 || d < 0 || n % be) return VIREO_ERR_UNSUPPORTED;
  if (d == 0) return VIREO_OK;
  const int rows_per_block = 8;
  gemv_generic_kernel<<<(d + rows_per_block - 1) / rows_per_block, 32 * rows_per_block, 0, s>>>(
      type, (const uint8_t*)w, x, y, n, d, row_bytes(type, n));
  return cuda_status(cudaGetLastError());
}

}  // namespace vireo
