// Internal declarations shared by the CUDA sources and the C-ABI layer.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "vireo_status.h"

namespace vireo {

struct StageGeom;
struct MoeDecodeParams;

// elements / bytes per block for the types this library reads (GGUF wire
// sizes, vireo src/gguf.c:27-38); 0 on success
inline int type_block(uint32_t t, int* be, int* bb) {
  switch (t) {
    case 0: *be = 1; *bb = 4; return 0;      // F32
    case 1: *be = 1; *bb = 2; return 0;      // F16
    case 6: *be = 32; *bb = 22; return 0;    // Q5_0
    case 8: *be = 32; *bb = 34; return 0;    // Q8_0
    case 12: *be = 256; *bb = 144; return 0; // Q4_K
    case 14: *be = 256; *bb = 210; return 0; // Q6_K
    default: return -1;
  }
}
inline uint64_t row_bytes(uint32_t t, int n) {
  int be, bb;
  if (type_block(t, &be, &bb)) return 0;
  return (uint64_t)(n / be) * (uint64_t)bb;
}

struct GemvParams;

bool fast_format(uint32_t type);
int stage_geom(uint32_t type, int K, StageGeom* sg);
const void* moe_decode_kernel_for(uint32_t gtype, uint32_t dtype, bool routed = false);
uint32_t moe_decode_layout(MoeDecodeParams* p, uint32_t smem_limit, int grid);
const void* gemv_kernel_for(uint32_t type);
uint32_t gemv_layout(GemvParams* p, uint32_t smem_limit, int max_units);

// batched (prefill) MoE FFN, prefill.cu
struct PrefillLayer {
  int d, fe, ne, k, renorm;
  const float* router;             // [ne][d] fp32
  const uint8_t* const* exp_tab;   // device [ne][3]: gate, up, down
  const int* own = nullptr;        // device [ne]: experts this handle computes (null = all)
};
struct PrefillScratch {
  __half* xa = nullptr;
  int32_t* ids = nullptr;
  float* wts = nullptr;
  int* counts = nullptr;
  int* cursor = nullptr;
  struct PTile* tiles = nullptr;
  int* n_mtiles = nullptr;
  int* ysrc = nullptr;     // [rows]: token slot (t * k + i) of each placed row
  float* wrow = nullptr;
  __half* xg = nullptr;
  __half* hg = nullptr;
  __half* yret = nullptr;  // [T * k][d]: each token slot's weighted expert output, f16
  __half* r2 = nullptr;
  __half* minmat = nullptr;  // Q4_K min block of every gate/up row (depends on the expert pointers)
  uint8_t* gu_pack = nullptr;  // repacked gate/up and down weight chunks (likewise)
  uint8_t* dn_pack = nullptr;
  bool minmat_ok = false;
  size_t c_xa = 0, c_ids = 0, c_wts = 0, c_counts = 0, c_cursor = 0, c_tiles = 0, c_n_mtiles = 0, c_ysrc = 0,
         c_wrow = 0, c_xg = 0, c_hg = 0, c_yret = 0, c_r2 = 0, c_minmat = 0, c_gu_pack = 0, c_dn_pack = 0;
};
int prefill_supported(int d, int fe, int ne, int k, uint32_t rt, uint32_t gt, uint32_t ut, uint32_t dt);
int prefill_run(const PrefillLayer& L, PrefillScratch* S, const void* hb_bf16, float* x, int T, const float* bias,
                int32_t* ids_out, float* wts_out, int* d_err, int num_sms, cudaStream_t st);
void prefill_scratch_free(PrefillScratch* s);
// pieces of prefill_run, shared with the expert-parallel path (ep.cu)
int prefill_kx(int d);
int prefill_prepare(const PrefillLayer& L, PrefillScratch* S, cudaStream_t st);
int prefill_route(const PrefillLayer& L, PrefillScratch* S, const void* hb, int T, const float* bias, int* d_err,
                  int num_sms, cudaStream_t st);
size_t prefill_row_capacity(size_t pairs, int ne);
int prefill_grow_rows(const PrefillLayer& L, PrefillScratch* S, size_t rows);
void prefill_scan_launch(const int* counts, int ne, PrefillScratch* S, cudaStream_t st);
// ysrc / ypeer: where row r's output goes, as f16: rank ysrc[r] >> 24's
// ypeer buffer, row ysrc[r] & 0xFFFFFF (a single-GPU call passes its own
// map and S->yret as the only peer; npeers > 1 means peer memory)
int prefill_experts(const PrefillLayer& L, PrefillScratch* S, size_t rows, int* d_err, int num_sms, cudaStream_t st,
                    const int* ysrc, __half* const* ypeer, int npeers);
// expert-parallel owner: row r of S->xg (over the M tiles prefill_scan laid
// out for `rows` rows) <- xr row xsrc[r] where xsrc[r] is in [0, n_slots)
void prefill_expand_launch(const PrefillScratch* S, size_t rows, const int* xsrc, const __half* xr, int Kx,
                           int n_slots, cudaStream_t st);
// x[t] += sum in slot order of yret[t * k + i] (slots whose id is -1 skipped)
void prefill_combine_launch(const int32_t* ids, const __half* yret, float* x, int T, int k, int d, cudaStream_t st);
int prefill_tile_rows();  // rows per activation tile (row ranges per expert are padded to it)

// generic kernels (any supported type/shape), generic_kernels.cu
int launch_dequant(uint32_t type, const void* src, float* dst, int n, cudaStream_t s);
int launch_gemv_generic(uint32_t type, const void* w, const float* x, float* y, int n, int d, cudaStream_t s);
int launch_embed(uint32_t type, const void* table, const int32_t* token, int vocab, float* dst, int n, int* err,
                 cudaStream_t s);

// process-wide device context
struct HostRange {
  const uint8_t* host;
  uint64_t bytes;
  uint8_t* dev;
};

struct Ctx {
  int device = -1;
  int num_sms = 0;
  uint32_t smem_optin = 0;
  cudaStream_t stream = nullptr;
  int* d_err = nullptr;   // device status word for stand-alone calls
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  std::vector<HostRange> ranges;
  std::mutex mu;
};

Ctx* ctx_get(int* status);
void set_last_error(int code);
int cuda_status(cudaError_t e);
void* ctx_scratch(Ctx* c, size_t bytes);  // grows, caller holds c->mu

// device-pointer GEMV with the fast path when possible
int gemv_dev(Ctx* c, uint32_t type, const void* w, const float* x, float* y, int n, int d, cudaStream_t s);
// The fast path only (VIREO_ERR_UNSUPPORTED when the type, shape or
// alignment rules it out): y = W . rmsnorm(x, norm_w, eps) when norm_w is
// set (x * (1 / sqrt(mean(x^2) + eps)) * norm_w), and an L2 prefetch of up
// to prefetch_bytes of each CTA's weight rows before the kernel waits on its
// predecessor on the stream.
int gemv_dev_fast(Ctx* c, uint32_t type, const void* w, const float* x, float* y, int n, int d, cudaStream_t s,
                  const float* norm_w, float eps, uint32_t prefetch_bytes);

}  // namespace vireo
