// gguf_moe_ffn_noalloc: the batch-1 MoE decode kernel for callers that may
// not allocate device memory.
//
// The launch is the one gguf_moe_ffn makes (same kernel, same parameters),
// except that the kernel's scratch (per-launch sync words, status word, tile
// counters, router partials, h, the experts' down outputs, the expert
// pointer table) lives in the file-scope array below instead of a
// cudaMalloc'd block, and the descriptor is taken per call instead of
// through a gguf_moe handle.  Nothing here calls cudaMalloc, cudaFree,
// stream creation or any allocating library routine.
//
// Set-up: the first call on a device (with that device current) takes the
// array's address with cudaGetSymbolAddress, reads the SM count and the
// shared-memory limit, and zeroes the array.  That first call must come
// before any stream capture.
//
// Every call first zeroes the words that must start at zero (the sync words,
// the status word and the tile counters; the kernel also puts the sync words
// and counters back), and uploads the expert pointer table.  Every call
// synchronises its stream before returning, also when a launch fails.  All calls on one device share the
// one array: calls whose work overlaps on the GPU (other streams, other host
// threads) race on it.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "gguf_moe.h"
#include "moe_decode.cuh"
#include "vireo_internal.h"

namespace vireo {
namespace {

// 256 KiB.  A layer needs the sync words (16.9 KiB), the status word, 128 B
// per 16 output rows of tile counters, 4 B per expert of router logits, 4 B
// per value of the k selected experts' h rows and of their d outputs, and
// 24 B per expert of pointers: 130.5 KiB for the OLMoE-shaped layer (d 2048,
// 64 experts top-8, fe 1024), 124.3 KiB for the Qwen3-shaped one.  A layer
// needing more is refused with VIREO_ERR_NOMEM.
constexpr size_t kNoAllocScratchBytes = 256 * 1024;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
struct DevSetup {
  bool done = false;
  uint8_t* scratch = nullptr;
  int num_sms = 0;
  uint32_t smem_limit = 0;
};
std::mutex g_setup_mu;
DevSetup g_setup[kMaxDevices];

size_t up256(size_t v) { return (v + 255) & ~(size_t)255; }

int device_setup(DevSetup** out) {
  int dev = -1;
  int st = cuda_status(cudaGetDevice(&dev));
  if (st) return st;
  if (dev < 0 || dev >= kMaxDevices) return VIREO_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lk(g_setup_mu);
  DevSetup& S = g_setup[dev];
  if (!S.done) {
    void* ptr = nullptr;
    if ((st = cuda_status(cudaGetSymbolAddress(&ptr, g_noalloc_scratch)))) return st;
    int sms = 0, optin = 0;
    if ((st = cuda_status(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev))) ||
        (st = cuda_status(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev))))
      return st;
    if ((st = cuda_status(cudaMemset(ptr, 0, kNoAllocScratchBytes)))) return st;
    S.scratch = (uint8_t*)ptr;
    S.num_sms = sms;
    // the same dynamic shared-memory ceiling the handle-based path sets
    S.smem_limit = (uint32_t)optin - 1024u;
    S.done = true;
  }
  *out = &S;
  return VIREO_OK;
}

}  // namespace
}  // namespace vireo

using namespace vireo;

extern "C" int gguf_moe_ffn_noalloc(const gguf_moe_desc* desc, const float* hb, float* x, int n_tok, int32_t* ids,
                                    float* wts, void* stream) {
  int st = VIREO_OK;
  auto fail = [](int code) {
    set_last_error(code);
    return code;
  };
  if (!desc || !hb || !x || n_tok < 0) return fail(VIREO_ERR_ARG);
  const gguf_moe_desc& D = *desc;
  // the shape and layout rules of gguf_moe_create
  if (D.dim <= 0 || D.ffn_exp <= 0 || D.n_experts <= 0 || D.n_used <= 0 || D.n_used > D.n_experts ||
      !D.router || !D.gate_exps || !D.up_exps || !D.down_exps)
    return fail(VIREO_ERR_ARG);
  if (D.router_type != T_F32 || D.gate_type != D.up_type || !fast_format(D.gate_type) ||
      !fast_format(D.down_type) || D.dim % kRouterChunk || D.dim > 8 * kRouterChunk || D.ffn_exp % kSegElems ||
      D.n_experts > 256 || D.n_used * D.ffn_exp > kMaxHValues ||
      D.n_used > kMaxTopK)
    return fail(VIREO_ERR_UNSUPPORTED);
  const uint64_t gsl = (uint64_t)D.ffn_exp * row_bytes(D.gate_type, D.dim);
  const uint64_t dsl = (uint64_t)D.dim * row_bytes(D.down_type, D.ffn_exp);
  if (D.gate_nbytes < gsl * D.n_experts || D.up_nbytes < gsl * D.n_experts || D.down_nbytes < dsl * D.n_experts)
    return fail(VIREO_ERR_ARG);
  const uint64_t gstep = D.gate_nbytes / D.n_experts, ustep = D.up_nbytes / D.n_experts,
                 dstep = D.down_nbytes / D.n_experts;
  if (((uintptr_t)D.router | (uintptr_t)D.gate_exps | (uintptr_t)D.up_exps | (uintptr_t)D.down_exps) % 16 ||
      gstep % 16 || ustep % 16 || dstep % 16)
    return fail(VIREO_ERR_UNSUPPORTED);
  if (((uintptr_t)hb % 16) || ((size_t)D.dim * 4) % 16) return fail(VIREO_ERR_ARG);

  // scratch layout inside the fixed array: the layer's scratch, then the
  // expert pointer table
  const size_t o_tab = moe_scratch_bytes(D.dim, D.ffn_exp, D.n_experts, D.n_used);
  const size_t need = o_tab + up256(sizeof(void*) * 3 * (size_t)D.n_experts);
  if (need > kNoAllocScratchBytes) return fail(VIREO_ERR_NOMEM);  // beyond the fixed scratch array
  if (n_tok == 0) return VIREO_OK;

  DevSetup* S = nullptr;
  if ((st = device_setup(&S))) return fail(st);

  MoeDecodeParams p;
  memset(&p, 0, sizeof(p));
  p.d = D.dim;
  p.fe = D.ffn_exp;
  p.ne = D.n_experts;
  p.k = D.n_used;
  p.renorm = D.topk_renorm;
  p.router = (const float*)D.router;
  if ((st = stage_geom(D.gate_type, D.dim, &p.sg_gu)) || (st = stage_geom(D.down_type, D.ffn_exp, &p.sg_d)))
    return fail(st);
  const uint32_t smem = moe_decode_layout(&p, S->smem_limit, S->num_sms);
  const void* kernel = moe_decode_kernel_for(D.gate_type, D.down_type);
  if (!smem || !kernel) return fail(VIREO_ERR_UNSUPPORTED);
  if ((st = cuda_status(
           cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S->smem_limit))))
    return fail(st);
  if (S->num_sms < D.n_used) return fail(VIREO_ERR_UNSUPPORTED);  // one CTA per expert group at least
  uint8_t* sb = S->scratch;
  moe_scratch_carve(sb, D.dim, D.ffn_exp, D.n_experts, D.n_used, nullptr, &p.s);
  p.exp_tab = (const uint8_t* const*)(sb + o_tab);
  // the words that must start at zero: sync words, status, tile counters
  const size_t zero_bytes = (size_t)((uint8_t*)p.s.logit_part - sb);

  // expert pointer table, staged on the stack (pageable: the copy has
  // consumed it when cudaMemcpyAsync returns)
  const uint8_t* tab[3 * 256];
  for (int ex = 0; ex < D.n_experts; ex++) {
    tab[3 * ex + 0] = (const uint8_t*)D.gate_exps + (uint64_t)ex * gstep;
    tab[3 * ex + 1] = (const uint8_t*)D.up_exps + (uint64_t)ex * ustep;
    tab[3 * ex + 2] = (const uint8_t*)D.down_exps + (uint64_t)ex * dstep;
  }
  cudaStream_t s = (cudaStream_t)stream;
  if ((st = cuda_status(cudaMemsetAsync(sb, 0, zero_bytes, s))) ||
      (st = cuda_status(
           cudaMemcpyAsync(sb + o_tab, tab, sizeof(void*) * 3 * (size_t)D.n_experts, cudaMemcpyHostToDevice, s))))
    return fail(st);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S->num_sms);
  cfg.blockDim = dim3(kDecodeThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // CTAs wait on one another's flags
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  for (int i = 0; i < n_tok; i++) {
    p.hb = hb + (size_t)i * p.d;
    p.x = x + (size_t)i * p.d;
    p.ids_out = ids ? ids + (size_t)i * p.k : nullptr;
    p.wts_out = wts ? wts + (size_t)i * p.k : nullptr;
    void* args[] = {&p};
    if ((st = cuda_status(cudaLaunchKernelExC(&cfg, kernel, args)))) {
      // earlier launches of this call may still be using the shared array:
      // wait for them before reporting, so that the next call starts clean
      cudaStreamSynchronize(s);
      return fail(st);
    }
  }
  // the kernel's status word: wait for the launches, read it back
  if ((st = cuda_status(cudaStreamSynchronize(s)))) return fail(st);
  int herr = 0;
  if ((st = cuda_status(cudaMemcpy(&herr, p.s.err, sizeof(int), cudaMemcpyDeviceToHost)))) return fail(st);
  if (herr) {
    // a launch gave up (timeout/abort): leave zeroed words for the next call
    cudaMemset(sb, 0, zero_bytes);
    return fail(herr);
  }
  return VIREO_OK;
}
