// C-ABI layer: the reference's gguf_compute.h functions, their device
// variants, and the MoE block (gguf_moe.h).  Host code only; kernels live
// in decode_kernels.cu / generic_kernels.cu.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <unordered_set>
#include <vector>

#include "gguf_compute.h"
#include "expert_store.h"
#include "gguf_moe.h"
#include "moe_decode.cuh"
#include "moe_view.h"
#include "vireo_internal.h"

namespace vireo {

static thread_local int t_last = VIREO_OK;
void set_last_error(int code) { t_last = code; }
int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return VIREO_OK;
  if (e == cudaErrorMemoryAllocation) return VIREO_ERR_NOMEM;
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return VIREO_ERR_NODEV;
  return VIREO_ERR_CUDA;
}

static std::mutex g_init_mu;
static Ctx* g_ctx = nullptr;
static int g_req_device = -1;

Ctx* ctx_get(int* status) {
  std::lock_guard<std::mutex> lk(g_init_mu);
  if (g_ctx) {
    *status = VIREO_OK;
    return g_ctx;
  }
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    *status = VIREO_ERR_NODEV;
    return nullptr;
  }
  Ctx* c = new Ctx();
  int dev = g_req_device;
  if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  cudaError_t e = cudaSetDevice(dev);
  cudaDeviceProp prop;
  if (e == cudaSuccess) e = cudaGetDeviceProperties(&prop, dev);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&c->d_err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(c->d_err, 0, sizeof(int));
  if (e != cudaSuccess) {
    *status = cuda_status(e);
    delete c;
    return nullptr;
  }
  c->device = dev;
  c->num_sms = prop.multiProcessorCount;
  c->smem_optin = (uint32_t)prop.sharedMemPerBlockOptin;
  g_ctx = c;
  *status = VIREO_OK;
  return c;
}

void* ctx_scratch(Ctx* c, size_t bytes) {
  if (bytes <= c->scratch_bytes) return c->scratch;
  if (c->scratch) cudaFree(c->scratch);
  c->scratch = nullptr;
  c->scratch_bytes = 0;
  size_t want = bytes + bytes / 4;
  if (cudaMalloc(&c->scratch, want) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  c->scratch_bytes = want;
  return c->scratch;
}

static std::mutex g_attr_mu;
static std::unordered_set<const void*> g_attr_done;
// dynamic shared memory available to the decode kernels: the opt-in limit
// minus room for their static shared memory
static uint32_t dyn_smem_limit(const Ctx* c) { return c->smem_optin - 1024u; }

static int ensure_smem_attr(const Ctx* c, const void* fn) {
  std::lock_guard<std::mutex> lk(g_attr_mu);
  if (g_attr_done.count(fn)) return VIREO_OK;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn_smem_limit(c));
  if (e != cudaSuccess) return cuda_status(e);
  // one shared-memory configuration for every kernel of a decode chain: an
  // SM can only hold CTAs of kernels that agree on it, and the programmatic
  // launches overlap only CTAs that can be co-resident
  e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return cuda_status(e);
  g_attr_done.insert(fn);
  return VIREO_OK;
}

int gemv_dev_fast(Ctx* c, uint32_t type, const void* w, const float* x, float* y, int n, int d, cudaStream_t s,
                  const float* norm_w, float eps, uint32_t prefetch_bytes) {
  if (n <= 0 || d <= 0) return VIREO_ERR_ARG;
  if (!fast_format(type) || n % kSegElems || d % 16 || ((uintptr_t)w % 16)) return VIREO_ERR_UNSUPPORTED;
  GemvParams p;
  memset(&p, 0, sizeof(p));
  if (stage_geom(type, n, &p.sg) != VIREO_OK) return VIREO_ERR_UNSUPPORTED;
  p.W = (const uint8_t*)w;
  p.x = x;
  p.y = y;
  p.n = n;
  p.d = d;
  p.err = c->d_err;
  p.norm_w = norm_w;
  p.eps = eps;
  p.prefetch_bytes = prefetch_bytes & ~15u;
  const int grid = std::min(c->num_sms, d / 16);
  // a ring deeper than the CTA's units only holds shared memory that the
  // next kernel's CTAs could use
  const int units_per_cta = (d / 16 + grid - 1) / grid;
  const uint32_t smem = gemv_layout(&p, dyn_smem_limit(c), units_per_cta);
  if (!smem) return VIREO_ERR_UNSUPPORTED;
  const void* fn = gemv_kernel_for(type);
  int st = ensure_smem_attr(c, fn);
  if (st) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kDecodeThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {&p};
  return cuda_status(cudaLaunchKernelExC(&cfg, fn, args));
}

int gemv_dev(Ctx* c, uint32_t type, const void* w, const float* x, float* y, int n, int d, cudaStream_t s) {
  if (n <= 0 || d < 0) return VIREO_ERR_ARG;
  if (d == 0) return VIREO_OK;
  const int st = gemv_dev_fast(c, type, w, x, y, n, d, s, nullptr, 0.f, 0u);
  if (st != VIREO_ERR_UNSUPPORTED) return st;
  return launch_gemv_generic(type, w, x, y, n, d, s);
}

static bool is_device_ptr(const void* p) {
  if (!p) return false;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

static const void* registered_dev(Ctx* c, const void* host, uint64_t bytes) {
  const uint8_t* h = (const uint8_t*)host;
  for (auto& r : c->ranges)
    if (h >= r.host && h + bytes <= r.host + r.bytes) return r.dev + (h - r.host);
  return nullptr;
}

static int read_status(Ctx* c, cudaStream_t s) {
  int st = cuda_status(cudaStreamSynchronize(s));
  if (st) return st;
  int herr = 0;
  st = cuda_status(cudaMemcpy(&herr, c->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (st) return st;
  if (herr) {
    cudaMemset(c->d_err, 0, sizeof(int));
    return herr;
  }
  return VIREO_OK;
}

static size_t up256(size_t v) { return (v + 255) & ~(size_t)255; }

}  // namespace vireo

using namespace vireo;

extern "C" {

int vireo_last_error(void) { return t_last; }

const char* vireo_status_string(int s) {
  switch (s) {
    case VIREO_OK: return "ok";
    case VIREO_ERR_ARG: return "invalid argument";
    case VIREO_ERR_CUDA: return "CUDA runtime error";
    case VIREO_ERR_UNSUPPORTED: return "unsupported tensor type or shape";
    case VIREO_ERR_TIMEOUT: return "device wait timed out";
    case VIREO_ERR_NOMEM: return "out of memory";
    case VIREO_ERR_IO: return "I/O error";
    case VIREO_ERR_NODEV: return "no CUDA device";
    default: return "unknown status";
  }
}

int vireo_device_init(int device) {
  {
    std::lock_guard<std::mutex> lk(g_init_mu);
    if (g_ctx) return g_ctx->device == device ? VIREO_OK : VIREO_ERR_ARG;
    g_req_device = device;
  }
  int st;
  Ctx* c = ctx_get(&st);
  return c ? VIREO_OK : st;
}

float gguf_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t e = (h >> 10) & 31u, m = h & 1023u;
  uint32_t bits;
  if (e == 31u) {
    bits = sign | 0x7f800000u | (m << 13);
  } else if (e == 0u) {
    float f = (float)m * 0x1p-24f;  // subnormal or zero: exact
    memcpy(&bits, &f, 4);
    bits |= sign;
  } else {
    bits = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

int vireo_sync(void* stream) {
  int st;
  Ctx* c = ctx_get(&st);
  if (!c) return st;
  return read_status(c, stream ? (cudaStream_t)stream : c->stream);
}

int gguf_matmul_dev(float* y, const float* x, const gguf_tensor* w, int n, int d, void* stream) {
  int st;
  Ctx* c = ctx_get(&st);
  if (!c) return st;
  if (!w || !y || !x || !w->data) return VIREO_ERR_ARG;
  return gemv_dev(c, w->ggml_type, w->data, x, y, n, d, stream ? (cudaStream_t)stream : c->stream);
}

int gguf_dequant_row_dev(uint32_t type, const void* src, float* dst, int n, void* stream) {
  int st;
  Ctx* c = ctx_get(&st);
  if (!c) return st;
  return launch_dequant(type, src, dst, n, stream ? (cudaStream_t)stream : c->stream);
}

void gguf_dequant_row(uint32_t type, const void* src, float* dst, int n) {
  int st;
  Ctx* c = ctx_get(&st);
  if (!c) {
    set_last_error(st);
    return;
  }
  int be, bb;
  if (type_block(type, &be, &bb) || n < 0 || n % be) {
    set_last_error(VIREO_ERR_UNSUPPORTED);
    return;
  }
  std::lock_guard<std::mutex> lk(c->mu);
  const size_t sb = (size_t)row_bytes(type, n), db = (size_t)n * 4;
  const bool sdev = is_device_ptr(src), ddev = is_device_ptr(dst);
  const void* s = sdev ? src : registered_dev(c, src, sb);
  uint8_t* scr = (uint8_t*)ctx_scratch(c, up256(sb) + up256(db));
  if (!scr) {
    set_last_error(VIREO_ERR_NOMEM);
    return;
  }
  if (!s) {
    if ((st = cuda_status(cudaMemcpyAsync(scr, src, sb, cudaMemcpyHostToDevice, c->stream)))) {
      set_last_error(st);
      return;
    }
    s = scr;
  }
  float* dd = ddev ? dst : (float*)(scr + up256(sb));
  st = launch_dequant(type, s, dd, n, c->stream);
  if (!st && !ddev) st = cuda_status(cudaMemcpyAsync(dst, dd, db, cudaMemcpyDeviceToHost, c->stream));
  if (!st) st = read_status(c, c->stream);
  set_last_error(st);
}

void gguf_matmul(float* y, const float* x, const gguf_tensor* w, int n, int d) {
  int st;
  Ctx* c = ctx_get(&st);
  if (!c) {
    set_last_error(st);
    return;
  }
  if (!w || !w->data || !x || !y || n <= 0 || d < 0) {
    set_last_error(VIREO_ERR_ARG);
    return;
  }
  int be, bb;
  if (type_block(w->ggml_type, &be, &bb) || n % be) {
    set_last_error(VIREO_ERR_UNSUPPORTED);
    return;
  }
  std::lock_guard<std::mutex> lk(c->mu);
  const size_t wb = (size_t)row_bytes(w->ggml_type, n) * (size_t)d, xb = (size_t)n * 4, yb = (size_t)d * 4;
  const bool wdev = is_device_ptr(w->data), xdev = is_device_ptr(x), ydev = is_device_ptr(y);
  const void* wd = wdev ? w->data : registered_dev(c, w->data, wb);
  const size_t need = (wd ? 0 : up256(wb)) + up256(xb) + up256(yb);
  uint8_t* scr = (uint8_t*)ctx_scratch(c, need);
  if (!scr) {
    set_last_error(VIREO_ERR_NOMEM);
    return;
  }
  size_t off = 0;
  if (!wd) {
    if ((st = cuda_status(cudaMemcpyAsync(scr, w->data, wb, cudaMemcpyHostToDevice, c->stream)))) {
      set_last_error(st);
      return;
    }
    wd = scr;
    off = up256(wb);
  }
  const float* xd = x;
  if (!xdev) {
    float* xs = (float*)(scr + off);
    off += up256(xb);
    if ((st = cuda_status(cudaMemcpyAsync(xs, x, xb, cudaMemcpyHostToDevice, c->stream)))) {
      set_last_error(st);
      return;
    }
    xd = xs;
  }
  float* yd = ydev ? y : (float*)(scr + off);
  st = gemv_dev(c, w->ggml_type, wd, xd, yd, n, d, c->stream);
  if (!st && !ydev) st = cuda_status(cudaMemcpyAsync(y, yd, yb, cudaMemcpyDeviceToHost, c->stream));
  if (!st) st = read_status(c, c->stream);
  set_last_error(st);
}

int gguf_weights_register(const void* host, uint64_t nbytes) {
  int st;
  Ctx* c = ctx_get(&st);
  if (!c) return st;
  if (!host || !nbytes) return VIREO_ERR_ARG;
  std::lock_guard<std::mutex> lk(c->mu);
  HostRange r;
  r.host = (const uint8_t*)host;
  r.bytes = nbytes;
  r.dev = nullptr;
  if ((st = cuda_status(cudaMalloc(&r.dev, nbytes)))) return st;
  if ((st = cuda_status(cudaMemcpy(r.dev, host, nbytes, cudaMemcpyHostToDevice)))) {
    cudaFree(r.dev);
    return st;
  }
  c->ranges.push_back(r);
  return VIREO_OK;
}

int gguf_weights_unregister(const void* host) {
  int st;
  Ctx* c = ctx_get(&st);
  if (!c) return st;
  std::lock_guard<std::mutex> lk(c->mu);
  for (size_t i = 0; i < c->ranges.size(); i++) {
    if (c->ranges[i].host == host) {
      cudaStreamSynchronize(c->stream);
      cudaFree(c->ranges[i].dev);
      c->ranges.erase(c->ranges.begin() + (long)i);
      return VIREO_OK;
    }
  }
  return VIREO_ERR_ARG;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// MoE block
// ---------------------------------------------------------------------------
struct gguf_moe {
  gguf_moe_desc desc;
  MoeDecodeParams prm;
  const void* kernel = nullptr;
  const void* rkernel = nullptr;  // routed variant (caller's route, no router phase)
  uint32_t smem = 0;
  int grid = 0;
  const uint8_t** d_exp_tab = nullptr;
  std::vector<const uint8_t*> h_exp_tab;
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  // host-API staging, the same layout on the device and in pinned host
  // memory: hb [n][d] | x [n][d] | status (16 B) | ids [n][k] | wts [n][k]
  uint8_t* d_io = nullptr;
  uint8_t* h_io = nullptr;
  uint8_t* h_io_dev = nullptr;  // h_io as the device addresses it (mapped pinned memory)
  void* owned[4] = {};  // device copies of the layer's tensors (gguf_moe_create_host)
  int io_cap = 0;
  bool pdl = true;
  cudaStream_t stream = nullptr;
  PrefillScratch pre;  // batched path, grown on demand
  int num_sms = 0;
};

int vireo::moe_view(gguf_moe* m, MoeView* v) {
  if (!m || !v) return VIREO_ERR_ARG;
  v->desc = &m->desc;
  v->exp_tab = m->d_exp_tab;
  v->pre = &m->pre;
  v->err = m->prm.s.err;
  v->num_sms = m->num_sms;
  v->stream = m->stream;
  return VIREO_OK;
}

static int moe_reset_scratch(gguf_moe* m, cudaStream_t s) {
  return cuda_status(cudaMemsetAsync(m->scratch, 0, m->scratch_bytes, s));
}

extern "C" {

// The layer rules gguf_moe_create applies to a descriptor, apart from where
// its tensors live and their alignment.
static int moe_check_shape(const gguf_moe_desc& D) {
  if (D.dim <= 0 || D.ffn_exp <= 0 || D.n_experts <= 0 || D.n_used <= 0 || D.n_used > D.n_experts ||
      !D.router || !D.gate_exps || !D.up_exps || !D.down_exps)
    return VIREO_ERR_ARG;
  if (D.router_type != T_F32 || D.gate_type != D.up_type || !fast_format(D.gate_type) ||
      !fast_format(D.down_type) || D.dim % kRouterChunk || D.dim > 8 * kRouterChunk || D.ffn_exp % kSegElems ||
      D.n_experts > 256 || D.n_used * D.ffn_exp > kMaxHValues ||
      D.n_used > kMaxTopK)
    return VIREO_ERR_UNSUPPORTED;
  const uint64_t gsl = (uint64_t)D.ffn_exp * row_bytes(D.gate_type, D.dim);
  const uint64_t dsl = (uint64_t)D.dim * row_bytes(D.down_type, D.ffn_exp);
  if (D.gate_nbytes < gsl * D.n_experts || D.up_nbytes < gsl * D.n_experts || D.down_nbytes < dsl * D.n_experts)
    return VIREO_ERR_ARG;
  if ((D.gate_nbytes / D.n_experts) % 16 || (D.up_nbytes / D.n_experts) % 16 || (D.down_nbytes / D.n_experts) % 16)
    return VIREO_ERR_UNSUPPORTED;
  return VIREO_OK;
}

int gguf_moe_create(const gguf_moe_desc* desc, gguf_moe** out) {
  int st;
  Ctx* c = ctx_get(&st);
  if (!c) return st;
  if (!desc || !out) return VIREO_ERR_ARG;
  *out = nullptr;
  const gguf_moe_desc& D = *desc;
  if ((st = moe_check_shape(D))) return st;
  const uint64_t gstep = D.gate_nbytes / D.n_experts, ustep = D.up_nbytes / D.n_experts,
                 dstep = D.down_nbytes / D.n_experts;
  if (((uintptr_t)D.router | (uintptr_t)D.gate_exps | (uintptr_t)D.up_exps | (uintptr_t)D.down_exps) % 16)
    return VIREO_ERR_UNSUPPORTED;

  gguf_moe* m = new gguf_moe();
  m->desc = D;
  MoeDecodeParams& p = m->prm;
  memset(&p, 0, sizeof(p));
  p.d = D.dim;
  p.fe = D.ffn_exp;
  p.ne = D.n_experts;
  p.k = D.n_used;
  p.renorm = D.topk_renorm;
  p.router = (const float*)D.router;
  if ((st = stage_geom(D.gate_type, D.dim, &p.sg_gu)) || (st = stage_geom(D.down_type, D.ffn_exp, &p.sg_d))) {
    delete m;
    return st;
  }
  m->smem = moe_decode_layout(&p, dyn_smem_limit(c), c->num_sms);
  m->kernel = moe_decode_kernel_for(D.gate_type, D.down_type);
  m->rkernel = moe_decode_kernel_for(D.gate_type, D.down_type, true);
  if (!m->smem || !m->kernel || !m->rkernel) {
    delete m;
    return VIREO_ERR_UNSUPPORTED;
  }
  if ((st = ensure_smem_attr(c, m->kernel)) || (st = ensure_smem_attr(c, m->rkernel))) {
    delete m;
    return st;
  }
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, m->kernel, kDecodeThreads, m->smem);
  if (e != cudaSuccess || per_sm < 1) {
    delete m;
    return e != cudaSuccess ? cuda_status(e) : VIREO_ERR_UNSUPPORTED;
  }
  // one CTA per SM; the k expert groups need at least one CTA each
  if (c->num_sms < D.n_used) {
    delete m;
    return VIREO_ERR_UNSUPPORTED;
  }
  m->grid = c->num_sms;
  m->num_sms = c->num_sms;

  // scratch: sync words, status, tile counters, router partials, h, down outputs
  m->scratch_bytes = moe_scratch_bytes(D.dim, D.ffn_exp, D.n_experts, D.n_used);
  if ((st = cuda_status(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking))) ||
      (st = cuda_status(cudaMalloc(&m->scratch, m->scratch_bytes))) ||
      (st = cuda_status(cudaMemset(m->scratch, 0, m->scratch_bytes)))) {
    gguf_moe_destroy(m);
    return st;
  }
  moe_scratch_carve((uint8_t*)m->scratch, D.dim, D.ffn_exp, D.n_experts, D.n_used, nullptr, &p.s);

  m->h_exp_tab.resize((size_t)3 * D.n_experts);
  for (int ex = 0; ex < D.n_experts; ex++) {
    m->h_exp_tab[3 * ex + 0] = (const uint8_t*)D.gate_exps + (uint64_t)ex * gstep;
    m->h_exp_tab[3 * ex + 1] = (const uint8_t*)D.up_exps + (uint64_t)ex * ustep;
    m->h_exp_tab[3 * ex + 2] = (const uint8_t*)D.down_exps + (uint64_t)ex * dstep;
  }
  if ((st = cuda_status(cudaMalloc(&m->d_exp_tab, sizeof(void*) * m->h_exp_tab.size()))) ||
      (st = cuda_status(cudaMemcpy(m->d_exp_tab, m->h_exp_tab.data(), sizeof(void*) * m->h_exp_tab.size(),
                                   cudaMemcpyHostToDevice)))) {
    gguf_moe_destroy(m);
    return st;
  }
  p.exp_tab = m->d_exp_tab;
  *out = m;
  return VIREO_OK;
}

// A layer whose tensors are in host memory (the mmap of a GGUF file):
// checked first, then the router and the three expert tensors are copied
// into device memory that the handle owns and frees on destroy.
int gguf_moe_create_host(const gguf_moe_desc* desc, gguf_moe** out) {
  int st;
  Ctx* c = ctx_get(&st);
  if (!c) return st;
  if (!desc || !out) return VIREO_ERR_ARG;
  *out = nullptr;
  const gguf_moe_desc& H = *desc;
  if ((st = moe_check_shape(H))) return st;
  const void* src[4] = {H.router, H.gate_exps, H.up_exps, H.down_exps};
  const uint64_t nb[4] = {(uint64_t)H.n_experts * row_bytes(H.router_type, H.dim), H.gate_nbytes, H.up_nbytes,
                          H.down_nbytes};
  void* dev[4] = {};
  for (int i = 0; i < 4 && !st; i++) {
    if ((st = cuda_status(cudaMalloc(&dev[i], nb[i])))) break;
    st = cuda_status(cudaMemcpy(dev[i], src[i], nb[i], cudaMemcpyHostToDevice));
  }
  gguf_moe_desc D = H;
  D.router = dev[0];
  D.gate_exps = dev[1];
  D.up_exps = dev[2];
  D.down_exps = dev[3];
  if (!st) st = gguf_moe_create(&D, out);
  if (st) {
    for (void* p : dev) cudaFree(p);
    return st;
  }
  for (int i = 0; i < 4; i++) (*out)->owned[i] = dev[i];
  return VIREO_OK;
}

// One launch of the decode kernel (or its routed variant) for one token,
// with programmatic stream serialization: the next token's CTAs take SMs as
// this launch's CTAs leave and run their weight-only prologue (barrier set-up,
// router rows) before griddepcontrol.wait, which orders everything that reads
// the previous kernel's output.  The launch is not marked cooperative (the
// driver refuses cooperative + programmatic launches), so co-residency of the
// grid's CTAs, which wait on one another's flags, rests on the grid being one
// CTA per SM with occupancy >= 1 (checked at create) and on nothing else
// holding the SMs; every such wait is bounded, so a launch that shares the
// GPU with another kernel that holds SMs ends with VIREO_ERR_TIMEOUT instead
// of hanging.
// The host call's input copy: the hidden rows from mapped pinned memory into
// device memory (the decode kernel's CTAs all read them), and the status
// word zeroed.  It lets the next kernel launch at once; that kernel's
// griddepcontrol.wait orders its reads after this copy.
__global__ void host_stage_kernel(const float4* src, float4* dst, size_t n4, int* status) {
  pdl_launch_dependents();
  if (blockIdx.x == 0 && threadIdx.x == 0) *status = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

static int moe_launch(gguf_moe* m, const void* kernel, void** args, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m->grid);
  cfg.blockDim = dim3(kDecodeThreads);
  cfg.dynamicSmemBytes = m->smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = m->pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelExC(&cfg, kernel, args);
  if (e != cudaSuccess && m->pdl) {
    cudaGetLastError();
    m->pdl = false;
    cfg.numAttrs = 0;
    e = cudaLaunchKernelExC(&cfg, kernel, args);
  }
  return cuda_status(e);
}

// n_tok decode launches; the kernels record failures in *err (and, when
// err_out is given, the last launch's last CTA reports there: status, done)
static int moe_ffn_launches(gguf_moe* m, const float* hb, float* x, int n_tok, int32_t* ids, float* wts,
                            cudaStream_t s, int* err, int* err_out = nullptr) {
  MoeDecodeParams p = m->prm;
  p.s.err = err;
  for (int i = 0; i < n_tok; i++) {
    p.err_out = i == n_tok - 1 ? err_out : nullptr;
    p.hb = hb + (size_t)i * p.d;
    p.x = x + (size_t)i * p.d;
    p.ids_out = ids ? ids + (size_t)i * p.k : nullptr;
    p.wts_out = wts ? wts + (size_t)i * p.k : nullptr;
    void* args[] = {&p};
    int st = moe_launch(m, m->kernel, args, s);
    if (st) return st;
  }
  return VIREO_OK;
}

int gguf_moe_ffn(gguf_moe* m, const float* hb, float* x, int n_tok, int32_t* ids, float* wts, void* stream) {
  if (!m || !hb || !x || n_tok < 0) return VIREO_ERR_ARG;
  if (((uintptr_t)hb % 16) || ((size_t)m->prm.d * 4) % 16) return VIREO_ERR_ARG;
  cudaStream_t s = stream ? (cudaStream_t)stream : m->stream;
  return moe_ffn_launches(m, hb, x, n_tok, ids, wts, s, m->prm.s.err);
}

}  // extern "C"

int vireo::moe_ffn_norm(gguf_moe* m, float* x, const float* y, const float* w, float eps, cudaStream_t s) {
  if (!m || !x || !y || !w) return VIREO_ERR_ARG;
  MoeDecodeParams p = m->prm;
  p.hb = nullptr;
  p.x = x;
  p.res_y = y;
  p.norm_w = w;
  p.norm_eps = eps;
  p.ids_out = nullptr;
  p.wts_out = nullptr;
  void* args[] = {&p};
  return moe_launch(m, m->kernel, args, s ? s : m->stream);
}

extern "C" {

int gguf_moe_ffn_routed(gguf_moe* m, const float* hb, float* x, int n_tok, const int32_t* ids, const float* wts,
                        const void* const* expert_ptrs, void* stream) {
  if (!m || !hb || !x || n_tok < 0 || (n_tok && (!ids || !wts || !expert_ptrs))) return VIREO_ERR_ARG;
  if (((uintptr_t)hb % 16) || ((size_t)m->prm.d * 4) % 16) return VIREO_ERR_ARG;
  cudaStream_t s = stream ? (cudaStream_t)stream : m->stream;
  MoeDecodeParams p = m->prm;
  const int k = p.k;
  MoeRoute r;
  memset(&r, 0, sizeof(r));
  for (int i = 0; i < n_tok; i++) {
    for (int t = 0; t < k; t++) {
      const int32_t e = ids[(size_t)i * k + t];
      const void* const* pt = expert_ptrs + ((size_t)i * k + t) * 3;
      const bool on = e >= 0 && e < p.ne && pt[0] && pt[1] && pt[2];
      if (on && (((uintptr_t)pt[0] | (uintptr_t)pt[1] | (uintptr_t)pt[2]) % 16)) return VIREO_ERR_UNSUPPORTED;
      r.ids[t] = on ? e : -1;
      r.wts[t] = on ? wts[(size_t)i * k + t] : -1.f;
      for (int j = 0; j < 3; j++) r.ptr[t][j] = on ? (const uint8_t*)pt[j] : nullptr;
    }
    p.hb = hb + (size_t)i * p.d;
    p.x = x + (size_t)i * p.d;
    p.ids_out = nullptr;
    p.wts_out = nullptr;
    void* args[] = {&p, &r};
    int st = moe_launch(m, m->rkernel, args, s);
    if (st) return st;
  }
  return VIREO_OK;
}

int gguf_moe_ffn_store(gguf_moe* m, ExpertStore* store, int layer, const float* hb, float* x, const int32_t* ids,
                       const float* wts, void* stream) {
  if (!m || !store || !ids || !wts) return VIREO_ERR_ARG;
  cudaStream_t s = stream ? (cudaStream_t)stream : m->stream;
  const int k = m->prm.k;
  ExpertView views[kMaxTopK];
  const void* ptrs[kMaxTopK * 3];
  int32_t rid[kMaxTopK];
  memset(views, 0, sizeof(views));
  memset(ptrs, 0, sizeof(ptrs));
  memset(rid, 0, sizeof(rid));
  int st = VIREO_OK;
  for (int t = 0; t < k; t++) {
    rid[t] = ids[t];
    if (ids[t] < 0 || expert_store_lookup_async(store, layer, ids[t], &views[t], s) != 0) {
      rid[t] = -1;  // the reference skips an expert whose lookup fails (gguf_run.c:201)
      memset(&views[t], 0, sizeof(views[t]));
    }
    ptrs[3 * t + 0] = views[t].gate;
    ptrs[3 * t + 1] = views[t].up;
    ptrs[3 * t + 2] = views[t].down;
  }
  st = gguf_moe_ffn_routed(m, hb, x, 1, rid, wts, ptrs, s);
  for (int t = 0; t < k; t++)
    if (views[t].slot) expert_store_release_after(store, &views[t], s);
  return st;
}

int gguf_moe_prefill(gguf_moe* m, const void* hb_bf16, float* x, int n_tok, const float* router_bias, int32_t* ids,
                     float* wts, void* stream) {
  if (!m || n_tok < 0 || (n_tok && (!hb_bf16 || !x))) return VIREO_ERR_ARG;
  const gguf_moe_desc& D = m->desc;
  if (!prefill_supported(D.dim, D.ffn_exp, D.n_experts, D.n_used, D.router_type, D.gate_type, D.up_type,
                         D.down_type))
    return VIREO_ERR_UNSUPPORTED;
  if (((uintptr_t)hb_bf16 | (uintptr_t)x) % 16) return VIREO_ERR_ARG;
  if (n_tok == 0) return VIREO_OK;
  cudaStream_t s = stream ? (cudaStream_t)stream : m->stream;
  PrefillLayer L;
  L.d = D.dim;
  L.fe = D.ffn_exp;
  L.ne = D.n_experts;
  L.k = D.n_used;
  L.renorm = D.topk_renorm;
  L.router = (const float*)D.router;
  L.exp_tab = m->d_exp_tab;
  return prefill_run(L, &m->pre, hb_bf16, x, n_tok, router_bias, ids, wts, m->prm.s.err, m->num_sms, s);
}

int gguf_moe_sync(gguf_moe* m, void* stream) {
  if (!m) return VIREO_ERR_ARG;
  cudaStream_t s = stream ? (cudaStream_t)stream : m->stream;
  int st = cuda_status(cudaStreamSynchronize(s));
  if (st) return st;
  int herr = 0;
  if ((st = cuda_status(cudaMemcpy(&herr, m->prm.s.err, sizeof(int), cudaMemcpyDeviceToHost)))) return st;
  if (herr) {
    moe_reset_scratch(m, s);
    cudaStreamSynchronize(s);
    return herr;
  }
  return VIREO_OK;
}

// One round trip for n_tok tokens: the inputs and a zeroed status word go
// to the device in one copy, the launches record failures in that word, and
// the outputs, the status and the selection come back in one copy.
int gguf_moe_ffn_host(gguf_moe* m, const float* hb, float* x, int n_tok, int32_t* ids, float* wts) {
  if (!m || !hb || !x || n_tok < 0) return VIREO_ERR_ARG;
  if (n_tok == 0) return VIREO_OK;
  const size_t d = (size_t)m->prm.d, k = (size_t)m->prm.k, n = (size_t)n_tok;
  const size_t o_x = n * d * 4, o_st = 2 * n * d * 4, o_ids = o_st + 16, o_wts = o_ids + n * k * 4,
               total = o_wts + n * k * 4;
  int st;
  if (n_tok > m->io_cap) {
    cudaFree(m->d_io);
    cudaFreeHost(m->h_io);
    m->d_io = nullptr;
    m->h_io = nullptr;
    m->h_io_dev = nullptr;
    m->io_cap = 0;
    void* hd = nullptr;
    if ((st = cuda_status(cudaMalloc(&m->d_io, total))) ||
        (st = cuda_status(cudaHostAlloc(&m->h_io, total, cudaHostAllocMapped))) ||
        (st = cuda_status(cudaHostGetDevicePointer(&hd, m->h_io, 0))))
      return st;
    m->h_io_dev = (uint8_t*)hd;
    m->io_cap = n_tok;
  }
  cudaStream_t s = m->stream;
  // One round trip through mapped pinned memory, no copy-engine transfers:
  // the previous call synchronised, so the buffer is free.  The hidden rows
  // go to device memory by a staging kernel; the residual rows are read and
  // written, and the selection written, by the decode kernels in host
  // memory directly (each CTA touches only its own rows); the status word
  // comes back through the last CTA of each launch.
  memcpy(m->h_io, hb, n * d * 4);
  memcpy(m->h_io + o_x, x, n * d * 4);
  memset(m->h_io + o_st, 0, 16);
  int* d_status = (int*)(m->d_io + o_st);
  const size_t n4 = n * d / 4;
  const int sg = (int)std::min<size_t>((n4 + 511) / 512, (size_t)m->num_sms);
  host_stage_kernel<<<sg, 512, 0, s>>>((const float4*)m->h_io_dev, (float4*)m->d_io, n4, d_status);
  st = cuda_status(cudaGetLastError());
  if (!st)
    st = moe_ffn_launches(m, (const float*)m->d_io, (float*)(m->h_io_dev + o_x), n_tok,
                          (int32_t*)(m->h_io_dev + o_ids), (float*)(m->h_io_dev + o_wts), s, d_status,
                          (int*)(m->h_io_dev + o_st));
  if (st) {
    cudaStreamSynchronize(s);
    return st;
  }
  // the last CTA's done word: it follows every output (the kernel fences its
  // host writes system-wide first), so the call returns without waiting for
  // the launch to be retired; the stream is still polled now and then, so a
  // launch that failed outright is reported instead of awaited
  volatile int* done = (volatile int*)(m->h_io + o_st + 4);
  for (long it = 0; !*done; it++) {
    if ((it & 4095) == 4095) {
      const cudaError_t q = cudaStreamQuery(s);
      if (q == cudaSuccess) {
        if (!*done) return VIREO_ERR_CUDA;  // retired without reporting
        break;
      }
      if (q != cudaErrorNotReady) return cuda_status(q);
    }
  }
  int herr = 0;
  memcpy(&herr, m->h_io + o_st, sizeof(int));
  if (herr) {
    // a launch gave up: its sync words may be left mid-protocol
    moe_reset_scratch(m, s);
    cudaStreamSynchronize(s);
    return herr;
  }
  memcpy(x, m->h_io + o_x, n * d * 4);
  if (ids) memcpy(ids, m->h_io + o_ids, n * k * 4);
  if (wts) memcpy(wts, m->h_io + o_wts, n * k * 4);
  return VIREO_OK;
}

int gguf_moe_set_expert_ptrs(gguf_moe* m, const void* const* gate, const void* const* up, const void* const* down) {
  if (!m) return VIREO_ERR_ARG;
  m->pre.minmat_ok = false;  // the batched path's min block follows the gate/up bytes
  for (int ex = 0; ex < m->desc.n_experts; ex++) {
    if (gate) m->h_exp_tab[3 * ex + 0] = (const uint8_t*)gate[ex];
    if (up) m->h_exp_tab[3 * ex + 1] = (const uint8_t*)up[ex];
    if (down) m->h_exp_tab[3 * ex + 2] = (const uint8_t*)down[ex];
  }
  for (auto* ptr : m->h_exp_tab)
    if (((uintptr_t)ptr) % 16) return VIREO_ERR_ARG;
  return cuda_status(cudaMemcpy(m->d_exp_tab, m->h_exp_tab.data(), sizeof(void*) * m->h_exp_tab.size(),
                                cudaMemcpyHostToDevice));
}

int gguf_moe_set_trace(gguf_moe* m, unsigned long long* dev_buf) {
  if (!m) return VIREO_ERR_ARG;
  m->prm.trace = dev_buf;
  return VIREO_OK;
}

int gguf_moe_grid(const gguf_moe* m) { return m ? m->grid : 0; }

// ---- shared expert: a one-expert layer over the shared tensors, run by the
// routed kernel with the gate weight formed on the device -------------------
struct gguf_moe_shexp {
  gguf_moe* m = nullptr;
  float* zero_router = nullptr;  // the one-expert layer's router (never read: routed launches)
  const float* gate_inp = nullptr;
  const uint8_t* ptr[3] = {};
};

int gguf_moe_shexp_create(const gguf_moe_shexp_desc* desc, gguf_moe_shexp** out) {
  if (!desc || !out || !desc->gate || !desc->up || !desc->down || desc->dim <= 0 || desc->ffn <= 0)
    return VIREO_ERR_ARG;
  *out = nullptr;
  gguf_moe_shexp* sh = new gguf_moe_shexp();
  int st = cuda_status(cudaMalloc(&sh->zero_router, (size_t)desc->dim * 4));
  if (!st) st = cuda_status(cudaMemset(sh->zero_router, 0, (size_t)desc->dim * 4));
  if (st) {
    gguf_moe_shexp_destroy(sh);
    return st;
  }
  gguf_moe_desc d;
  memset(&d, 0, sizeof(d));
  d.dim = desc->dim;
  d.ffn_exp = desc->ffn;
  d.n_experts = 1;
  d.n_used = 1;
  d.router_type = T_F32;
  d.gate_type = desc->gate_type;
  d.up_type = desc->up_type;
  d.down_type = desc->down_type;
  d.router = sh->zero_router;
  d.gate_exps = desc->gate;
  d.up_exps = desc->up;
  d.down_exps = desc->down;
  d.gate_nbytes = (uint64_t)desc->ffn * row_bytes(desc->gate_type, desc->dim);
  d.up_nbytes = (uint64_t)desc->ffn * row_bytes(desc->up_type, desc->dim);
  d.down_nbytes = (uint64_t)desc->dim * row_bytes(desc->down_type, desc->ffn);
  if ((st = gguf_moe_create(&d, &sh->m))) {
    gguf_moe_shexp_destroy(sh);
    return st;
  }
  sh->gate_inp = desc->gate_inp;
  sh->ptr[0] = (const uint8_t*)desc->gate;
  sh->ptr[1] = (const uint8_t*)desc->up;
  sh->ptr[2] = (const uint8_t*)desc->down;
  *out = sh;
  return VIREO_OK;
}

int gguf_moe_shexp_ffn(gguf_moe_shexp* sh, const float* hb, float* x, int n_tok, void* stream) {
  if (!sh || !hb || !x || n_tok < 0) return VIREO_ERR_ARG;
  gguf_moe* m = sh->m;
  if (((uintptr_t)hb % 16) || ((uintptr_t)sh->gate_inp % 16)) return VIREO_ERR_ARG;
  cudaStream_t s = stream ? (cudaStream_t)stream : m->stream;
  MoeDecodeParams p = m->prm;
  MoeRoute r;
  memset(&r, 0, sizeof(r));
  r.ids[0] = 0;
  r.wts[0] = 1.0f;  // replaced on the device by sigmoid(gate_inp . hb) when there is a gate
  for (int j = 0; j < 3; j++) r.ptr[0][j] = sh->ptr[j];
  p.sh_gate = sh->gate_inp;
  p.ids_out = nullptr;
  p.wts_out = nullptr;
  for (int i = 0; i < n_tok; i++) {
    p.hb = hb + (size_t)i * p.d;
    p.x = x + (size_t)i * p.d;
    void* args[] = {&p, &r};
    int st = moe_launch(m, m->rkernel, args, s);
    if (st) return st;
  }
  return VIREO_OK;
}

int gguf_moe_shexp_sync(gguf_moe_shexp* sh, void* stream) { return sh ? gguf_moe_sync(sh->m, stream) : VIREO_ERR_ARG; }

void gguf_moe_shexp_destroy(gguf_moe_shexp* sh) {
  if (!sh) return;
  if (sh->m) gguf_moe_destroy(sh->m);
  if (sh->zero_router) cudaFree(sh->zero_router);
  delete sh;
}

void gguf_moe_destroy(gguf_moe* m) {
  if (!m) return;
  if (m->stream) cudaStreamSynchronize(m->stream);
  prefill_scratch_free(&m->pre);
  cudaFree(m->scratch);
  cudaFree(m->d_exp_tab);
  cudaFree(m->d_io);
  cudaFreeHost(m->h_io);
  for (void* p : m->owned) cudaFree(p);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

}  // extern "C"
