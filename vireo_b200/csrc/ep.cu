// Expert-parallel batched MoE FFN (prefill) across the GPUs of one node.
//
// The reference has no batched path and no distribution at all (moe_ffn,
// vireo src/gguf_run.c:185-214, runs one token at a time on the host).  This
// file spreads the batched path of prefill.cu over G ranks, one process per
// GPU: rank r holds its own slice of the tokens and computes the experts
// placed on it; the tokens' rows travel to the experts and the expert outputs
// travel back, each as one NCCL all-to-all over NVLink.
//
// One call, rank r, T local tokens, k slots each (pairs = T k):
//   route     prep + router GEMM + top-k on the local tokens (prefill.cu)
//   count     pair -> owning rank of its expert; per-destination counts; an
//             all-gather of the counts gives every rank the full [G][G]
//             matrix (one host read per call: NCCL needs the sizes)
//   dispatch  each pair's activation row (f16, Kx columns) with a 16-byte tail
//             {expert, gate weight} is packed by destination and sent
//   experts   received rows are grouped by (local) expert and run through the
//             tcgen05 gate/up and down GEMMs of prefill.cu
//   return    output rows go back to their source ranks in arrival order
//   combine   x[t] += sum over rank order of the returned rows (the reference's
//             combine order, gguf_run.c:209, 213)
// Every output row is computed by the same GEMM arithmetic as on one GPU, and
// the combine order is the same, so the result is bit-identical to
// gguf_moe_prefill on one GPU.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2; in a process that has
// already loaded it, e.g. through PyTorch, that copy is used).  Host-side
// waits on the stream are bounded: a peer that stops answering ends the call
// with VIREO_ERR_TIMEOUT and aborts the communicator.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdint.h>
#include <string.h>
#include <time.h>

#include <algorithm>
#include <mutex>
#include <numeric>
#include <vector>

#include "gguf_moe.h"
#include "moe_view.h"
#include "vireo_internal.h"

namespace vireo {

constexpr int kEpMaxWorld = 64;
constexpr int kEpTailHalves = 8;  // 16-byte row tail: expert id, gate weight, 2 spare words
constexpr double kEpWaitSeconds = 60.0;

// ---- NCCL entry points, resolved once ---------------------------------------
struct NcclApi {
  decltype(&ncclGetUniqueId) getUniqueId = nullptr;
  decltype(&ncclCommInitRank) commInitRank = nullptr;
  decltype(&ncclCommDestroy) commDestroy = nullptr;
  decltype(&ncclCommAbort) commAbort = nullptr;
  decltype(&ncclCommGetAsyncError) getAsyncError = nullptr;
  decltype(&ncclGroupStart) groupStart = nullptr;
  decltype(&ncclGroupEnd) groupEnd = nullptr;
  decltype(&ncclSend) send = nullptr;
  decltype(&ncclRecv) recv = nullptr;
  decltype(&ncclAllGather) allGather = nullptr;
  bool ok = false;
};

static const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
#define VIREO_NCCL_SYM(field, name) api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name))
    VIREO_NCCL_SYM(getUniqueId, "ncclGetUniqueId");
    VIREO_NCCL_SYM(commInitRank, "ncclCommInitRank");
    VIREO_NCCL_SYM(commDestroy, "ncclCommDestroy");
    VIREO_NCCL_SYM(commAbort, "ncclCommAbort");
    VIREO_NCCL_SYM(getAsyncError, "ncclCommGetAsyncError");
    VIREO_NCCL_SYM(groupStart, "ncclGroupStart");
    VIREO_NCCL_SYM(groupEnd, "ncclGroupEnd");
    VIREO_NCCL_SYM(send, "ncclSend");
    VIREO_NCCL_SYM(recv, "ncclRecv");
    VIREO_NCCL_SYM(allGather, "ncclAllGather");
#undef VIREO_NCCL_SYM
    api.ok = api.getUniqueId && api.commInitRank && api.commDestroy && api.commAbort && api.getAsyncError &&
             api.groupStart && api.groupEnd && api.send && api.recv && api.allGather;
  });
  return api;
}

struct EpOffsets {
  int off[kEpMaxWorld];
};

// ---- kernels ------------------------------------------------------------------
// pair -> destination rank and its index among that rank's rows
__global__ void ep_route(const int32_t* ids, const int32_t* owner, int pairs, int* sendcnt, int* pdest, int* ppos) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= pairs) return;
  const int e = ids[p];
  int dst = -1, pos = -1;
  if (e >= 0) {
    dst = owner[e];
    pos = atomicAdd(&sendcnt[dst], 1);
  }
  pdest[p] = dst;
  ppos[p] = pos;
}

// dispatch rows: the token's activation row + {expert, weight} tail; one warp per pair
__global__ void ep_pack(const __half* xa, const int32_t* ids, const float* wts, const int* pdest, const int* ppos,
                        int pairs, int k, int Kx, const __grid_constant__ EpOffsets so, __half* sendbuf) {
  const int p = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (p >= pairs) return;
  const int dst = pdest[p];
  if (dst < 0) return;
  const int rs = Kx + kEpTailHalves;
  __half* row = sendbuf + (size_t)(so.off[dst] + ppos[p]) * rs;
  const uint4* s4 = reinterpret_cast<const uint4*>(xa + (size_t)(p / k) * Kx);
  uint4* d4 = reinterpret_cast<uint4*>(row);
  for (int i = lane; i < Kx / 8; i += 32) d4[i] = s4[i];
  if (lane == 0) {
    int32_t* tail = reinterpret_cast<int32_t*>(row + Kx);
    tail[0] = ids[p];
    tail[1] = __float_as_int(wts[p]);
    tail[2] = 0;
    tail[3] = 0;
  }
}

// received rows per local expert; a row whose expert is not held here is
// counted nowhere and flagged
__global__ void ep_hist(const __half* recvbuf, int R, int Kx, int ne, const int* own, int* counts, int* err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R) return;
  const int e = reinterpret_cast<const int32_t*>(recvbuf + (size_t)i * (Kx + kEpTailHalves) + Kx)[0];
  if (e < 0 || e >= ne || !own[e]) {
    atomicCAS(err, 0, VIREO_ERR_ARG);
    return;
  }
  atomicAdd(&counts[e], 1);
}

// received row i -> a row of its expert's range (prefill_scan's cursors)
__global__ void ep_place(const __half* recvbuf, int R, int Kx, int ne, const int* own, int* cursor, int* rrow,
                         float* wrow, __half* xg) {
  const int i = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (i >= R) return;
  const __half* row = recvbuf + (size_t)i * (Kx + kEpTailHalves);
  const int32_t* tail = reinterpret_cast<const int32_t*>(row + Kx);
  const int e = tail[0];
  int pos = -1;
  if (lane == 0) {
    if (e >= 0 && e < ne && own[e]) {
      pos = atomicAdd(&cursor[e], 1);
      wrow[pos] = __int_as_float(tail[1]);
    }
    rrow[i] = pos;
  }
  pos = __shfl_sync(0xffffffffu, pos, 0);
  if (pos < 0) return;
  const uint4* s4 = reinterpret_cast<const uint4*>(row);
  uint4* d4 = reinterpret_cast<uint4*>(xg + (size_t)pos * Kx);
  for (int c = lane; c < Kx / 8; c += 32) d4[c] = s4[c];
}

// output rows in arrival order (the order their sources expect them back)
__global__ void ep_gather(const float* y, const int* rrow, int R, int d, float* ysend) {
  const int i = blockIdx.x;
  if (i >= R) return;
  const int r = rrow[i];
  const float4* s = reinterpret_cast<const float4*>(y + (size_t)(r < 0 ? 0 : r) * d);
  float4* o = reinterpret_cast<float4*>(ysend + (size_t)i * d);
  for (int c = threadIdx.x; c < d / 4; c += blockDim.x) o[c] = r < 0 ? make_float4(0.f, 0.f, 0.f, 0.f) : s[c];
}

// x[t] += sum over rank order of the returned rows (prefill_combine's order)
__global__ void ep_combine(const int* pdest, const int* ppos, const __grid_constant__ EpOffsets so, const float* yret,
                           float* x, int T, int k, int d) {
  const int t = blockIdx.x;
  if (t >= T) return;
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float acc = 0.f;
    for (int i = 0; i < k; i++) {
      const int dst = pdest[(size_t)t * k + i];
      if (dst >= 0) acc = __fadd_rn(acc, yret[(size_t)(so.off[dst] + ppos[(size_t)t * k + i]) * d + c]);
    }
    x[(size_t)t * d + c] = __fadd_rn(x[(size_t)t * d + c], acc);
  }
}

}  // namespace vireo

using namespace vireo;

struct gguf_moe_ep {
  gguf_moe* m = nullptr;
  int rank = 0, world = 1, device = 0;
  ncclComm_t comm = nullptr;
  bool broken = false;
  std::vector<int32_t> owner;
  int32_t* d_owner = nullptr;
  int* d_own = nullptr;
  int* d_sendcnt = nullptr;  // [world]
  int* d_cntmat = nullptr;   // [world][world], row = source rank
  int* h_cntmat = nullptr;   // pinned
  int* d_rcounts = nullptr;  // [ne] received rows per expert
  int* d_pdest = nullptr;
  int* d_ppos = nullptr;
  int* d_rrow = nullptr;
  __half* sendbuf = nullptr;
  __half* recvbuf = nullptr;
  float* ysend = nullptr;
  float* yret = nullptr;
  size_t c_pairs = 0, c_recv = 0;
};

static int ep_grow(void** p, size_t* cap, size_t n, size_t bytes_each) {
  n = std::max<size_t>(n, 1);
  if (*p && *cap >= n) return VIREO_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  if (cudaMalloc(p, n * bytes_each) != cudaSuccess) {
    cudaGetLastError();
    return VIREO_ERR_NOMEM;
  }
  *cap = n;
  return VIREO_OK;
}

static double now_s() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return ts.tv_sec + 1e-9 * ts.tv_nsec;
}

// Waits for the stream with a wall-clock bound, watching the communicator
// for asynchronous errors; on either failure the communicator is aborted.
static int ep_wait(gguf_moe_ep* ep, cudaStream_t s) {
  const NcclApi& N = nccl();
  const double t0 = now_s();
  for (;;) {
    cudaError_t e = cudaStreamQuery(s);
    if (e == cudaSuccess) return VIREO_OK;
    if (e != cudaErrorNotReady) return cuda_status(e);
    ncclResult_t ae = ncclSuccess;
    if (N.getAsyncError(ep->comm, &ae) != ncclSuccess || (ae != ncclSuccess && ae != ncclInProgress)) {
      N.commAbort(ep->comm);
      ep->comm = nullptr;
      ep->broken = true;
      return VIREO_ERR_CUDA;
    }
    if (now_s() - t0 > kEpWaitSeconds) {
      N.commAbort(ep->comm);
      ep->comm = nullptr;
      ep->broken = true;
      return VIREO_ERR_TIMEOUT;
    }
    struct timespec ts = {0, 20000};
    nanosleep(&ts, nullptr);
  }
}

extern "C" {

int gguf_moe_ep_unique_id(void* id128) {
  if (!id128) return VIREO_ERR_ARG;
  const NcclApi& N = nccl();
  if (!N.ok) return VIREO_ERR_UNSUPPORTED;
  ncclUniqueId id;
  if (N.getUniqueId(&id) != ncclSuccess) return VIREO_ERR_CUDA;
  memcpy(id128, id.internal, NCCL_UNIQUE_ID_BYTES);
  return VIREO_OK;
}

int gguf_moe_ep_place(const double* expected_load, int n_experts, int world, int32_t* owner) {
  if (!expected_load || !owner || n_experts < 1 || world < 1 || world > kEpMaxWorld) return VIREO_ERR_ARG;
  // heaviest expert first onto the least-loaded rank that still has room;
  // every rank holds ceil or floor of n_experts / world experts
  std::vector<int> order(n_experts);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(),
                   [&](int a, int b) { return expected_load[a] > expected_load[b]; });
  std::vector<double> load(world, 0.0);
  std::vector<int> held(world, 0);
  const int base = n_experts / world, extra = n_experts % world;
  for (int e : order) {
    int best = -1;
    for (int r = 0; r < world; r++) {
      const int cap = base + (r < extra ? 1 : 0);
      if (held[r] >= cap) continue;
      if (best < 0 || load[r] < load[best]) best = r;
    }
    if (best < 0) return VIREO_ERR_ARG;
    owner[e] = best;
    load[best] += expected_load[e];
    held[best]++;
  }
  return VIREO_OK;
}

int gguf_moe_ep_offsets(const int32_t* counts, int world, int rank, int32_t* send_off, int32_t* recv_off,
                        int32_t* recv_cnt, int32_t* recv_total) {
  if (!counts || world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world || !send_off || !recv_off ||
      !recv_cnt)
    return VIREO_ERR_ARG;
  int64_t so = 0, ro = 0;
  for (int q = 0; q < world; q++) {
    const int32_t sc = counts[(size_t)rank * world + q], rc = counts[(size_t)q * world + rank];
    if (sc < 0 || rc < 0) return VIREO_ERR_ARG;
    send_off[q] = (int32_t)so;
    recv_off[q] = (int32_t)ro;
    recv_cnt[q] = rc;
    so += sc;
    ro += rc;
  }
  if (so > INT32_MAX || ro > INT32_MAX) return VIREO_ERR_ARG;
  if (recv_total) *recv_total = (int32_t)ro;
  return VIREO_OK;
}

void gguf_moe_ep_destroy(gguf_moe_ep* ep);

int gguf_moe_ep_create(const gguf_moe_desc* desc, const int32_t* owner, int rank, int world, const void* id128,
                       gguf_moe_ep** out) {
  if (!desc || !owner || !id128 || !out || world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world)
    return VIREO_ERR_ARG;
  *out = nullptr;
  const int ne = desc->n_experts;
  if (!prefill_supported(desc->dim, desc->ffn_exp, ne, desc->n_used, desc->router_type, desc->gate_type,
                         desc->up_type, desc->down_type))
    return VIREO_ERR_UNSUPPORTED;
  for (int e = 0; e < ne; e++)
    if (owner[e] < 0 || owner[e] >= world) return VIREO_ERR_ARG;
  const NcclApi& N = nccl();
  if (!N.ok) return VIREO_ERR_UNSUPPORTED;
  gguf_moe_ep* ep = new gguf_moe_ep();
  ep->rank = rank;
  ep->world = world;
  ep->owner.assign(owner, owner + ne);
  int st;
  if ((st = gguf_moe_create(desc, &ep->m))) {
    delete ep;
    return st;
  }
  cudaGetDevice(&ep->device);
  std::vector<int> own(ne);
  for (int e = 0; e < ne; e++) own[e] = owner[e] == rank;
  if ((st = cuda_status(cudaMalloc(&ep->d_owner, ne * 4))) || (st = cuda_status(cudaMalloc(&ep->d_own, ne * 4))) ||
      (st = cuda_status(cudaMalloc(&ep->d_sendcnt, kEpMaxWorld * 4))) ||
      (st = cuda_status(cudaMalloc(&ep->d_cntmat, kEpMaxWorld * kEpMaxWorld * 4))) ||
      (st = cuda_status(cudaMalloc(&ep->d_rcounts, 256 * 4))) ||
      (st = cuda_status(cudaMallocHost(&ep->h_cntmat, kEpMaxWorld * kEpMaxWorld * 4))) ||
      (st = cuda_status(cudaMemcpy(ep->d_owner, owner, ne * 4, cudaMemcpyHostToDevice))) ||
      (st = cuda_status(cudaMemcpy(ep->d_own, own.data(), ne * 4, cudaMemcpyHostToDevice)))) {
    gguf_moe_ep_destroy(ep);
    return st;
  }
  ncclUniqueId id;
  memcpy(id.internal, id128, NCCL_UNIQUE_ID_BYTES);
  if (N.commInitRank(&ep->comm, world, id, rank) != ncclSuccess) {
    ep->comm = nullptr;
    gguf_moe_ep_destroy(ep);
    return VIREO_ERR_CUDA;
  }
  *out = ep;
  return VIREO_OK;
}

int gguf_moe_prefill_ep(gguf_moe_ep* ep, const void* hb_bf16, float* x, int n_tok, const float* router_bias,
                        int32_t* ids_out, float* wts_out, void* stream) {
  if (!ep || n_tok < 0 || (n_tok && (!hb_bf16 || !x))) return VIREO_ERR_ARG;
  if (ep->broken || !ep->comm) return VIREO_ERR_CUDA;
  if (((uintptr_t)hb_bf16 | (uintptr_t)x) % 16) return VIREO_ERR_ARG;
  MoeView v;
  int rc;
  if ((rc = moe_view(ep->m, &v))) return rc;
  const gguf_moe_desc& D = *v.desc;
  const NcclApi& N = nccl();
  cudaStream_t s = stream ? (cudaStream_t)stream : v.stream;
  const int G = ep->world, r = ep->rank, d = D.dim, k = D.n_used, ne = D.n_experts;
  const int Kx = prefill_kx(d), rs = Kx + kEpTailHalves;
  const size_t pairs = (size_t)n_tok * k;
  PrefillLayer L;
  L.d = d;
  L.fe = D.ffn_exp;
  L.ne = ne;
  L.k = k;
  L.renorm = D.topk_renorm;
  L.router = (const float*)D.router;
  L.exp_tab = v.exp_tab;
  L.own = ep->d_own;
  PrefillScratch* S = v.pre;

  if (ep->c_pairs < pairs || !ep->d_pdest) {
    size_t c = 0;
    for (void** p : {(void**)&ep->d_pdest, (void**)&ep->d_ppos, (void**)&ep->sendbuf, (void**)&ep->yret})
      if (*p) cudaFree(*p), *p = nullptr;
    ep->c_pairs = 0;
    if ((rc = ep_grow((void**)&ep->d_pdest, &c, pairs, 4)) || (rc = ep_grow((void**)&ep->d_ppos, &c, pairs, 4)) ||
        (rc = ep_grow((void**)&ep->sendbuf, &c, pairs, (size_t)rs * 2)) ||
        (rc = ep_grow((void**)&ep->yret, &c, pairs, (size_t)d * 4)))
      return rc;
    ep->c_pairs = std::max<size_t>(pairs, 1);
  }
  // route the local tokens (this handle's router; only its own experts are packed)
  if (n_tok > 0 && (rc = prefill_route(L, S, hb_bf16, n_tok, router_bias, v.err, v.num_sms, s))) return rc;
  if (n_tok == 0 && (rc = prefill_prepare(L, S, s))) return rc;
  if ((rc = cuda_status(cudaMemsetAsync(ep->d_sendcnt, 0, G * 4, s)))) return rc;
  if (pairs) ep_route<<<(unsigned)((pairs + 255) / 256), 256, 0, s>>>(S->ids, ep->d_owner, (int)pairs, ep->d_sendcnt,
                                                                      ep->d_pdest, ep->d_ppos);
  // the [G][G] count matrix on every rank, then on the host
  if (N.allGather(ep->d_sendcnt, ep->d_cntmat, (size_t)G, ncclInt32, ep->comm, s) != ncclSuccess) return VIREO_ERR_CUDA;
  if ((rc = cuda_status(cudaMemcpyAsync(ep->h_cntmat, ep->d_cntmat, (size_t)G * G * 4, cudaMemcpyDeviceToHost, s))) ||
      (rc = ep_wait(ep, s)))
    return rc;
  int32_t soff[kEpMaxWorld], roff[kEpMaxWorld], rcnt[kEpMaxWorld], R = 0;
  if ((rc = gguf_moe_ep_offsets(ep->h_cntmat, G, r, soff, roff, rcnt, &R))) return rc;
  EpOffsets so;
  memset(&so, 0, sizeof(so));
  for (int q = 0; q < G; q++) so.off[q] = soff[q];
  // receive side buffers and the GEMM rows
  if (ep->c_recv < (size_t)R || !ep->recvbuf) {
    size_t c = 0;
    for (void** p : {(void**)&ep->recvbuf, (void**)&ep->ysend, (void**)&ep->d_rrow})
      if (*p) cudaFree(*p), *p = nullptr;
    ep->c_recv = 0;
    if ((rc = ep_grow((void**)&ep->recvbuf, &c, R, (size_t)rs * 2)) ||
        (rc = ep_grow((void**)&ep->ysend, &c, R, (size_t)d * 4)) || (rc = ep_grow((void**)&ep->d_rrow, &c, R, 4)))
      return rc;
    ep->c_recv = std::max<size_t>(R, 1);
  }
  const size_t rows = prefill_row_capacity((size_t)R, ne);
  if ((rc = prefill_grow_rows(L, S, rows))) return rc;
  // dispatch
  if (pairs)
    ep_pack<<<(unsigned)((pairs + 7) / 8), 256, 0, s>>>(S->xa, S->ids, S->wts, ep->d_pdest, ep->d_ppos, (int)pairs, k,
                                                        Kx, so, ep->sendbuf);
  const size_t rb = (size_t)rs * 2;
  if (N.groupStart() != ncclSuccess) return VIREO_ERR_CUDA;
  for (int q = 0; q < G; q++) {
    const int sc = ep->h_cntmat[r * G + q];
    if (sc > 0 && N.send((const uint8_t*)ep->sendbuf + soff[q] * rb, sc * rb, ncclUint8, q, ep->comm, s) != ncclSuccess)
      return N.groupEnd(), VIREO_ERR_CUDA;
    if (rcnt[q] > 0 && N.recv((uint8_t*)ep->recvbuf + roff[q] * rb, rcnt[q] * rb, ncclUint8, q, ep->comm, s) != ncclSuccess)
      return N.groupEnd(), VIREO_ERR_CUDA;
  }
  if (N.groupEnd() != ncclSuccess) return VIREO_ERR_CUDA;
  // experts held here
  if ((rc = cuda_status(cudaMemsetAsync(ep->d_rcounts, 0, 256 * 4, s)))) return rc;
  if (R > 0) ep_hist<<<(R + 255) / 256, 256, 0, s>>>(ep->recvbuf, R, Kx, ne, ep->d_own, ep->d_rcounts, v.err);
  prefill_scan_launch(ep->d_rcounts, ne, S, s);
  if (R > 0)
    ep_place<<<(R + 7) / 8, 256, 0, s>>>(ep->recvbuf, R, Kx, ne, ep->d_own, S->cursor, ep->d_rrow, S->wrow, S->xg);
  if ((rc = prefill_experts(L, S, rows, v.err, v.num_sms, s))) return rc;
  if (R > 0) ep_gather<<<R, 256, 0, s>>>(S->y, ep->d_rrow, R, d, ep->ysend);
  // return the output rows to their sources
  const size_t yb = (size_t)d * 4;
  if (N.groupStart() != ncclSuccess) return VIREO_ERR_CUDA;
  for (int q = 0; q < G; q++) {
    const int sc = ep->h_cntmat[r * G + q];
    if (rcnt[q] > 0 && N.send((const uint8_t*)ep->ysend + roff[q] * yb, rcnt[q] * yb, ncclUint8, q, ep->comm, s) != ncclSuccess)
      return N.groupEnd(), VIREO_ERR_CUDA;
    if (sc > 0 && N.recv((uint8_t*)ep->yret + soff[q] * yb, sc * yb, ncclUint8, q, ep->comm, s) != ncclSuccess)
      return N.groupEnd(), VIREO_ERR_CUDA;
  }
  if (N.groupEnd() != ncclSuccess) return VIREO_ERR_CUDA;
  if (n_tok > 0) ep_combine<<<n_tok, 256, 0, s>>>(ep->d_pdest, ep->d_ppos, so, ep->yret, x, n_tok, k, d);
  if (ids_out && pairs && cudaMemcpyAsync(ids_out, S->ids, pairs * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return cuda_status(cudaGetLastError());
  if (wts_out && pairs && cudaMemcpyAsync(wts_out, S->wts, pairs * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return cuda_status(cudaGetLastError());
  return cuda_status(cudaGetLastError());
}

int gguf_moe_ep_sync(gguf_moe_ep* ep, void* stream) {
  if (!ep) return VIREO_ERR_ARG;
  if (ep->broken || !ep->comm) return VIREO_ERR_CUDA;
  MoeView v;
  int rc = moe_view(ep->m, &v);
  if (rc) return rc;
  rc = ep_wait(ep, stream ? (cudaStream_t)stream : v.stream);
  if (rc) return rc;
  return gguf_moe_sync(ep->m, stream);
}

gguf_moe* gguf_moe_ep_layer(gguf_moe_ep* ep) { return ep ? ep->m : nullptr; }

void gguf_moe_ep_destroy(gguf_moe_ep* ep) {
  if (!ep) return;
  if (ep->comm) {
    const NcclApi& N = nccl();
    cudaDeviceSynchronize();
    N.commDestroy(ep->comm);
  }
  for (void* p : {(void*)ep->d_owner, (void*)ep->d_own, (void*)ep->d_sendcnt, (void*)ep->d_cntmat,
                  (void*)ep->d_rcounts, (void*)ep->d_pdest, (void*)ep->d_ppos, (void*)ep->d_rrow, (void*)ep->sendbuf,
                  (void*)ep->recvbuf, (void*)ep->ysend, (void*)ep->yret})
    if (p) cudaFree(p);
  if (ep->h_cntmat) cudaFreeHost(ep->h_cntmat);
  if (ep->m) gguf_moe_destroy(ep->m);
  delete ep;
}

}  // extern "C"
