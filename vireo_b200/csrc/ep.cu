// Expert-parallel batched MoE FFN (prefill) across the GPUs of one node.
//
// The reference has no batched path and no distribution at all (moe_ffn,
// vireo src/gguf_run.c:185-214, runs one token at a time on the host).  This
// file spreads the batched path of prefill.cu over G ranks, one process per
// GPU: rank r routes its own slice of the tokens and computes the experts
// placed on it.  The exchange is done by the kernels themselves over NVLink
// peer memory (CUDA IPC mappings of every rank's buffers), not by a copy
// collective:
//
//   route     prep + router GEMM + top-k on the local tokens (prefill.cu);
//             per expert, the local pair count and each pair's index in it
//   count     every rank stores its [ne] counts into every rank's signal
//             buffer (peer memory) and raises its flag there; once all flags
//             are up, every rank knows the [G][ne] matrix and computes from
//             it, on the device, where each of its pairs lands in its
//             expert's row range on the owning rank (the ranges are laid out
//             as prefill_scan lays them out); no host synchronisation anywhere
//             in a call
//   dispatch  one warp per token writes each pair's gate weight and origin
//             at its row on the owning rank, the token's activation row into
//             its rows on this rank, and the row ONCE into the receive buffer
//             of every other rank holding one of its experts (peer stores;
//             a token with several experts on one peer crosses NVLink once),
//             then a barrier
//   experts   the owner copies each received row into its expert rows
//             (prefill_expand), then runs the tcgen05 gate/up and down
//             GEMMs of prefill.cu over its rows; the down GEMM's epilogue
//             stores each output row, rounded to f16, into the SOURCE rank's
//             return buffer over
//             NVLink, tile by tile while the next tiles' MMAs run (one
//             kernel: GEMM + return)
//   combine   after a barrier, x[t] += sum over rank order of the returned
//             rows in fp32 (the reference's combine order, gguf_run.c:209, 213)
// Every output row comes from the same GEMM arithmetic as on one GPU, is
// rounded to f16 as on one GPU, and the combine (prefill_combine) is the
// same kernel in the same order, so the results equal gguf_moe_prefill's on
// one GPU for the same routing.
//
// Ordering across ranks: every rank's writes into a peer's buffers are
// followed by a system-scope fence and the end of the kernel; then a barrier
// over peer memory (ep_signal: each rank raises its flag of the phase, the
// number of the call, on every rank and waits, bounded, for every rank's
// flag in its own buffer); a rank reads the data only after its own copy of
// that barrier.  A buffer a peer writes in call n + 1 was last read in call
// n before this rank raised a flag of call n that the writer waited for.
//
// NCCL (communicator set-up, the IPC handle exchange, the last barrier at
// destroy) is loaded at run time (dlopen
// of libnccl.so.2; in a process that already loaded it, e.g. through PyTorch,
// that copy is used).  Host-side waits on the stream (gguf_moe_ep_sync, set-up)
// are bounded: a peer that stops answering ends them with VIREO_ERR_TIMEOUT and aborts the
// communicator.  Peer memory is only ever written with ordinary
// loads and stores; no bulk or tensor copy engine touches it.
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
#include "pdl_launch.cuh"
#include "vireo_ptx.cuh"

namespace vireo {

constexpr int kEpMaxWorld = 8;    // one node
constexpr int kEpMaxExperts = 128;
constexpr double kEpWaitSeconds = 60.0;
constexpr int kEpSplit = 4;  // warps sharing one token's row in the dispatch

// ---- NCCL entry points, resolved once ---------------------------------------
struct NcclApi {
  decltype(&ncclGetUniqueId) getUniqueId = nullptr;
  decltype(&ncclCommInitRank) commInitRank = nullptr;
  decltype(&ncclCommDestroy) commDestroy = nullptr;
  decltype(&ncclCommAbort) commAbort = nullptr;
  decltype(&ncclCommGetAsyncError) getAsyncError = nullptr;
  decltype(&ncclAllGather) allGather = nullptr;
  decltype(&ncclAllReduce) allReduce = nullptr;
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
    VIREO_NCCL_SYM(allGather, "ncclAllGather");
    VIREO_NCCL_SYM(allReduce, "ncclAllReduce");
#undef VIREO_NCCL_SYM
    api.ok = api.getUniqueId && api.commInitRank && api.commDestroy && api.commAbort && api.getAsyncError &&
             api.allGather && api.allReduce;
  });
  return api;
}

// where this rank's pairs go: every rank's operand buffers and, per expert,
// the first row this rank's pairs take in that expert's range on its owner
struct EpDispatch {
  __half* xg[kEpMaxWorld];
  float* wrow[kEpMaxWorld];
  int* ysrc[kEpMaxWorld];
  __half* xr[kEpMaxWorld];  // receive buffers: [world * max_tok][Kx], slot = source rank * max_tok + token
  int* xsrc[kEpMaxWorld];   // [rows_cap]: a row's receive slot, or -1 when placed directly
  const int* dst_off;       // [ne], device (ep_layout)
  int rows_cap;             // rows of every rank's operand buffers
  int max_tok;
};

// ---- kernels ------------------------------------------------------------------
// per expert: the local pair count and each pair's index among them
__global__ void ep_count(const int32_t* ids, int pairs, int* cnt, int* pos) {
  pdl_wait();
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= pairs) return;
  const int e = ids[p];
  pos[p] = e >= 0 ? atomicAdd(&cnt[e], 1) : -1;
}

// The row layout of every owner (gguf_moe_ep_rows on the device): experts in
// index order, each range padded to the GEMM tile, sources in rank order
// inside a range.  dst_off[e]: the first row of this rank's pairs in expert
// e's range on owner[e]; totals[e]: rows expert e receives if held here, else
// 0 (the counts prefill_scan lays out).  One block, thread e per expert.
// cstride: ints between two ranks' count rows in cntall.
__device__ void ep_layout_body(const int* cntall, int cstride, const int32_t* owner, int G, int ne, int rank,
                               int tile, int* dst_off, int* totals) {
  __shared__ int pad[kEpMaxExperts], own_s[kEpMaxExperts];
  const int e = threadIdx.x;
  int n = 0, b = 0, q = 0;
  if (e < ne) {
    for (int s = 0; s < G; s++) {
      const int c = cntall[s * cstride + e];
      if (s < rank) b += c;
      n += c;
    }
    q = owner[e];
    pad[e] = (n + tile - 1) / tile * tile;
    own_s[e] = q;
  }
  __syncthreads();
  if (e < ne) {
    int base = 0;  // padded ranges of the experts before e on the same owner
    for (int i = 0; i < e; i++)
      if (own_s[i] == q) base += pad[i];
    dst_off[e] = base + b;
    totals[e] = q == rank ? n : 0;
  }
}

// The signal buffer every rank exports (CUDA IPC): each rank's per-expert
// counts, written by that rank into every peer's copy, and one flag per
// (phase, rank) on its own 128-byte line; a flag holds the number of the
// call whose phase the rank has reached (calls are numbered alike on every
// rank: all ranks make the same calls in the same order).
struct EpSig {
  int cnt[kEpMaxWorld][kEpMaxExperts];
  unsigned int flag[3][kEpMaxWorld][32];
};
constexpr int kSigCounts = 0, kSigDispatched = 1, kSigReturned = 2;
struct EpPeers {
  EpSig* sig[kEpMaxWorld];
};

// Bounded wait until *f >= v (a peer's flag in this rank's memory).
__device__ bool ep_wait_flag(const volatile unsigned int* f, unsigned int v, int* err) {
  const unsigned long long t0 = now_ns();
  while (*f < v) {
    if (now_ns() - t0 > kWaitLimitNs) {
      atomicCAS(err, 0, VIREO_ERR_TIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// The count exchange over peer memory (in place of a count all-gather) and
// the layout: thread e stores this rank's count of expert e into every
// rank's signal buffer, the counts are made visible system-wide, thread 0
// raises this rank's counts flag on every rank, threads q < G wait for rank
// q's flag here, then the layout of ep_layout_body from the gathered counts.
__global__ void ep_exchange(int* cnt, EpSig* mine, const __grid_constant__ EpPeers P, unsigned int call,
                            const int32_t* owner, int G, int ne, int rank, int tile, int* dst_off, int* totals,
                            int* err) {
  pdl_wait();
  const int e = threadIdx.x;
  if (e < ne) {
    const int c = cnt[e];
    cnt[e] = 0;  // zero for the next call's ep_count (the buffer starts zeroed)
    for (int q = 0; q < G; q++) P.sig[q]->cnt[rank][e] = c;
  }
  __threadfence_system();
  __syncthreads();
  if (e < G) *reinterpret_cast<volatile unsigned int*>(&P.sig[e]->flag[kSigCounts][rank][0]) = call;
  __shared__ int ok;
  if (e == 0) ok = 1;
  __syncthreads();
  if (e < G && !ep_wait_flag(&mine->flag[kSigCounts][e][0], call, err)) ok = 0;
  __syncthreads();
  __threadfence_system();
  if (!ok) return;
  ep_layout_body(&mine->cnt[0][0], kEpMaxExperts, owner, G, ne, rank, tile, dst_off, totals);
}

// A barrier over peer memory: every kernel before this one on the stream has
// completed (its peer stores fenced system-wide), lane q raises this rank's
// flag of the phase on rank q and waits for rank q's flag here.
__global__ void ep_signal(EpSig* mine, const __grid_constant__ EpPeers P, int phase, unsigned int call, int G,
                          int rank, int* err) {
  pdl_wait();
  const int q = threadIdx.x;
  __threadfence_system();
  if (q < G) {
    *reinterpret_cast<volatile unsigned int*>(&P.sig[q]->flag[phase][rank][0]) = call;
    ep_wait_flag(&mine->flag[phase][q][0], call, err);
  }
  __threadfence_system();
}

// kEpSplit warps per token, each copying one part of the row.  Lane j < k
// of the first takes slot j: the gate weight, the return slot and the row's
// source (its receive slot, or -1) go to the slot's row on its owner.  The
// token's activation row is read once and
// stored into each of its rows held on this rank, and ONCE into the receive
// buffer of every other rank that holds one of its experts (that owner
// copies it into its rows: prefill_expand), so a token with several experts
// on one peer crosses NVLink once.
__global__ void ep_dispatch(const __half* __restrict__ xa, const int32_t* ids, const float* wts,
                            const int32_t* owner, const int* pos, int n_tok, int k, int Kx, int rank,
                            const __grid_constant__ EpDispatch D, int* err) {
  pdl_wait();
  const int w = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int t = w / kEpSplit, part = w % kEpSplit;
  if (t < n_tok) {
    const int p = t * k + lane;
    int q = -1, row = -1;
    if (lane < k) {
      const int e = ids[p];
      if (e >= 0) {
        q = owner[e];
        row = D.dst_off[e] + pos[p];
        if (row >= D.rows_cap) {  // inconsistent counts: never write past a buffer
          if (part == 0) atomicCAS(err, 0, VIREO_ERR_ARG);
          q = row = -1;
        } else if (part == 0) {
          D.wrow[q][row] = wts[p];
          D.ysrc[q][row] = (rank << 24) | p;
          D.xsrc[q][row] = q == rank ? -1 : rank * D.max_tok + t;
        }
      }
    }
    const unsigned remote = __reduce_or_sync(0xffffffffu, q >= 0 && q != rank ? 1u << q : 0u);
    const unsigned local = __ballot_sync(0xffffffffu, q == rank);
    const uint4* s4 = reinterpret_cast<const uint4*>(xa + (size_t)t * Kx);
    const int per = (Kx / 8 + kEpSplit - 1) / kEpSplit, c_beg = part * per, n16 = min(Kx / 8, c_beg + per);
    constexpr int kVec = 3;
    for (int c0 = c_beg + lane; c0 < n16; c0 += 32 * kVec) {
      uint4 v[kVec];
#pragma unroll
      for (int j = 0; j < kVec; j++)
        if (c0 + 32 * j < n16) v[j] = __ldg(s4 + c0 + 32 * j);
      for (unsigned m = local; m; m &= m - 1) {
        const int r2 = __shfl_sync(0xffffffffu, row, __ffs(m) - 1);
        uint4* d4 = reinterpret_cast<uint4*>(D.xg[rank] + (size_t)r2 * Kx);
#pragma unroll
        for (int j = 0; j < kVec; j++)
          if (c0 + 32 * j < n16) d4[c0 + 32 * j] = v[j];
      }
      for (unsigned m = remote; m; m &= m - 1) {
        const int q2 = __ffs(m) - 1;
        uint4* d4 = reinterpret_cast<uint4*>(D.xr[q2] + ((size_t)rank * D.max_tok + t) * Kx);
#pragma unroll
        for (int j = 0; j < kVec; j++)
          if (c0 + 32 * j < n16) d4[c0 + 32 * j] = v[j];
      }
    }
  }
  __threadfence_system();
}


}  // namespace vireo

using namespace vireo;

struct gguf_moe_ep {
  gguf_moe* m = nullptr;
  int rank = 0, world = 1, max_tok = 0, ne = 0;
  ncclComm_t comm = nullptr;
  bool broken = false;
  std::vector<int32_t> owner;
  int32_t* d_owner = nullptr;
  int* d_own = nullptr;
  int* d_cnt = nullptr;     // [ne] local pairs per expert
  int* d_totals = nullptr;  // [ne]
  int* d_dstoff = nullptr;  // [ne]
  int* d_pos = nullptr;     // [max_tok * k]
  int* d_bar = nullptr;     // barrier word
  // this rank's exported buffers (peers write them)
  size_t rows_cap = 0;
  __half* xg = nullptr;     // [rows_cap][Kx]
  float* wrow = nullptr;    // [rows_cap]
  int* ysrc = nullptr;      // [rows_cap]
  __half* yret = nullptr;   // [max_tok * k][d] f16 returned rows
  __half* xr = nullptr;     // [world * max_tok][Kx] rows received from the sources
  int* xsrc = nullptr;      // [rows_cap] receive slot of each row (-1: placed by its source)
  // every rank's buffers as mapped here (own entry = the local pointer)
  __half* p_xg[kEpMaxWorld] = {};
  float* p_wrow[kEpMaxWorld] = {};
  int* p_ysrc[kEpMaxWorld] = {};
  __half* p_yret[kEpMaxWorld] = {};
  __half* p_xr[kEpMaxWorld] = {};
  int* p_xsrc[kEpMaxWorld] = {};
  EpSig* sig = nullptr;                 // this rank's signal buffer (peers write it)
  EpSig* p_sig[kEpMaxWorld] = {};
  unsigned int call = 0;                // calls made so far (the same on every rank)
  bool mapped[kEpMaxWorld] = {};
};

static double now_s() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return ts.tv_sec + 1e-9 * ts.tv_nsec;
}

static void ep_abort(gguf_moe_ep* ep) {
  if (ep->comm) nccl().commAbort(ep->comm);
  ep->comm = nullptr;
  ep->broken = true;
}

// Waits for the stream with a wall-clock bound, watching the communicator
// for asynchronous errors; on any failure the communicator is aborted.
static int ep_wait(gguf_moe_ep* ep, cudaStream_t s) {
  const NcclApi& N = nccl();
  const double t0 = now_s();
  for (;;) {
    cudaError_t e = cudaStreamQuery(s);
    if (e == cudaSuccess) return VIREO_OK;
    if (e != cudaErrorNotReady) {
      ep_abort(ep);
      return cuda_status(e);
    }
    ncclResult_t ae = ncclSuccess;
    if (N.getAsyncError(ep->comm, &ae) != ncclSuccess || (ae != ncclSuccess && ae != ncclInProgress)) {
      ep_abort(ep);
      return VIREO_ERR_CUDA;
    }
    if (now_s() - t0 > kEpWaitSeconds) {
      ep_abort(ep);
      return VIREO_ERR_TIMEOUT;
    }
    struct timespec ts = {0, 20000};
    nanosleep(&ts, nullptr);
  }
}

static int ep_barrier(gguf_moe_ep* ep, cudaStream_t s) {
  return nccl().allReduce(ep->d_bar, ep->d_bar, 1, ncclInt32, ncclSum, ep->comm, s) == ncclSuccess ? VIREO_OK
                                                                                                   : VIREO_ERR_CUDA;
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
  if (!expected_load || !owner || n_experts < 1 || world < 1 || world > 64) return VIREO_ERR_ARG;
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

int gguf_moe_ep_rows(const int32_t* counts, const int32_t* owner, int n_experts, int world, int rank,
                     int32_t* dst_off, int32_t* rows_here) {
  if (!counts || !owner || !dst_off || n_experts < 1 || world < 1 || world > 64 || rank < 0 || rank >= world)
    return VIREO_ERR_ARG;
  const int tile = prefill_tile_rows();
  std::vector<int64_t> next(world, 0);  // running base of each owner's ranges
  int64_t here = 0;
  for (int e = 0; e < n_experts; e++) {
    const int q = owner[e];
    if (q < 0 || q >= world) return VIREO_ERR_ARG;
    int64_t total = 0, before = 0;
    for (int s = 0; s < world; s++) {
      const int32_t c = counts[(size_t)s * n_experts + e];
      if (c < 0) return VIREO_ERR_ARG;
      if (s < rank) before += c;
      total += c;
    }
    dst_off[e] = (int32_t)(next[q] + before);
    next[q] += (total + tile - 1) / tile * tile;
    if (q == rank) here += total;
  }
  for (int q = 0; q < world; q++)
    if (next[q] > INT32_MAX) return VIREO_ERR_ARG;
  if (rows_here) *rows_here = (int32_t)here;
  return VIREO_OK;
}

void gguf_moe_ep_destroy(gguf_moe_ep* ep);

int gguf_moe_ep_create(const gguf_moe_desc* desc, const int32_t* owner, int rank, int world, int max_tokens,
                       const void* id128, gguf_moe_ep** out) {
  if (!desc || !owner || !id128 || !out || world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world ||
      max_tokens < 1)
    return VIREO_ERR_ARG;
  *out = nullptr;
  const int ne = desc->n_experts, k = desc->n_used, d = desc->dim;
  if (!prefill_supported(d, desc->ffn_exp, ne, k, desc->router_type, desc->gate_type, desc->up_type,
                         desc->down_type) ||
      ne > kEpMaxExperts)
    return VIREO_ERR_UNSUPPORTED;
  if ((int64_t)max_tokens * k >= (1 << 24)) return VIREO_ERR_ARG;  // pair ids travel in 24 bits
  for (int e = 0; e < ne; e++)
    if (owner[e] < 0 || owner[e] >= world) return VIREO_ERR_ARG;
  const NcclApi& N = nccl();
  if (!N.ok) return VIREO_ERR_UNSUPPORTED;
  gguf_moe_ep* ep = new gguf_moe_ep();
  ep->rank = rank;
  ep->world = world;
  ep->max_tok = max_tokens;
  ep->ne = ne;
  ep->owner.assign(owner, owner + ne);
  int st;
  if ((st = gguf_moe_create(desc, &ep->m))) {
    delete ep;
    return st;
  }
  std::vector<int> own(ne);
  for (int e = 0; e < ne; e++) own[e] = owner[e] == rank;
  const int Kx = prefill_kx(d);
  const size_t pairs_cap = (size_t)max_tokens * k;
  // the most rows any rank can receive: every pair of every rank
  ep->rows_cap = prefill_row_capacity(pairs_cap * world, ne);
  if ((st = cuda_status(cudaMalloc(&ep->d_owner, ne * 4))) || (st = cuda_status(cudaMalloc(&ep->d_own, ne * 4))) ||
      (st = cuda_status(cudaMalloc(&ep->d_cnt, ne * 4))) ||
      (st = cuda_status(cudaMalloc(&ep->d_totals, ne * 4))) || (st = cuda_status(cudaMalloc(&ep->d_dstoff, ne * 4))) ||
      (st = cuda_status(cudaMalloc(&ep->d_pos, pairs_cap * 4))) || (st = cuda_status(cudaMalloc(&ep->d_bar, 16))) ||
      (st = cuda_status(cudaMalloc(&ep->xg, ep->rows_cap * Kx * 2))) ||
      (st = cuda_status(cudaMalloc(&ep->wrow, ep->rows_cap * 4))) ||
      (st = cuda_status(cudaMalloc(&ep->ysrc, ep->rows_cap * 4))) ||
      (st = cuda_status(cudaMalloc(&ep->yret, pairs_cap * d * 2))) ||
      (st = cuda_status(cudaMalloc(&ep->xr, (size_t)world * max_tokens * Kx * 2))) ||
      (st = cuda_status(cudaMalloc(&ep->xsrc, ep->rows_cap * 4))) ||
      (st = cuda_status(cudaMalloc(&ep->sig, sizeof(EpSig)))) ||
      (st = cuda_status(cudaMemset(ep->sig, 0, sizeof(EpSig)))) ||
      (st = cuda_status(cudaMemset(ep->d_bar, 0, 16))) || (st = cuda_status(cudaMemset(ep->d_cnt, 0, ne * 4))) ||
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
  // exchange the IPC handles of the exported buffers, with max_tokens:
  // every rank must size its buffers alike (a peer writes up to its own
  // max_tokens * n_used rows into them)
  struct {
    cudaIpcMemHandle_t h[7];
    int64_t max_tok, pad;
  } mine;
  static_assert(sizeof(mine) % 16 == 0, "exchange record");
  mine.max_tok = max_tokens;
  mine.pad = 0;
  void* bufs[7] = {ep->xg, ep->wrow, ep->ysrc, ep->yret, ep->sig, ep->xr, ep->xsrc};
  for (int i = 0; i < 7; i++)
    if ((st = cuda_status(cudaIpcGetMemHandle(&mine.h[i], bufs[i])))) {
      gguf_moe_ep_destroy(ep);
      return st;
    }
  std::vector<decltype(mine)> all((size_t)world);
  void *d_mine = nullptr, *d_all = nullptr;
  cudaStream_t s0 = nullptr;
  st = cuda_status(cudaStreamCreateWithFlags(&s0, cudaStreamNonBlocking));
  if (!st) st = cuda_status(cudaMalloc(&d_mine, sizeof(mine)));
  if (!st) st = cuda_status(cudaMalloc(&d_all, sizeof(mine) * world));
  if (!st) st = cuda_status(cudaMemcpy(d_mine, &mine, sizeof(mine), cudaMemcpyHostToDevice));
  if (!st && N.allGather(d_mine, d_all, sizeof(mine), ncclUint8, ep->comm, s0) != ncclSuccess) st = VIREO_ERR_CUDA;
  if (!st) st = ep_wait(ep, s0);
  if (!st) st = cuda_status(cudaMemcpy(all.data(), d_all, sizeof(mine) * world, cudaMemcpyDeviceToHost));
  if (d_mine) cudaFree(d_mine);
  if (d_all) cudaFree(d_all);
  if (s0) cudaStreamDestroy(s0);
  for (int q = 0; q < world && !st; q++)
    if (all[q].max_tok != max_tokens) st = VIREO_ERR_ARG;
  for (int q = 0; q < world && !st; q++) {
    if (q == rank) {
      ep->p_xg[q] = ep->xg;
      ep->p_wrow[q] = ep->wrow;
      ep->p_ysrc[q] = ep->ysrc;
      ep->p_yret[q] = ep->yret;
      ep->p_sig[q] = ep->sig;
      ep->p_xr[q] = ep->xr;
      ep->p_xsrc[q] = ep->xsrc;
      continue;
    }
    void* ptr[7] = {};
    for (int i = 0; i < 7 && !st; i++)
      st = cuda_status(cudaIpcOpenMemHandle(&ptr[i], all[q].h[i], cudaIpcMemLazyEnablePeerAccess));
    ep->p_xg[q] = (__half*)ptr[0];
    ep->p_wrow[q] = (float*)ptr[1];
    ep->p_ysrc[q] = (int*)ptr[2];
    ep->p_yret[q] = (__half*)ptr[3];
    ep->p_sig[q] = (EpSig*)ptr[4];
    ep->p_xr[q] = (__half*)ptr[5];
    ep->p_xsrc[q] = (int*)ptr[6];
    ep->mapped[q] = true;
  }
  if (st) {
    gguf_moe_ep_destroy(ep);
    return st;
  }
  *out = ep;
  return VIREO_OK;
}

int gguf_moe_prefill_ep(gguf_moe_ep* ep, const void* hb_bf16, float* x, int n_tok, const float* router_bias,
                        int32_t* ids_out, float* wts_out, void* stream) {
  if (!ep || n_tok < 0 || (n_tok && (!hb_bf16 || !x))) return VIREO_ERR_ARG;
  if (ep->broken || !ep->comm) return VIREO_ERR_CUDA;
  if (n_tok > ep->max_tok) return VIREO_ERR_ARG;
  if (((uintptr_t)hb_bf16 | (uintptr_t)x) % 16) return VIREO_ERR_ARG;
  MoeView v;
  int rc;
  if ((rc = moe_view(ep->m, &v))) return rc;
  const gguf_moe_desc& D = *v.desc;
  const NcclApi& N = nccl();
  cudaStream_t s = stream ? (cudaStream_t)stream : v.stream;
  const int G = ep->world, r = ep->rank, d = D.dim, k = D.n_used, ne = D.n_experts;
  const int Kx = prefill_kx(d);
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

  // route the local tokens (only this rank's experts are packed)
  if (n_tok > 0 && (rc = prefill_route(L, S, hb_bf16, n_tok, router_bias, v.err, v.num_sms, s))) return rc;
  if (n_tok == 0 && (rc = prefill_prepare(L, S, s))) return rc;
  if (pairs && (rc = pdl_launch(ep_count, dim3((unsigned)((pairs + 255) / 256)), dim3(256), 0, s, (const int32_t*)S->ids,
                                (int)pairs, ep->d_cnt, ep->d_pos)))
    return rc;
  // the [G][ne] count matrix on every rank, exchanged over peer memory, and
  // the row layout from it, on the device
  const unsigned int call = ++ep->call;
  EpPeers P;
  memset(&P, 0, sizeof(P));
  for (int q = 0; q < G; q++) P.sig[q] = ep->p_sig[q];
  if ((rc = pdl_launch(ep_exchange, dim3(1), dim3(kEpMaxExperts), 0, s, ep->d_cnt, ep->sig, P, call,
                       (const int32_t*)ep->d_owner, G, ne, r, prefill_tile_rows(), ep->d_dstoff, ep->d_totals, v.err)))
    return rc;
  EpDispatch Dp;
  memset(&Dp, 0, sizeof(Dp));
  for (int q = 0; q < G; q++) {
    Dp.xg[q] = ep->p_xg[q];
    Dp.wrow[q] = ep->p_wrow[q];
    Dp.ysrc[q] = ep->p_ysrc[q];
    Dp.xr[q] = ep->p_xr[q];
    Dp.xsrc[q] = ep->p_xsrc[q];
  }
  Dp.dst_off = ep->d_dstoff;
  Dp.rows_cap = (int)ep->rows_cap;
  Dp.max_tok = ep->max_tok;
  // the GEMMs of this rank run on the exported operand buffers, sized for the
  // most rows any call can bring (no host read of the counts)
  S->xg = ep->xg;
  S->wrow = ep->wrow;
  S->c_xg = ep->rows_cap * Kx * 2;
  S->c_wrow = ep->rows_cap * 4;
  const size_t rows = ep->rows_cap;
  if ((rc = prefill_grow_rows(L, S, rows))) return rc;
  // dispatch into the owners' operands (a token's row once per other owner),
  // then every rank's rows and receive buffer are in place
  if (n_tok && (rc = pdl_launch(ep_dispatch, dim3((unsigned)(((size_t)n_tok * kEpSplit + 7) / 8)), dim3(256), 0, s,
                                (const __half*)S->xa, (const int32_t*)S->ids, (const float*)S->wts,
                                (const int32_t*)ep->d_owner, (const int*)ep->d_pos, n_tok, k, Kx, r, Dp, v.err)))
    return rc;
  if ((rc = pdl_launch(ep_signal, dim3(1), dim3(32), 0, s, ep->sig, P, (int)kSigDispatched, call, G, r, v.err)))
    return rc;
  // the experts held here (rows received once per token copied into each of
  // its rows); the down GEMM returns each row to its source rank
  prefill_scan_launch(ep->d_totals, ne, S, s);
  if (G > 1) prefill_expand_launch(S, rows, ep->xsrc, ep->xr, Kx, G * ep->max_tok, s);
  if ((rc = prefill_experts(L, S, rows, v.err, v.num_sms, s, ep->ysrc, ep->p_yret, G))) return rc;
  if ((rc = pdl_launch(ep_signal, dim3(1), dim3(32), 0, s, ep->sig, P, (int)kSigReturned, call, G, r, v.err)))
    return rc;
  prefill_combine_launch(S->ids, ep->yret, x, n_tok, k, d, s);
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
  const bool clean = cudaDeviceSynchronize() == cudaSuccess;
  for (int q = 0; q < kEpMaxWorld; q++)
    if (ep->mapped[q])
      for (void* p : {(void*)ep->p_xg[q], (void*)ep->p_wrow[q], (void*)ep->p_ysrc[q], (void*)ep->p_yret[q],
                      (void*)ep->p_sig[q], (void*)ep->p_xr[q], (void*)ep->p_xsrc[q]})
        if (p) cudaIpcCloseMemHandle(p);
  if (ep->comm) {
    // the peers unmap this rank's buffers before any of them is freed: one
    // last barrier when the device is clean; after a fault the communicator
    // is aborted instead, which does not wait for peers
    const NcclApi& N = nccl();
    if (clean && ep_barrier(ep, nullptr) == VIREO_OK && cudaDeviceSynchronize() == cudaSuccess)
      N.commDestroy(ep->comm);
    else
      N.commAbort(ep->comm);
  }
  if (ep->m) {
    // the layer's batched scratch points at this handle's buffers: detach them
    MoeView v;
    if (!moe_view(ep->m, &v)) {
      if (v.pre->xg == ep->xg) v.pre->xg = nullptr, v.pre->c_xg = 0;
      if (v.pre->wrow == ep->wrow) v.pre->wrow = nullptr, v.pre->c_wrow = 0;
    }
    gguf_moe_destroy(ep->m);
  }
  for (void* p : {(void*)ep->d_owner, (void*)ep->d_own, (void*)ep->d_cnt, (void*)ep->d_totals, (void*)ep->d_dstoff,
                  (void*)ep->d_pos, (void*)ep->d_bar, (void*)ep->xg, (void*)ep->wrow, (void*)ep->ysrc,
                  (void*)ep->yret, (void*)ep->sig, (void*)ep->xr, (void*)ep->xsrc})
    if (p) cudaFree(p);
  delete ep;
}

}  // extern "C"
