// ExpertStore on the GPU: resident MoE experts in device memory, the same
// lease-LRU pager as the reference (vireo src/expert_store.c:7-111) with the
// host buffers replaced by frames of one device allocation.
//
// Reference behaviour kept: slots per (layer, expert) (:7-24); register
// records the slices and their total size (:32-37); while a miss would put
// resident bytes over a non-zero budget the coldest resident unleased expert
// (smallest last-use tick) is evicted, and when every resident expert is
// leased the load goes over budget (:46-58); a lookup counts a request, then
// a hit or a miss, stamps the slot with ++tick and takes a lease (:67-89);
// an unregistered expert gives -1 and a zeroed view (:70); release drops one
// lease and zeroes the view (:91-95); stats copy the counters (:97-102).
//
// Device side: a resident expert is one frame [gate | up | down] (each slice
// 256-byte aligned) in a chunk of device memory, allocated first-fit from a
// coalescing free list.  With a budget the chunk holds budget / (first
// expert's bytes) + 1 frames of the first expert's size, so when every
// expert has that size a frame fits whenever the byte count does; eviction
// follows the byte count alone, exactly as the reference, and a frame that
// finds no hole (slices of other sizes fragmented the chunk) gets a separate
// allocation.  Misses are copied host -> device on the store's copy stream,
// from the host image (create_host), from the fd's pages mapped and pinned,
// or through a pinned staging buffer after pread; each load records an
// event on the copy stream, and every later lookup of the expert orders the
// caller's work after it until the copy is seen complete.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <stdint.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <map>
#include <vector>

#include "expert_store.h"
#include "vireo_internal.h"

namespace {

uint64_t up256(uint64_t v) { return (v + 255) & ~(uint64_t)255; }

struct Chunk {
  uint8_t* base = nullptr;
  uint64_t size = 0;
  std::map<uint64_t, uint64_t> free_;  // offset -> bytes

  uint8_t* alloc(uint64_t need) {
    for (auto it = free_.begin(); it != free_.end(); ++it) {
      if (it->second >= need) {
        const uint64_t off = it->first, sz = it->second;
        free_.erase(it);
        if (sz > need) free_[off + need] = sz - need;
        return base + off;
      }
    }
    return nullptr;
  }
  void release(uint8_t* p, uint64_t bytes) {
    uint64_t off = (uint64_t)(p - base), sz = bytes;
    auto next = free_.lower_bound(off);
    if (next != free_.end() && off + sz == next->first) {
      sz += next->second;
      next = free_.erase(next);
    }
    if (next != free_.begin()) {
      auto prev = std::prev(next);
      if (prev->first + prev->second == off) {
        prev->second += sz;
        return;
      }
    }
    free_[off] = sz;
  }
};

struct Slot {
  ExpertSlices loc{};
  uint64_t bytes = 0;  // gate + up + down (the budget's unit, as the reference)
  uint64_t frame = 0;  // bytes of the device frame
  bool registered = false, resident = false;
  int lease = 0;
  uint64_t last_used = 0;
  uint8_t* dev = nullptr;
  int chunk = -1;  // index into chunks, or -1 for a separate allocation
  cudaEvent_t ready = nullptr;  // recorded on the copy stream after the last load
  bool loaded = false;          // that load is known to have completed
};

}  // namespace

struct ExpertStore {
  int device = 0;
  bool managed = false;  // reference-API stores: managed memory (host-readable views)
  // backing store
  int fd = -1;
  const uint8_t* image = nullptr;  // host image (create_host) or the fd's mapping
  uint64_t image_size = 0;
  bool image_mapped = false, image_registered = false;
  uint8_t* staging = nullptr;  // pinned, for pread when the fd cannot be mapped and pinned
  uint64_t staging_size = 0;
  cudaStream_t copy = nullptr;
  // cache
  int n_layers = 0, n_experts = 0;
  std::vector<Slot> slots;
  std::vector<Chunk> chunks;
  uint64_t tick = 0, resident_bytes = 0, capacity_bytes = 0;
  ExpertStats st{};
  ExpertStatsExt ext{};
  // deferred releases: (slot, event) pairs; each holds one lease
  std::vector<std::pair<int, cudaEvent_t>> pending;
  std::vector<cudaEvent_t> event_pool;
};

namespace {

cudaEvent_t get_event(ExpertStore* s) {
  if (!s->event_pool.empty()) {
    cudaEvent_t e = s->event_pool.back();
    s->event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
  return e;
}

void poll_pending(ExpertStore* s) {
  size_t w = 0;
  for (size_t i = 0; i < s->pending.size(); i++) {
    auto pr = s->pending[i];
    if (cudaEventQuery(pr.second) == cudaSuccess) {
      Slot& sl = s->slots[pr.first];
      if (sl.lease > 0) sl.lease--;
      s->event_pool.push_back(pr.second);
    } else {
      s->pending[w++] = pr;
    }
  }
  s->pending.resize(w);
  cudaGetLastError();  // cudaErrorNotReady is not an error here
}

int lru_victim(ExpertStore* s) {
  int victim = -1;
  uint64_t best = UINT64_MAX;
  for (int i = 0; i < (int)s->slots.size(); i++) {
    const Slot& sl = s->slots[i];
    if (sl.resident && sl.lease == 0 && sl.last_used < best) {
      best = sl.last_used;
      victim = i;
    }
  }
  return victim;
}

void evict(ExpertStore* s, int i) {
  Slot& sl = s->slots[i];
  if (sl.chunk >= 0) {
    s->chunks[sl.chunk].release(sl.dev, sl.frame);
  } else if (sl.dev) {
    cudaFree(sl.dev);
  }
  sl.dev = nullptr;
  sl.chunk = -1;
  sl.resident = false;
  s->resident_bytes -= sl.bytes;
  s->st.experts_resident--;
  s->ext.evictions++;
}

cudaError_t device_alloc(ExpertStore* s, uint8_t** p, uint64_t bytes) {
  if (s->managed) {
    cudaError_t e = cudaMallocManaged((void**)p, bytes);
    if (e != cudaSuccess) return e;
    cudaMemAdvise(*p, bytes, cudaMemAdviseSetPreferredLocation, s->device);
    cudaMemAdvise(*p, bytes, cudaMemAdviseSetAccessedBy, s->device);
    cudaGetLastError();  // advice is best effort
    return cudaSuccess;
  }
  return cudaMalloc((void**)p, bytes);
}

// a frame for slot i: from a chunk, else a separate allocation.  No expert
// is evicted here: eviction is the byte-count rule of lookup_impl alone.
bool place(ExpertStore* s, int i) {
  Slot& sl = s->slots[i];
  if (s->chunks.empty()) {
    // first use.  Budgeted: room for budget / bytes + 1 frames of this
    // expert's size.  Unbounded: grow by >= 256 MiB.
    Chunk c;
    c.size = s->capacity_bytes ? up256((s->capacity_bytes / std::max<uint64_t>(sl.bytes, 1) + 1) * sl.frame)
                               : std::max<uint64_t>(256ull << 20, sl.frame);
    if (device_alloc(s, &c.base, c.size) != cudaSuccess) return false;
    c.free_[0] = c.size;
    s->chunks.push_back(c);
  }
  for (;;) {
    for (int c = 0; c < (int)s->chunks.size(); c++) {
      uint8_t* p = s->chunks[c].alloc(sl.frame);
      if (p) {
        sl.dev = p;
        sl.chunk = c;
        return true;
      }
    }
    if (s->capacity_bytes) break;
    Chunk c;  // unbounded: add a chunk
    c.size = std::max<uint64_t>(256ull << 20, sl.frame);
    if (device_alloc(s, &c.base, c.size) != cudaSuccess) return false;
    c.free_[0] = c.size;
    s->chunks.push_back(c);
  }
  // no hole of this size in the budgeted chunk
  if (device_alloc(s, &sl.dev, sl.frame) != cudaSuccess) return false;
  sl.chunk = -1;
  return true;
}

// enqueue the three slice copies of slot i on the copy stream
bool load(ExpertStore* s, int i) {
  Slot& sl = s->slots[i];
  const uint64_t offs[3] = {sl.loc.gate_off, sl.loc.up_off, sl.loc.down_off};
  const uint32_t lens[3] = {sl.loc.gate_bytes, sl.loc.up_bytes, sl.loc.down_bytes};
  uint64_t dst = 0;
  bool ok = true;
  for (int k = 0; k < 3; k++) {
    s->st.bytes_read += lens[k];
    if (s->image && offs[k] + lens[k] <= s->image_size) {
      ok = ok && cudaMemcpyAsync(sl.dev + dst, s->image + offs[k], lens[k], cudaMemcpyHostToDevice, s->copy) ==
                     cudaSuccess;
    } else if (s->fd >= 0 && s->staging && lens[k] <= s->staging_size) {
      // the staging buffer is reused: the previous copy out of it must be done
      ok = ok && cudaStreamSynchronize(s->copy) == cudaSuccess;
      ok = ok && pread(s->fd, s->staging, lens[k], (off_t)offs[k]) == (ssize_t)lens[k];
      ok = ok && cudaMemcpyAsync(sl.dev + dst, s->staging, lens[k], cudaMemcpyHostToDevice, s->copy) ==
                     cudaSuccess;
    } else {
      ok = false;
    }
    s->ext.h2d_bytes += lens[k];
    dst += up256(lens[k]);
  }
  s->ext.copies++;
  if (ok && !sl.ready) ok = cudaEventCreateWithFlags(&sl.ready, cudaEventDisableTiming) == cudaSuccess;
  if (ok) ok = cudaEventRecord(sl.ready, s->copy) == cudaSuccess;
  sl.loaded = false;
  return ok;
}

// Orders work after slot i's last load: the host (sync) or `stream` (NULL =
// the legacy default stream) waits for the load's event unless the load is
// already known complete.  False if a CUDA call fails.
bool order_after_load(Slot& sl, bool sync, cudaStream_t stream) {
  if (sl.loaded || !sl.ready) return true;
  const cudaError_t q = cudaEventQuery(sl.ready);
  if (q == cudaSuccess) {
    sl.loaded = true;
    return true;
  }
  if (q != cudaErrorNotReady) return false;
  cudaGetLastError();  // cudaErrorNotReady is not an error here
  if (sync) {
    if (cudaEventSynchronize(sl.ready) != cudaSuccess) return false;
    sl.loaded = true;
    return true;
  }
  return cudaStreamWaitEvent(stream, sl.ready, 0) == cudaSuccess;
}

void fill_view(const Slot& sl, int i, ExpertView* v, ExpertStore* s) {
  v->gate = sl.dev;
  v->up = sl.dev + up256(sl.loc.gate_bytes);
  v->down = sl.dev + up256(sl.loc.gate_bytes) + up256(sl.loc.up_bytes);
  v->slot = &s->slots[i];
}

// lookup body.  sync: the view is usable by the host and by any stream on
// return; otherwise `stream` (NULL = the legacy default stream) is ordered
// after the expert's copy, on a hit as well as on a miss.
int lookup_impl(ExpertStore* s, int layer, int expert, ExpertView* view, cudaStream_t stream, bool sync) {
  if (!s || !view) return -1;
  if (layer < 0 || layer >= s->n_layers || expert < 0 || expert >= s->n_experts) {
    memset(view, 0, sizeof(*view));
    return -1;
  }
  const int i = layer * s->n_experts + expert;
  Slot& sl = s->slots[i];
  s->st.requests++;
  if (!sl.registered) {
    memset(view, 0, sizeof(*view));
    return -1;
  }
  if (sl.resident) {
    s->st.hits++;
  } else {
    s->st.misses++;
    poll_pending(s);
    if (s->capacity_bytes) {
      while (s->resident_bytes + sl.bytes > s->capacity_bytes) {
        const int v = lru_victim(s);
        if (v < 0) break;  // all resident experts are leased: stay over budget
        evict(s, v);
      }
      if (s->resident_bytes + sl.bytes > s->capacity_bytes) s->ext.over_budget_loads++;
    }
    if (!place(s, i) || !load(s, i)) {
      if (sl.dev) {
        if (sl.chunk >= 0) s->chunks[sl.chunk].release(sl.dev, sl.frame);
        else cudaFree(sl.dev);
      }
      sl.dev = nullptr;
      sl.chunk = -1;
      memset(view, 0, sizeof(*view));
      return -1;
    }
    sl.resident = true;
    s->resident_bytes += sl.bytes;
    s->st.experts_resident++;
  }
  if (!order_after_load(sl, sync, stream)) {
    cudaStreamSynchronize(s->copy);  // last resort: the copy is done when this returns
    sl.loaded = true;
  }
  sl.last_used = ++s->tick;
  sl.lease++;
  fill_view(sl, i, view, s);
  return 0;
}

ExpertStore* new_store(uint64_t capacity_bytes, int n_layers, int n_experts) {
  if (n_layers <= 0 || n_experts <= 0) return nullptr;
  ExpertStore* s = new ExpertStore();
  if (cudaGetDevice(&s->device) != cudaSuccess ||
      cudaStreamCreateWithFlags(&s->copy, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    delete s;
    return nullptr;
  }
  s->n_layers = n_layers;
  s->n_experts = n_experts;
  s->slots.resize((size_t)n_layers * n_experts);
  s->capacity_bytes = capacity_bytes;
  return s;
}

}  // namespace

extern "C" {

ExpertStore* expert_store_create(int fd, uint64_t capacity_bytes, int n_layers, int n_experts) {
  ExpertStore* s = new_store(capacity_bytes, n_layers, n_experts);
  if (!s) return nullptr;
  s->managed = true;
  s->fd = fd;
  // map the file and pin the mapping for direct DMA; else pread + pinned staging
  struct stat sb;
  if (fd >= 0 && fstat(fd, &sb) == 0 && sb.st_size > 0) {
    void* m = mmap(nullptr, (size_t)sb.st_size, PROT_READ, MAP_SHARED, fd, 0);
    if (m != MAP_FAILED) {
      if (cudaHostRegister(m, (size_t)sb.st_size, cudaHostRegisterReadOnly) == cudaSuccess) {
        s->image = (const uint8_t*)m;
        s->image_size = (uint64_t)sb.st_size;
        s->image_mapped = s->image_registered = true;
      } else {
        cudaGetLastError();
        munmap(m, (size_t)sb.st_size);
      }
    }
  }
  return s;
}

ExpertStore* expert_store_create_host(const void* base, uint64_t size, uint64_t capacity_bytes, int n_layers,
                                      int n_experts) {
  if (!base || !size) return nullptr;
  ExpertStore* s = new_store(capacity_bytes, n_layers, n_experts);
  if (!s) return nullptr;
  s->image = (const uint8_t*)base;
  s->image_size = size;
  // pin the image for the store's lifetime unless the caller already did
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, base) == cudaSuccess && attr.type == cudaMemoryTypeHost) {
    s->image_registered = false;
  } else {
    cudaGetLastError();
    if (cudaHostRegister((void*)base, size, cudaHostRegisterReadOnly) == cudaSuccess) s->image_registered = true;
    else cudaGetLastError();
  }
  return s;
}

void expert_store_register(ExpertStore* s, int layer, int expert, const ExpertSlices* loc) {
  if (!s || !loc || layer < 0 || layer >= s->n_layers || expert < 0 || expert >= s->n_experts) return;
  Slot& sl = s->slots[(size_t)layer * s->n_experts + expert];
  sl.loc = *loc;
  sl.bytes = (uint64_t)loc->gate_bytes + loc->up_bytes + loc->down_bytes;
  sl.frame = up256(loc->gate_bytes) + up256(loc->up_bytes) + up256(loc->down_bytes);
  sl.registered = true;
  // reads through pread need a staging buffer as large as the largest slice
  const uint64_t mx = std::max<uint64_t>(loc->gate_bytes, std::max(loc->up_bytes, loc->down_bytes));
  if (!s->image && s->fd >= 0 && mx > s->staging_size) {
    if (s->staging) {
      cudaStreamSynchronize(s->copy);
      cudaFreeHost(s->staging);
      s->staging = nullptr;
      s->staging_size = 0;
    }
    if (cudaMallocHost((void**)&s->staging, mx) == cudaSuccess) s->staging_size = mx;
    else cudaGetLastError();
  }
}

int expert_store_lookup(ExpertStore* s, int layer, int expert, ExpertView* view) {
  return lookup_impl(s, layer, expert, view, nullptr, true);
}

int expert_store_lookup_async(ExpertStore* s, int layer, int expert, ExpertView* view, void* stream) {
  return lookup_impl(s, layer, expert, view, (cudaStream_t)stream, false);
}

void expert_store_release(ExpertStore* s, ExpertView* view) {
  (void)s;
  if (view && view->slot) {
    Slot* sl = (Slot*)view->slot;
    if (sl->lease > 0) sl->lease--;
  }
  if (view) memset(view, 0, sizeof(*view));
}

int expert_store_release_after(ExpertStore* s, ExpertView* view, void* stream) {
  if (!s || !view) return -1;
  if (view->slot) {
    const int i = (int)((Slot*)view->slot - s->slots.data());
    cudaEvent_t e = get_event(s);
    if (e && cudaEventRecord(e, (cudaStream_t)stream) == cudaSuccess) {
      s->pending.emplace_back(i, e);  // the lease ends when the event completes
    } else {
      if (e) s->event_pool.push_back(e);
      cudaStreamSynchronize((cudaStream_t)stream);
      Slot& sl = s->slots[i];
      if (sl.lease > 0) sl.lease--;
    }
  }
  memset(view, 0, sizeof(*view));
  return 0;
}

void expert_store_stats(const ExpertStore* s, ExpertStats* out) {
  if (!s || !out) return;
  *out = s->st;
  out->resident_bytes = s->resident_bytes;
  out->capacity_bytes = s->capacity_bytes;
  out->experts_resident = s->st.experts_resident;
}

void expert_store_stats_ext(const ExpertStore* s, ExpertStatsExt* out) {
  if (!s || !out) return;
  *out = s->ext;
}

void expert_store_destroy(ExpertStore* s) {
  if (!s) return;
  if (s->copy) cudaStreamSynchronize(s->copy);
  for (auto& pr : s->pending) {
    cudaEventSynchronize(pr.second);
    cudaEventDestroy(pr.second);
  }
  for (cudaEvent_t e : s->event_pool) cudaEventDestroy(e);
  for (auto& sl : s->slots) {
    if (sl.resident && sl.chunk < 0 && sl.dev) cudaFree(sl.dev);
    if (sl.ready) cudaEventDestroy(sl.ready);
  }
  for (auto& c : s->chunks) cudaFree(c.base);
  if (s->staging) cudaFreeHost(s->staging);
  if (s->image_registered) cudaHostUnregister((void*)s->image);
  if (s->image_mapped) munmap((void*)s->image, (size_t)s->image_size);
  if (s->copy) cudaStreamDestroy(s->copy);
  delete s;
}

}  // extern "C"
