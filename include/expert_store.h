/* ExpertStore on the GPU: an HBM-resident cache of MoE expert weights.
 *
 * Drop-in for the reference's ExpertStore (vireo src/expert_store.h:22-52):
 * the same types (ABI-identical ExpertStats, ExpertSlices, ExpertView), the
 * same calls and the same policy (lease-pinned LRU by a global tick under a
 * byte budget; over budget only when every resident expert is leased;
 * lookup of an unregistered expert returns -1 with a zeroed view; release
 * zeroes the view).  What changes is where a resident expert lives: in
 * device memory (HBM), so that the GPU kernels read it at HBM speed.
 *
 * expert_store_create (reference semantics): the backing store is the open
 * file fd (a GGUF file; slices by absolute offset) and capacity_bytes is the
 * DEVICE byte budget (0 = unbounded).  Resident experts live in CUDA managed
 * memory placed on the device: the view pointers are valid on the device and
 * on the host (a host read migrates the pages), as the reference's callers
 * and tests expect.  lookup is synchronous: the bytes are resident when it
 * returns.
 *
 * Extensions (no counterpart in the reference):
 *  - expert_store_create_host: the backing store is a host memory image
 *    (offsets relative to base; pinned by the store while it lives) and the
 *    cache is plain device memory; views are device pointers only.
 *  - expert_store_lookup_async: a miss is copied host -> device on the
 *    store's copy stream and the call returns at once; `stream` (NULL = the
 *    legacy default stream) is made to wait for the expert's copy on a miss,
 *    and also on a hit while an earlier lookup's copy of that expert may
 *    still be running.
 *  - expert_store_release_after: the lease ends when the work queued on
 *    `stream` so far has completed (the expert may not be evicted or
 *    overwritten before).
 *  - expert_store_stats_ext: copy counters.
 * Not thread-safe (as the reference).
 */
#ifndef VIREO_EXPERT_STORE_H
#define VIREO_EXPERT_STORE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    uint64_t requests, hits, misses, bytes_read;
    uint64_t resident_bytes, capacity_bytes, experts_resident;
} ExpertStats;

/* Where one expert's three weight slices live in the backing store. */
typedef struct {
    uint64_t gate_off, up_off, down_off; /* absolute byte offsets */
    uint32_t gate_bytes, up_bytes, down_bytes;
} ExpertSlices;

/* A leased view of one resident expert. Valid until release(). */
typedef struct {
    const void *gate, *up, *down;
    void *slot; /* opaque lease handle; do not touch */
} ExpertView;

typedef struct ExpertStore ExpertStore;

/* replaces src/expert_store.h:43-44 */
ExpertStore *expert_store_create(int fd, uint64_t capacity_bytes, int n_layers, int n_experts);
/* replaces src/expert_store.h:45-46 */
void expert_store_register(ExpertStore *s, int layer, int expert, const ExpertSlices *loc);
/* replaces src/expert_store.h:47-49: loads the expert to the device if it is
 * not resident (evicting the coldest unleased expert while over budget),
 * leases it and fills view; 0 on success, -1 unregistered or failed load. */
int expert_store_lookup(ExpertStore *s, int layer, int expert, ExpertView *view);
/* replaces src/expert_store.h:50 */
void expert_store_release(ExpertStore *s, ExpertView *view);
/* replaces src/expert_store.h:51 */
void expert_store_stats(const ExpertStore *s, ExpertStats *out);
/* replaces src/expert_store.h:52 */
void expert_store_destroy(ExpertStore *s);

/* ---- extensions (no reference counterpart) ---------------------------- */
ExpertStore *expert_store_create_host(const void *base, uint64_t size, uint64_t capacity_bytes, int n_layers,
                                      int n_experts);
int expert_store_lookup_async(ExpertStore *s, int layer, int expert, ExpertView *view, void *stream);
int expert_store_release_after(ExpertStore *s, ExpertView *view, void *stream);

typedef struct {
    uint64_t h2d_bytes;  /* bytes copied host -> device (misses) */
    uint64_t copies;     /* miss copies issued */
    uint64_t evictions;
    uint64_t over_budget_loads; /* loads that left resident bytes over the budget (all leased) */
} ExpertStatsExt;
void expert_store_stats_ext(const ExpertStore *s, ExpertStatsExt *out);

#ifdef __cplusplus
}
#endif
#endif
