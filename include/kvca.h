/*
 * kvca.h - C ABI of the B200 (sm_100a) paged-KV adapter hot path.
 *
 * Two families of entry points live behind this header:
 *
 *   1. Slot metadata and the clock sweep over a packed slot_meta array.
 *      Each slot has one unsigned word holding a pin count (low half) and a
 *      usage count (high half): uint8 words carry 4+4 bits, uint16 words 8+8
 *      bits (adapter.py:17-36, adapter.py:1419-1432 of the reference).
 *      These replace the six torch-extension ops that adapter.py calls on
 *      its packed-metadata branch (csrc/ascend/adapter_meta_kernels.h:6-47,
 *      call sites adapter.py:316-330, :397-415, :437-454, :477-491,
 *      :557-593, :615-645).
 *
 *   2. Row movers between a block-paged cache and contiguous chunks.
 *      These replace actual_blocks.index_select / index_copy_
 *      (adapter.py:543, adapter.py:653-656, adapter.py:779-787) and the
 *      slot_mapping-driven single-layer KV transfer (adapter.py:1200-1243,
 *      adapter.py:1275-1285).
 *
 * Conventions
 *   - Every pointer named d_* is a device pointer on the current device.
 *   - Every entry point enqueues work on `stream` and returns without
 *     synchronising.  The return value reports host-side argument errors and
 *     launch failures only.  Errors found on the device (an id outside its
 *     table, too few reusable slots) are written to d_status, a caller-owned
 *     array of two int64 words: d_status[0] = first error code (0 = none),
 *     d_status[1] = the offending value.  The first error wins; the caller
 *     clears the words.
 *   - meta_bits selects the slot_meta word: 8 (uint8) or 16 (uint16).
 *   - No entry point allocates device memory.
 */
#ifndef KVCA_H_
#define KVCA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* kvca_stream_t; /* same type as cudaStream_t */

/* Status codes (host return values and d_status[0]). */
#define KVCA_OK 0
#define KVCA_ERR_INSUFFICIENT_CAPACITY 1 /* reference: InsufficientCapacityError, adapter.py:525 */
#define KVCA_ERR_BAD_INDEX 2             /* reference: IndexError from index_select / index_fill_ */
#define KVCA_ERR_BAD_ARGUMENT 3          /* reference: TORCH_CHECK, kv_adapter_cuda.cu:43-51 */
#define KVCA_ERR_CUDA 4                  /* launch or runtime failure */
#define KVCA_ERR_SIZE_LIMIT 5            /* table larger than a fixed-capacity entry point takes */
#define KVCA_ERR_DEVICE_TIMEOUT 6        /* a bounded device-side wait gave up (value: CTA index) */
#define KVCA_ERR_BLOCK_NOT_FOUND 7       /* reference: BlockNotFoundError, adapter.py:805 (value: id) */

/* Clock-sweep victim order (see kvca_pop_reusable_slots). */
#define KVCA_POP_ORDER_GROUPED 0
#define KVCA_POP_ORDER_PREFIX 1

/* Row-mover flags. */
#define KVCA_FLAG_SKIP_NEGATIVE 1 /* index < 0 marks a padding row: skip it, no error */
/* One side of a move lives in pinned host memory that the device reaches at
 * the same address (cudaHostAlloc under unified addressing; check with
 * kvca_host_memory_usable): rows move with plain SIMT loads and stores over
 * the host link, never with bulk copies. */
#define KVCA_FLAG_HOST_MEMORY 2
/* kvca_scatter_gather only (given in both flag words): no kernel that may
 * still run when this launch starts writes the scatter's source rows or
 * either index array; in a chain of kvca_scatter_gather launches on one
 * stream, none of them writes them (they were produced before the chain, or
 * on another stream the chain waited for).  The launch then reads them
 * while the launches before it drain, and only its reads of paged rows and
 * its stores wait for those. */
#define KVCA_FLAG_INPUTS_READY 4

/* Upper bound on planes per row-mover call. */
#define KVCA_MAX_PLANES 256

/* ABI version of this header. */
int kvca_abi_version(void);

/* Number of SMs of the current device (0 when no device is usable). */
int kvca_device_sm_count(void);

/* ------------------------------------------------------------------------ */
/* Slot metadata                                                             */
/* ------------------------------------------------------------------------ */

/*
 * Replaces inspect_load_requests (csrc/ascend/adapter_meta_kernels.h:6-9;
 * strict semantics adapter.py:417-431).  For each request i:
 *   cur[i] = l2p[ids[i]];  resident[i] = cur[i] >= 0;
 *   resident: pin_out[i] = pin(slot_meta[cur[i]]) + 1 (not wrapped),
 *             usage_out[i] = min(usage + 1, USAGE_MAX);
 *   else pin_out[i] = 0, usage_out[i] = 0.
 * usage_out has the slot_meta word type.
 */
int kvca_inspect_load_requests(int meta_bits, const int64_t* d_l2p, int64_t num_logical,
                               const void* d_slot_meta, int64_t num_slots,
                               const int64_t* d_ids, int64_t count, int64_t* d_cur_out,
                               uint8_t* d_resident_out, int64_t* d_pin_out, void* d_usage_out,
                               int64_t* d_status, kvca_stream_t stream);

/*
 * Replaces inspect_save_requests (csrc/ascend/adapter_meta_kernels.h:11-14;
 * strict semantics adapter.py:456-470).  existing[i] = cur[i] >= 0;
 * usage_out[i] = existing ? min(usage + 1, USAGE_MAX) : 1.
 */
int kvca_inspect_save_requests(int meta_bits, const int64_t* d_l2p, int64_t num_logical,
                               const void* d_slot_meta, int64_t num_slots,
                               const int64_t* d_ids, int64_t count, int64_t* d_cur_out,
                               uint8_t* d_existing_out, void* d_usage_out, int64_t* d_status,
                               kvca_stream_t stream);

/*
 * Replaces pop_reusable_slots (csrc/ascend/adapter_meta_kernels.h:16-20;
 * grouped order = the strict path adapter.py:472-525; prefix order = the
 * reference CUDA kernel's selection, csrc/kv_adapter_cuda.cu:101-231).
 *
 * A slot is available when its pin count is 0 and it is not listed in
 * d_blocked.  Scan order starts at *d_search_start and wraps.  T is the
 * smallest usage value such that at least `count` available slots have
 * usage <= T.
 *   GROUPED: all available slots with usage 0 in scan order, then usage 1,
 *            ..., then the first ones with usage T, until `count`.
 *   PREFIX:  the first `count` available slots in scan order with usage <= T.
 * If T > 0 every slot's usage becomes max(usage - T, 0).  Then
 * *d_search_start = (d_out[count - 1] + 1) % num_slots.
 * Too few available slots: d_status gets KVCA_ERR_INSUFFICIENT_CAPACITY and
 * neither slot_meta nor search_start changes.
 *
 * d_scratch_bitmap: kvca_pop_scratch_bytes(num_slots) bytes, all zero on
 * entry and zero again on exit: ceil(num_slots / 32) uint32 words of
 * blocked-slot bitmap and, for tables of 65,536 to 2^24 slots, the working
 * area of the whole-GPU sweep (those tables run on a cooperative grid of one
 * CTA per SM: each CTA takes a contiguous range of the scan order, and one
 * bounded grid barrier joins them unless the first range already holds the
 * victims).  Calls sharing one scratch must be ordered on one stream.
 */
size_t kvca_pop_scratch_bytes(int64_t num_slots);
int kvca_pop_reusable_slots(int meta_bits, int order, void* d_slot_meta, int64_t num_slots,
                            int64_t* d_search_start, const int64_t* d_blocked,
                            int64_t num_blocked, int64_t count, int64_t* d_out,
                            uint32_t* d_scratch_bitmap, int64_t* d_status,
                            kvca_stream_t stream);

/*
 * kvca_pop_reusable_slots for callers that cannot allocate device memory.
 * No counterpart in the reference: it exists for callers that may not call
 * cudaMalloc (a serving loop whose device memory is reserved up front and
 * must not touch the allocator again, host runtimes that hold no device
 * allocator, embeddings whose memory budget is fixed at start-up).  Same
 * semantics and result as kvca_pop_reusable_slots, but the blocked-slot
 * bitmap is a device array inside this library (128 KiB per GPU that loads
 * the library, held until the process exits), so there is no scratch
 * argument.
 *   - num_slots above KVCA_NOALLOC_MAX_SLOTS is rejected with
 *     KVCA_ERR_SIZE_LIMIT before anything is launched.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.
 *   - All calls on a device share the array: calls that may overlap on the
 *     GPU (different streams without ordering between them) race and must
 *     not be issued.  Each call clears the words it uses before marking its
 *     blocked slots, so whatever an earlier call left there has no effect.
 *   - d_status is required (KVCA_ERR_BAD_ARGUMENT without it when count > 0):
 *     a blocked id outside [0, num_slots) (KVCA_ERR_BAD_INDEX, value = the
 *     id) and too few reusable slots (KVCA_ERR_INSUFFICIENT_CAPACITY) are
 *     found on the device and reported only there; either leaves slot_meta
 *     and search_start untouched (d_out then holds no defined result).
 *   - The array's address is looked up once per device and kept for the
 *     life of the process; after cudaDeviceReset on a device this entry
 *     point must not be called on that device again.
 *   - Allocates nothing (no cudaMalloc, no cudaFree, no allocating library
 *     routine).
 */
#define KVCA_NOALLOC_MAX_SLOTS 1048576
int kvca_pop_reusable_slots_noalloc(int meta_bits, int order, void* d_slot_meta,
                                    int64_t num_slots, int64_t* d_search_start,
                                    const int64_t* d_blocked, int64_t num_blocked, int64_t count,
                                    int64_t* d_out, int64_t* d_status, kvca_stream_t stream);

/* Replaces choose_pop_launch_warps (csrc/binding.cpp:74-78): warps per CTA
 * of the pop kernel for a table of num_slots slots. */
int64_t kvca_choose_pop_launch_warps(int64_t num_slots);

/*
 * Replaces commit_load_metadata (csrc/ascend/adapter_meta_kernels.h:22-32;
 * strict semantics adapter.py:595-604), in this order:
 *   l2p[evicted] = -1;
 *   l2p[miss_ids] = miss_slots; p2l[miss_slots] = miss_ids;
 *   slot_meta[hit_slots] = pack(hit_pins, hit_usage);
 *   slot_meta[miss_slots] = pack(1, miss_usage).
 * hit_usage / miss_usage have the slot_meta word type.  A miss id listed
 * more than once keeps the slot of its last occurrence, as index_put_
 * applied in order leaves it.
 */
int kvca_commit_load_metadata(int meta_bits, int64_t* d_l2p, int64_t num_logical, int64_t* d_p2l,
                              void* d_slot_meta, int64_t num_slots, const int64_t* d_evicted,
                              int64_t num_evicted, const int64_t* d_miss_ids,
                              const int64_t* d_miss_slots, int64_t num_miss,
                              const int64_t* d_hit_slots, const int64_t* d_hit_pins,
                              const void* d_hit_usage, int64_t num_hit, const void* d_miss_usage,
                              int64_t* d_status, kvca_stream_t stream);

/*
 * Replaces commit_save_metadata (csrc/ascend/adapter_meta_kernels.h:34-42;
 * strict semantics adapter.py:647-651):
 *   l2p[evicted] = -1; l2p[ids] = slots; p2l[slots] = ids;
 *   slot_meta[slots] = pack(final_pins, final_usage).
 * final_pins / final_usage have the slot_meta word type.  An id listed more
 * than once keeps the slot of its last occurrence (index_put_ in order).
 */
int kvca_commit_save_metadata(int meta_bits, int64_t* d_l2p, int64_t num_logical, int64_t* d_p2l,
                              void* d_slot_meta, int64_t num_slots, const int64_t* d_evicted,
                              int64_t num_evicted, const int64_t* d_ids, const int64_t* d_slots,
                              const void* d_final_pins, const void* d_final_usage, int64_t count,
                              int64_t* d_status, kvca_stream_t stream);

/*
 * Replaces release_metadata (csrc/ascend/adapter_meta_kernels.h:44-47;
 * strict semantics adapter.py:332-336): for slot = l2p[ids[i]],
 * pin = (pin - 1) mod 2^(meta_bits/2); usage unchanged.  A released pin of 0
 * therefore wraps to the field maximum, as in the strict path.
 */
int kvca_release_metadata(int meta_bits, const int64_t* d_l2p, int64_t num_logical,
                          void* d_slot_meta, int64_t num_slots, const int64_t* d_ids,
                          int64_t count, int64_t* d_status, kvca_stream_t stream);

/*
 * Device-resident clock stream: for step s in [0, num_steps):
 *   v = pop(alloc_per_step, no blocked slots)           -> d_victims[s*alloc_per_step ...]
 *   slot_meta[v] = pack(pin(slot_meta[v]), 1)           (victim refilled, as a save miss)
 *   r = d_reaccess[s*reaccess_per_step ...]
 *   slot_meta[r] = pack(pin, min(usage + 1, USAGE_MAX)) (hits; values read before any write)
 * One launch runs every step.  On too few available slots it stops, sets
 * d_status and writes the number of completed steps to *d_steps_done.
 * reaccess_per_step <= 8192.  No reference counterpart as one call: it is the
 * strict-path sequence pop (adapter.py:472-525), commit (adapter.py:647-651)
 * and usage bump (adapter.py:1414-1416) run back to back.
 */
int kvca_clock_stream(int meta_bits, int order, void* d_slot_meta, int64_t num_slots,
                      int64_t* d_search_start, int64_t num_steps, int64_t alloc_per_step,
                      const int64_t* d_reaccess, int64_t reaccess_per_step, int64_t* d_victims,
                      int64_t* d_steps_done, int64_t* d_status, kvca_stream_t stream);

/*
 * kvca_clock_stream computed in epochs: identical results (victims,
 * slot_meta, search_start, steps_done, status), one launch.  While no pop
 * needs aging, usage never decreases, so a run of steps is resolved at once:
 * the available usage-0 slots in scan order are the candidates, and a
 * candidate is passed over exactly when its first re-access comes at a step
 * before the one that would take it.  Steps that need aging run one by one.
 * The passes over slots, candidates and events run on a cooperative grid of
 * `ctas` CTAs (0: one per SM; 1: one CTA), joined by grid barriers whose
 * waits are bounded (a wait that runs out reports KVCA_ERR_DEVICE_TIMEOUT).
 * d_scratch: kvca_clock_stream_scratch_bytes(num_slots) = 32 * num_slots +
 * 16384 bytes, 8-byte aligned, whose bytes from 20 * num_slots to
 * 32 * num_slots are zero on entry (the call leaves them zero); num_slots and
 * num_steps * alloc_per_step below 2^31.  Calls sharing scratch must be
 * ordered on one stream.
 */
size_t kvca_clock_stream_scratch_bytes(int64_t num_slots);
int kvca_clock_stream_batched(int meta_bits, int order, void* d_slot_meta, int64_t num_slots,
                              int64_t* d_search_start, int64_t num_steps, int64_t alloc_per_step,
                              const int64_t* d_reaccess, int64_t reaccess_per_step,
                              int64_t* d_victims, int64_t* d_steps_done, void* d_scratch,
                              int ctas, int64_t* d_status, kvca_stream_t stream);

/*
 * One-call planning of KVCacheAdapter.load (adapter.py:257-307, the
 * orchestration that otherwise takes inspect, two nonzero compactions, a pop
 * and an eviction-plan compaction, each synchronising the host).  One CTA:
 *   inspect, hits / misses compacted in request order (hit slots, their
 *   pin + 1 and usage + 1; miss ids), pop(#miss) with the hit slots blocked
 *   (victims), the eviction plan of the victims (evict_ids / evict_slots:
 *   victims whose previous logical id differs from the miss id), the hits'
 *   usage re-read after the pop's aging when there were misses, and the
 *   returned slot per request (result).
 * d_counts[7] = n_hit, n_miss, n_evict, error code, error value, and the
 * status word's code and value as the launch found them (an error latched
 * by an earlier launch whose status was not read yet).  Output
 * arrays hold `count` entries; only the first n_* are defined.  The caller
 * then moves the evicted payloads, loads the misses and commits with
 * kvca_commit_load_metadata (miss usage 1).  d_scratch_bitmap as for
 * kvca_pop_reusable_slots.  No reference counterpart as one call.
 */
int kvca_plan_load(int meta_bits, int order, const int64_t* d_l2p, int64_t num_logical,
                   const int64_t* d_p2l, void* d_slot_meta, int64_t num_slots,
                   int64_t* d_search_start, const int64_t* d_ids, int64_t count,
                   uint32_t* d_scratch_bitmap, int64_t* d_result, int64_t* d_hit_slots,
                   int64_t* d_hit_pins, void* d_hit_usage, int64_t* d_miss_ids,
                   int64_t* d_victims, int64_t* d_evict_ids, int64_t* d_evict_slots,
                   int64_t* d_counts, int64_t* d_status, kvca_stream_t stream);

/*
 * One-call planning of KVCacheAdapter.save (adapter.py:221-243): existing /
 * missing ids, pop(#missing) with the existing slots blocked (allocated),
 * the selected slot per request, final pins and usage read after the pop
 * (missing: 1; existing: usage + 1 saturating), and the eviction plan over
 * all selected slots in request order.  d_move_slots is d_selected with the
 * earlier occurrences of a repeated existing slot set to -1, so a row
 * scatter with KVCA_FLAG_SKIP_NEGATIVE leaves the last row, as the
 * reference's index_copy_ (adapter.py:656) applied in order does.  d_counts
 * as for kvca_plan_load with n_existing first.  The caller then spills the
 * evicted payloads, scatters the new data and commits with
 * kvca_commit_save_metadata.
 */
int kvca_plan_save(int meta_bits, int order, const int64_t* d_l2p, int64_t num_logical,
                   const int64_t* d_p2l, void* d_slot_meta, int64_t num_slots,
                   int64_t* d_search_start, const int64_t* d_ids, int64_t count,
                   uint32_t* d_scratch_bitmap, int64_t* d_selected, int64_t* d_move_slots,
                   void* d_final_pins, void* d_final_usage, int64_t* d_allocated,
                   int64_t* d_evict_ids, int64_t* d_evict_slots, int64_t* d_counts,
                   int64_t* d_status, kvca_stream_t stream);

/*
 * A block store driven from the GPU: the in-memory backend
 * (InMemoryBlockStoreBackend, adapter.py:679-833) with its storage tensor
 * on the device, or a host tier in pinned host memory (the role of
 * LMCacheBackend, adapter.py:836-1062; move_flags = KVCA_FLAG_HOST_MEMORY,
 * present and scratch stay in device memory).  Row l of the store holds
 * logical block l at
 * storage + l * storage_row_stride; present[l] != 0 once block l was saved.
 * scratch holds one int32 per logical block, zero on entry and left zero.
 */
typedef struct kvca_device_store {
  uint64_t storage;
  int64_t storage_row_stride;
  uint8_t* present;
  int32_t* scratch;
  int32_t move_flags; /* KVCA_FLAG_HOST_MEMORY when storage is pinned host memory */
} kvca_device_store;

/*
 * KVCacheAdapter.load (adapter.py:257-307) against a device-resident store,
 * enqueued as one sequence with no host synchronisation: kvca_plan_load,
 * the spill of evicted payloads into the store (backend.save_blocks,
 * adapter.py:735-756; a repeated evicted id keeps its last payload), the
 * store's presence check of the misses (adapter.py:801-806), the fill of the
 * victims from the store (adapter.py:779-787) and the commit (miss usage 1).
 * Spill and fill of each victim run in one exchange launch, so with a host
 * store both directions of the host link are busy at once; a miss that the
 * same call spills is filled by a second launch after every spill.
 * actual_blocks: slot s at d_actual + s * actual_row_stride, row_bytes each.
 * d_work: 9 * count int64, d_work_meta: count slot_meta words.  d_result:
 * the returned slot per request.  d_counts: 8 words, the first 7 as for
 * kvca_plan_load; a miss absent from the store gives code
 * KVCA_ERR_BLOCK_NOT_FOUND after the spill and before any fill or commit, as
 * the reference's backend raises.  No reference counterpart as one call.
 */
int kvca_load_device_store(int meta_bits, int order, int64_t* d_l2p, int64_t num_logical,
                           int64_t* d_p2l, void* d_slot_meta, int64_t num_slots,
                           int64_t* d_search_start, const int64_t* d_ids, int64_t count,
                           uint32_t* d_scratch_bitmap, const kvca_device_store* store,
                           uint64_t d_actual, int64_t actual_row_stride, int64_t row_bytes,
                           int64_t* d_work, void* d_work_meta, int64_t* d_result,
                           int64_t* d_counts, int64_t* d_status, kvca_stream_t stream);

/*
 * KVCacheAdapter.save (adapter.py:205-255) against a device-resident store,
 * one sequence with no host synchronisation: kvca_plan_save, the spill of
 * evicted payloads into the store, the commit and the scatter of
 * d_block_data (count rows of row_bytes, contiguous) into the selected
 * slots (a repeated slot keeps its last row).  d_work: 5 * count int64,
 * d_work_meta: 2 * count slot_meta words.  d_counts as for kvca_plan_save.
 */
int kvca_save_device_store(int meta_bits, int order, int64_t* d_l2p, int64_t num_logical,
                           int64_t* d_p2l, void* d_slot_meta, int64_t num_slots,
                           int64_t* d_search_start, const int64_t* d_ids, int64_t count,
                           uint32_t* d_scratch_bitmap, const kvca_device_store* store,
                           uint64_t d_actual, int64_t actual_row_stride, int64_t row_bytes,
                           uint64_t d_block_data, int64_t* d_work, void* d_work_meta,
                           int64_t* d_counts, int64_t* d_status, kvca_stream_t stream);

/*
 * A KVCacheAdapter over a device-resident store, described once: the
 * arguments of kvca_load_device_store / kvca_save_device_store that stay
 * the same from call to call (tables, store, cache rows, work arrays for up
 * to work_ids ids per call, the 8-word count vector on the device and a
 * pinned host copy of it, the status pair, the stream).  The session calls
 * below enqueue the same sequence as those entry points, copy the counts to
 * counts_host and wait for the stream, so a caller pays one call per
 * load / save and reads the result from host memory.  Calls on one session
 * must not overlap (one host thread).  No reference
 * counterpart as one call (the reference's load / save,
 * adapter.py:205-307, synchronise the host several times per call).
 */
typedef struct kvca_adapter_session {
  int32_t meta_bits;
  int32_t order;
  int64_t* l2p;
  int64_t num_logical;
  int64_t* p2l;
  void* slot_meta;
  int64_t num_slots;
  int64_t* search_start;
  uint32_t* scratch_bitmap;    /* kvca_pop_scratch_bytes(num_slots), zero */
  kvca_device_store store;
  uint64_t actual;
  int64_t actual_row_stride;
  int64_t row_bytes;
  int64_t* work;               /* 9 x work_ids int64 */
  void* work_meta;             /* 2 x work_ids slot_meta words */
  int64_t work_ids;
  int64_t* counts;             /* device, 8 int64 */
  int64_t* counts_host;        /* pinned host memory the device reaches at the same address, 9 int64:
                                  the last call's 8 counts, then its sequence number */
  int64_t* status;             /* device status pair */
  kvca_stream_t stream;
  int64_t sequence;            /* calls made so far (the session calls advance it) */
} kvca_adapter_session;

/* KVCacheAdapter.load of count ids (count <= work_ids): d_result gets the
 * slot of each id; counts_host the counts of kvca_load_device_store (error
 * codes included) when it returns.  When the call is one launch, that launch
 * writes the counts and the sequence number into counts_host as its last
 * action and the host waits for them there (no copy, no stream
 * synchronisation); otherwise the counts are copied and the stream waited
 * for.  Returns a host-side status. */
int kvca_session_load(kvca_adapter_session* s, const int64_t* d_ids, int64_t count, int64_t* d_result);

/* KVCacheAdapter.save of count ids and their rows (count <= work_ids);
 * counts_host gets the counts of kvca_save_device_store, as for the load. */
int kvca_session_save(kvca_adapter_session* s, const int64_t* d_ids, int64_t count, uint64_t d_block_data);

/*
 * One decode step of a paged cache's block bookkeeping, for num_seqs
 * sequences that each append one token per step.  The num_need sequences
 * d_need[] (distinct) whose current block is full get new blocks: pop
 * (kvca_pop_reusable_slots, no blocked slots) -> d_victims[num_need]; each
 * victim's previous logical id is unmapped; victim j is committed as logical
 * id *d_next_logical + j, pinned, usage 1 (kvca_commit_save_metadata with
 * pins and usage 1); the full block (slot of d_cur_logical[q]) is released
 * (kvca_release_metadata); d_cur_block / d_cur_logical / d_pos of the
 * sequence are reset and *d_next_logical advances.  Then for every sequence
 * d_slot_mapping[q] = d_cur_block[q] * block_size + d_pos[q] (the token's
 * slot, adapter.py:1275-1285) and d_pos[q] += 1.  One launch, no host
 * synchronisation (capturable in a graph).  Bad ids or too few reusable
 * slots go to d_status and change nothing.  No reference counterpart as
 * one call.
 */
int kvca_append_step(int meta_bits, int order, void* d_slot_meta, int64_t num_slots,
                     int64_t* d_search_start, int64_t* d_l2p, int64_t num_logical, int64_t* d_p2l,
                     const int64_t* d_need, int64_t num_need, int64_t* d_cur_block,
                     int64_t* d_cur_logical, int64_t* d_pos, int64_t num_seqs, int64_t block_size,
                     int64_t* d_next_logical, int64_t* d_victims, int64_t* d_slot_mapping,
                     uint32_t* d_scratch_bitmap, int64_t* d_status, kvca_stream_t stream);

/*
 * num_steps decode steps of kvca_append_step in one launch (one CTA; runs of
 * more than 256 steps take one launch per 256, in stream order): step s
 * gives new blocks to the sequences d_need[d_need_offsets[s] ..
 * d_need_offsets[s + 1]), writes their victims to d_victims from index
 * d_need_offsets[s] on and its slot_mapping to d_slot_mapping[s * num_seqs ..
 * (s + 1) * num_seqs).  The results equal num_steps kvca_append_step calls;
 * a serving loop that knows which sequences fill a block in the next steps
 * (decode with a fixed batch) books them all at once, ahead of their token
 * moves.  d_need_offsets (num_steps + 1 entries, device memory) must be
 * non-decreasing within [0, num_need] with at most num_seqs entries per step,
 * else KVCA_ERR_BAD_INDEX and nothing changes.  An error at step s (bad ids,
 * too few reusable slots) leaves steps 0..s-1 done, step s unchanged, and
 * stops.  No reference counterpart as one call (the composition is
 * adapter.py:472-525 -> :647-651 -> :309-336 per step).
 */
int kvca_append_steps(int meta_bits, int order, void* d_slot_meta, int64_t num_slots,
                      int64_t* d_search_start, int64_t* d_l2p, int64_t num_logical, int64_t* d_p2l,
                      const int64_t* d_need, const int64_t* d_need_offsets, int64_t num_need,
                      int64_t num_steps, int64_t* d_cur_block, int64_t* d_cur_logical,
                      int64_t* d_pos, int64_t num_seqs, int64_t block_size,
                      int64_t* d_next_logical, int64_t* d_victims, int64_t* d_slot_mapping,
                      int64_t* d_status, kvca_stream_t stream);

/* Failure-detection self-test: one thread waits, with the bounded wait of
 * the batched clock stream's grid barriers, for *d_flag to differ from
 * `from`.  If it does not within about 0.3 s, d_status gets
 * KVCA_ERR_DEVICE_TIMEOUT (value -1) and the kernel returns; the context
 * stays usable.  No reference counterpart. */
int kvca_wait_selftest(const uint32_t* d_flag, uint32_t from, int64_t* d_status, kvca_stream_t stream);

/* 1 when [p, p + bytes) is pinned host memory that kernels can reach at the
 * same address, else 0.  No reference counterpart. */
int kvca_host_memory_usable(const void* p, int64_t bytes);

/* ------------------------------------------------------------------------ */
/* Row movers                                                                */
/* ------------------------------------------------------------------------ */

/*
 * A paged side: num_planes planes (one per layer and K/V), each an array of
 * num_blocks blocks of block_size rows.  Row r of the call lives at
 *   plane_ptrs[p] + (idx / block_size) * block_stride + (idx % block_size) * row_stride
 * with idx = index[r] (index == NULL means idx = r).  block_size = 1 makes
 * whole blocks the rows (block-granular moves); block_size > 1 with a token
 * slot_mapping makes tokens the rows (adapter.py:1275-1285).
 * plane_ptrs is a HOST array of num_planes device addresses.
 */
typedef struct kvca_paged_desc {
  const uint64_t* plane_ptrs;
  int64_t num_blocks;
  int64_t block_size;
  int64_t block_stride;
  int64_t row_stride;
  const int64_t* index;
} kvca_paged_desc;

/*
 * A contiguous side: row r of plane p lives at
 *   base + (r / rows_per_chunk) * chunk_stride + (r % rows_per_chunk) * row_stride
 *        + p * plane_stride
 * e.g. an LMCache-style chunk [K/V x layer][rows_per_chunk][row] per chunk has
 * plane_stride = rows_per_chunk * row_bytes and
 * chunk_stride = num_planes * plane_stride.
 */
typedef struct kvca_chunk_desc {
  uint64_t base;
  int64_t rows_per_chunk;
  int64_t chunk_stride;
  int64_t row_stride;
  int64_t plane_stride;
} kvca_chunk_desc;

/*
 * Spill and fill of the same slots in one pass (one plane): for each row j,
 * the bytes of slot slots->index[j] go to store row store->index[j] and the
 * slot is then filled from store row d_fill_rows[j]; a negative store or
 * fill index skips that part, a negative slot the row.  The adapter's load
 * with evictions (backend.save_blocks of the victims, adapter.py:735-756,
 * then the fill, :779-787) as one launch: with the store in pinned host
 * memory (KVCA_FLAG_HOST_MEMORY) both directions of the host link run at
 * once.  Spill and fill store rows must be disjoint (a row spilled and
 * filled in one call has no defined order).  No reference counterpart.
 */
int kvca_exchange(const kvca_paged_desc* slots, const kvca_paged_desc* store,
                  const int64_t* d_fill_rows, int64_t num_rows, int64_t row_bytes, int32_t flags,
                  int64_t* d_status, kvca_stream_t stream);

/* Paged -> contiguous: per plane, index_select of rows (adapter.py:543). */
int kvca_gather(const kvca_paged_desc* src, const kvca_chunk_desc* dst, int64_t num_planes,
                int64_t num_rows, int64_t row_bytes, int32_t flags, int64_t* d_status,
                kvca_stream_t stream);

/* Contiguous -> paged: per plane, index_copy_ of rows (adapter.py:653-656). */
int kvca_scatter(const kvca_chunk_desc* src, const kvca_paged_desc* dst, int64_t num_planes,
                 int64_t num_rows, int64_t row_bytes, int32_t flags, int64_t* d_status,
                 kvca_stream_t stream);

/*
 * A kvca_scatter and a kvca_gather in one launch (the scatter's arguments
 * first, then the gather's, then the flags of each): the CTAs are split between the
 * two by bytes.  Results equal the two calls, provided the moves touch
 * disjoint bytes (nothing orders one before the other).  For a decode
 * loop, whose steps move a few MiB each (the token scatter of step i and the
 * spill gather of the blocks step i + 1 evicts, which step i does not
 * write), one launch instead of two.  Up to 32 MiB moved by the two
 * together the CTAs are split between the moves; above it every CTA moves
 * its share of the scatter, then of the gather.  Without 16-byte alignment,
 * or with KVCA_FLAG_HOST_MEMORY, the two moves take two launches, the
 * scatter first.  No reference counterpart.
 */
int kvca_scatter_gather(const kvca_chunk_desc* s_src, const kvca_paged_desc* s_dst, int64_t s_planes,
                        int64_t s_rows, int64_t s_row_bytes, const kvca_paged_desc* g_src,
                        const kvca_chunk_desc* g_dst, int64_t g_planes, int64_t g_rows,
                        int64_t g_row_bytes, int32_t s_flags, int32_t g_flags, int64_t* d_status,
                        kvca_stream_t stream);

/*
 * The moves of a booked decode cycle in one launch (the victims and the
 * num_steps x num_seqs slot mapping that kvca_append_steps writes).  For
 * each step q in order, with the result of running them one after the other:
 *   1. the spill gather of victims[offsets[q] .. offsets[q + 1]): block rows
 *      (block_row_bytes each, block_src->block_size 1, index = victims) of
 *      every plane to spill rows offsets[q] .. (the gather of adapter.py:543);
 *   2. the token scatter of token rows q * num_seqs + s (tokens, chunk
 *      layout; chunk_stride 0 with rows_per_chunk = num_seqs moves the same
 *      rows every step) to slots token_dst->index[q * num_seqs + s]
 *      (reshape-and-cache, adapter.py:1275-1285).
 * One cooperative launch of one CTA per SM streams every step's rows; items
 * wait for earlier steps only where a step's rows depend on them (a token
 * row landing in a block that this or an earlier step evicts waits for that
 * gather; a gather of a block that an earlier step wrote waits for that
 * scatter).  token_dst and block_src describe the same cache (same planes,
 * num_blocks and block_stride).  Slots must be distinct across the call (a
 * slot given twice ends with either row); negative slots and victims with
 * KVCA_FLAG_SKIP_NEGATIVE skip their rows, other ids outside the cache give
 * KVCA_ERR_BAD_INDEX (their rows skipped), offsets that do not start at 0,
 * decrease or pass num_victims (the entries of block_src->index) or
 * spill_rows give KVCA_ERR_BAD_ARGUMENT and move nothing.  1 <= num_steps
 * <= 32; rows, strides and addresses 16-byte aligned; a block's token rows
 * and its block row lie within block_stride.
 * d_scratch: kvca_move_cycle_scratch_bytes(num_blocks) bytes, zeroed once
 * and kept for the cache's life (launches that use one scratch must not
 * overlap); after KVCA_ERR_DEVICE_TIMEOUT zero it again.  No reference
 * counterpart.
 */
int64_t kvca_move_cycle_scratch_bytes(int64_t num_blocks);
int kvca_move_cycle(const kvca_chunk_desc* tokens, const kvca_paged_desc* token_dst, int64_t token_row_bytes,
                    const kvca_paged_desc* block_src, int64_t num_victims, const kvca_chunk_desc* spill,
                    int64_t block_row_bytes, int64_t num_planes, const int64_t* d_offsets, int64_t num_steps,
                    int64_t num_seqs, int64_t spill_rows, int32_t flags, void* d_scratch, int64_t* d_status,
                    kvca_stream_t stream);

/*
 * Measurement aid, not an adapter path: moves `rows` rows of row_bytes (64,
 * 128, 256, 576, 1152 or 2048) between two dense buffers through a uint32
 * permutation, scatter (dst row d_perm[r] = src row r) or gather (dst row r
 * = src row d_perm[r]), on `ctas` CTAs of 256 threads, with no other index
 * work.  The rate it reaches is the ceiling that random-row moves of that
 * width are measured against (the copy bandwidth is the ceiling of
 * sequential moves only).  No reference counterpart.
 */
int kvca_row_ceiling(const void* d_src, void* d_dst, const uint32_t* d_perm, int64_t rows, int64_t row_bytes,
                     int scatter, int ctas, kvca_stream_t stream);

/* Paged -> paged in one pass: dst[dst.index[r]] = src[src.index[r]]
 * (the index_select + index_copy_ pair of adapter.py:779-787). */
int kvca_copy_paged(const kvca_paged_desc* src, const kvca_paged_desc* dst, int64_t num_planes,
                    int64_t num_rows, int64_t row_bytes, int32_t flags, int64_t* d_status,
                    kvca_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* KVCA_H_ */
