// Internal launch interface between the C ABI layer (binding.cpp) and the
// sm_100a kernels (kv_adapter_cuda.cu).  Arguments are already validated by
// the caller; every function enqueues on `stream` and returns the CUDA error
// of the launch.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "kvca.h"

namespace kvca {

// Row-mover side descriptors as the kernels see them (plane table by value).
struct PagedSide {
  uint64_t planes[KVCA_MAX_PLANES];
  const int64_t* index;
  int64_t num_blocks;
  int64_t block_size;
  int64_t block_stride;
  int64_t row_stride;
};

struct ChunkSide {
  uint64_t base;
  int64_t rows_per_chunk;
  int64_t chunk_stride;
  int64_t row_stride;
  int64_t plane_stride;
};

enum class MoveKind : int { kGather = 0, kScatter = 1, kCopyPaged = 2 };

struct MoveArgs {
  MoveKind kind;
  const PagedSide* src_paged;  // gather / copy
  const ChunkSide* src_chunk;  // scatter
  const PagedSide* dst_paged;  // scatter / copy
  const ChunkSide* dst_chunk;  // gather
  int64_t num_planes;
  int64_t num_rows;
  int64_t row_bytes;
  int vec_bytes;  // 16, 8, 4, 2 or 1: widest access every address allows
  int32_t flags;
  int64_t* status;
  const int64_t* gate = nullptr;  // copy only: move nothing unless *gate != 0 (SIMT kernel)
};

cudaError_t launch_move(const MoveArgs& args, cudaStream_t stream);

// A scatter and a gather that touch disjoint bytes, in one launch when both
// move 16-byte vectors in device memory (else two launches, scatter first).
cudaError_t launch_scatter_gather(const MoveArgs& scatter, const MoveArgs& gather, cudaStream_t stream);

// The moves of a booked decode cycle in one launch (kvca_move_cycle): per
// step q, the gather of victims[offsets[q] .. offsets[q + 1]) to those spill
// rows, then the scatter of token rows q * num_seqs + s through
// cache->index (the num_steps x num_seqs slot mapping).  16-byte rows only.
struct CycleArgs {
  const PagedSide* cache;  // token view: block_size tokens per block, row_stride between tokens
  const int64_t* victims;
  int64_t num_victims;     // entries of victims
  const int64_t* offsets;  // num_steps + 1, on the device
  const ChunkSide* src;    // token rows
  const ChunkSide* spill;  // one row per victim entry
  int64_t num_planes;
  int64_t num_steps;  // 1 .. kMoveCycleMaxSteps
  int64_t num_seqs;
  int64_t spill_rows;
  int64_t token_row_bytes;
  int64_t block_row_bytes;
  int32_t flags;
  unsigned char* scratch;  // move_cycle_scratch_bytes(cache->num_blocks), zeroed once
  int64_t* status;
};

constexpr int64_t kMoveCycleMaxSteps = 32;
constexpr size_t kCycleHeaderBytes = 512;
// Bytes of one warp's share of work (an item, staged in half of the warp's
// buffer): whole rows of at most this many bytes together, longer rows in
// pieces.
#ifndef KVCA_CYCLE_ITEM_BYTES
#define KVCA_CYCLE_ITEM_BYTES 16384
#endif
constexpr int64_t kMoveCycleItemBytes = KVCA_CYCLE_ITEM_BYTES;

// Planes per item for rows of row_bytes.
inline int64_t move_cycle_group(int64_t row_bytes, int64_t num_planes) {
  int64_t g = kMoveCycleItemBytes / (row_bytes > 0 ? row_bytes : 1);
  if (g < 1) g = 1;
  return g < num_planes ? g : num_planes;
}

// Pieces per row (1 unless a row is longer than an item).
inline int64_t move_cycle_segments(int64_t row_bytes) {
  return row_bytes <= kMoveCycleItemBytes ? 1 : (row_bytes + kMoveCycleItemBytes - 1) / kMoveCycleItemBytes;
}

size_t move_cycle_scratch_bytes(int64_t num_blocks);
cudaError_t launch_move_cycle(const CycleArgs& args, cudaStream_t stream);

// Spill + fill of the same slots in one launch (one plane): row j sends slot
// slots->index[j] to store row store->index[j] and fills it from store row
// fill_from[j]; negative indices skip that part.  With *gate != 0 only the
// spill runs.
struct ExchangeArgs {
  const PagedSide* slots;
  const PagedSide* store;
  const int64_t* fill_from;
  const int64_t* gate;
  int64_t num_rows;
  int64_t row_bytes;
  int vec_bytes;
  int32_t flags;
  int64_t* status;
};

cudaError_t launch_exchange(const ExchangeArgs& args, cudaStream_t stream);

cudaError_t launch_inspect_load(int meta_bits, const int64_t* l2p, int64_t num_logical,
                                const void* meta, int64_t num_slots, const int64_t* ids,
                                int64_t count, int64_t* cur_out, uint8_t* resident_out,
                                int64_t* pin_out, void* usage_out, int64_t* status,
                                cudaStream_t stream);

cudaError_t launch_inspect_save(int meta_bits, const int64_t* l2p, int64_t num_logical,
                                const void* meta, int64_t num_slots, const int64_t* ids,
                                int64_t count, int64_t* cur_out, uint8_t* existing_out,
                                void* usage_out, int64_t* status, cudaStream_t stream);

int pop_threads_for(int meta_bits, int64_t num_slots);

// Bytes of scratch kvca_pop_reusable_slots takes: the blocked-slot bitmap,
// then (tables that the whole-GPU pop handles) its grid words and counts.
size_t pop_scratch_bytes(int64_t num_slots);

cudaError_t launch_pop(int meta_bits, int order, void* meta, int64_t num_slots,
                       int64_t* search_start, const int64_t* blocked, int64_t num_blocked,
                       int64_t count, int64_t* out, uint32_t* bitmap, int64_t* status,
                       cudaStream_t stream);

cudaError_t launch_commit_load(int meta_bits, int64_t* l2p, int64_t num_logical, int64_t* p2l,
                               void* meta, int64_t num_slots, const int64_t* evicted,
                               int64_t num_evicted, const int64_t* miss_ids,
                               const int64_t* miss_slots, int64_t num_miss,
                               const int64_t* hit_slots, const int64_t* hit_pins,
                               const void* hit_usage, int64_t num_hit, const void* miss_usage,
                               int64_t* status, cudaStream_t stream);

cudaError_t launch_commit_save(int meta_bits, int64_t* l2p, int64_t num_logical, int64_t* p2l,
                               void* meta, int64_t num_slots, const int64_t* evicted,
                               int64_t num_evicted, const int64_t* ids, const int64_t* slots,
                               const void* final_pins, const void* final_usage, int64_t count,
                               int64_t* status, cudaStream_t stream);

cudaError_t launch_release(int meta_bits, const int64_t* l2p, int64_t num_logical, void* meta,
                           int64_t num_slots, const int64_t* ids, int64_t count, int64_t* status,
                           cudaStream_t stream);

cudaError_t launch_clock_stream(int meta_bits, int order, void* meta, int64_t num_slots,
                                int64_t* search_start, int64_t num_steps, int64_t alloc_per_step,
                                const int64_t* reaccess, int64_t reaccess_per_step,
                                int64_t* victims, int64_t* steps_done, int64_t* status,
                                cudaStream_t stream);

// Bytes of the batched stream's grid words after its 32 bytes per slot.
constexpr size_t kClockStreamGridBytes = 16384;

// ctas: CTAs of the cooperative grid (0: one per SM; 1: a single CTA).
cudaError_t launch_clock_stream_batched(int meta_bits, int order, void* meta, int64_t num_slots,
                                        int64_t* search_start, int64_t num_steps,
                                        int64_t alloc_per_step, const int64_t* reaccess,
                                        int64_t reaccess_per_step, int64_t* victims,
                                        int64_t* steps_done, unsigned char* scratch, int ctas,
                                        int64_t* status, cudaStream_t stream);

cudaError_t launch_plan_load(int meta_bits, int order, const int64_t* l2p, int64_t num_logical,
                             const int64_t* p2l, void* meta, int64_t num_slots,
                             int64_t* search_start, const int64_t* ids, int64_t count,
                             uint32_t* bitmap, int64_t* result, int64_t* hit_slots,
                             int64_t* hit_pins, void* hit_usage, int64_t* miss_ids, int64_t* victims,
                             int64_t* evict_ids, int64_t* evict_slots, int64_t* counts,
                             int64_t* status, cudaStream_t stream);

cudaError_t launch_plan_save(int meta_bits, int order, const int64_t* l2p, int64_t num_logical,
                             const int64_t* p2l, void* meta, int64_t num_slots,
                             int64_t* search_start, const int64_t* ids, int64_t count,
                             uint32_t* bitmap, int64_t* selected, int64_t* move_slots,
                             void* final_pins, void* final_usage, int64_t* allocated,
                             int64_t* evict_ids, int64_t* evict_slots, int64_t* counts,
                             int64_t* status, cudaStream_t stream);

// Fused load / save with a device-resident block store: memset, plan, finish
// (metadata); the caller then enqueues the row moves (load: the exchange and
// the gated fill; save: the spill and the data scatter).  Work layouts:
// load  int64 [hit_slots, hit_pins, miss_ids, victims, evict_ids, evict_slots,
//              xslot, spill_to, fill_from] x count, meta [hit_usage] x count,
//       counts 8 words (counts[7]: the gate of the fill that follows spills);
// save  int64 [selected, allocated, evict_ids, evict_slots, move_slots] x count,
//       meta [final_pins, final_usage] x count.
cudaError_t launch_store_load_meta(int meta_bits, int order, int64_t* l2p, int64_t num_logical,
                                   int64_t* p2l, void* meta, int64_t num_slots,
                                   int64_t* search_start, const int64_t* ids, int64_t count,
                                   uint32_t* bitmap, int32_t* scratch, uint8_t* present,
                                   int64_t* work, void* work_meta, int64_t* result,
                                   int64_t* counts, int64_t* status, cudaStream_t stream);

cudaError_t launch_store_save_meta(int meta_bits, int order, int64_t* l2p, int64_t num_logical,
                                   int64_t* p2l, void* meta, int64_t num_slots,
                                   int64_t* search_start, const int64_t* ids, int64_t count,
                                   uint32_t* bitmap, int32_t* scratch, uint8_t* present,
                                   int64_t* work, void* work_meta, int64_t* counts,
                                   int64_t* status, cudaStream_t stream);

cudaError_t launch_append_step(int meta_bits, int order, void* meta, int64_t num_slots,
                               int64_t* search_start, int64_t* l2p, int64_t num_logical,
                               int64_t* p2l, const int64_t* need, int64_t num_need,
                               int64_t* cur_block, int64_t* cur_logical, int64_t* pos,
                               int64_t num_seqs, int64_t block_size, int64_t* next_logical,
                               uint32_t* bitmap, int64_t* victims, int64_t* slot_mapping,
                               int64_t* status, cudaStream_t stream);

cudaError_t launch_append_steps(int meta_bits, int order, void* meta, int64_t num_slots,
                                int64_t* search_start, int64_t* l2p, int64_t num_logical,
                                int64_t* p2l, const int64_t* need, const int64_t* need_offsets,
                                int64_t num_need, int64_t num_steps, int64_t* cur_block,
                                int64_t* cur_logical, int64_t* pos, int64_t num_seqs,
                                int64_t block_size, int64_t* next_logical, int64_t* victims,
                                int64_t* slot_mapping, int64_t* status, cudaStream_t stream);

// Rows of a small device-store call moved inside its one launch.
struct StoreRowArgs {
  uint64_t actual;
  int64_t actual_stride;
  uint64_t storage;
  int64_t storage_stride;
  uint64_t data;  // save only
  int64_t row_bytes;
  int vec;
};

// The whole device-store load / save in one single-CTA launch (plan, finish,
// row copies), for calls whose rows are small; same work layouts and results
// as launch_store_*_meta followed by the row movers.
cudaError_t launch_store_load_small(int meta_bits, int order, int64_t* l2p, int64_t num_logical, int64_t* p2l,
                                    void* meta, int64_t num_slots, int64_t* search_start, const int64_t* ids,
                                    int64_t count, uint32_t* bitmap, int32_t* scratch, uint8_t* present,
                                    int64_t* work, void* work_meta, int64_t* result, int64_t* counts,
                                    int64_t* status, const StoreRowArgs& rows, cudaStream_t stream, int64_t* host_counts = nullptr,
                                    int64_t seq = 0);
cudaError_t launch_store_save_small(int meta_bits, int order, int64_t* l2p, int64_t num_logical, int64_t* p2l,
                                    void* meta, int64_t num_slots, int64_t* search_start, const int64_t* ids,
                                    int64_t count, uint32_t* bitmap, int32_t* scratch, uint8_t* present,
                                    int64_t* work, void* work_meta, int64_t* counts, int64_t* status,
                                    const StoreRowArgs& rows, cudaStream_t stream, int64_t* host_counts = nullptr,
                                    int64_t seq = 0);

cudaError_t launch_wait_selftest(const uint32_t* flag, uint32_t from, int64_t* status,
                                 cudaStream_t stream);

}  // namespace kvca
