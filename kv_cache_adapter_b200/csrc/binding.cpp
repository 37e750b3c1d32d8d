// C ABI of the adapter hot path (declared in include/kvca.h).
//
// This layer checks host-visible arguments (sizes, null pointers, word
// widths, plane counts), picks the widest vector access that every address
// and stride allows, and hands off to the sm_100a launchers.  It allocates
// nothing and never synchronises the stream.

#include <chrono>

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "kvca.h"
#include "kvca_launch.h"

namespace {

constexpr int kAbiVersion = 1;

int status_of(cudaError_t e) { return e == cudaSuccess ? KVCA_OK : KVCA_ERR_CUDA; }

bool valid_meta_bits(int bits) { return bits == 8 || bits == 16; }

// Largest power-of-two access width (<= 16) dividing x.
int align_of(uint64_t x) {
  if (x % 16 == 0) return 16;
  if (x % 8 == 0) return 8;
  if (x % 4 == 0) return 4;
  if (x % 2 == 0) return 2;
  return 1;
}

int min_align(int a, uint64_t x) {
  const int b = align_of(x);
  return a < b ? a : b;
}

bool check_paged(const kvca_paged_desc* d, int64_t num_planes, int64_t row_bytes, int* vec) {
  if (d == nullptr || d->plane_ptrs == nullptr) return false;
  if (d->num_blocks < 0 || d->block_size < 1 || d->block_stride < 0 || d->row_stride < 0)
    return false;
  if (d->block_size > 1 && d->row_stride < row_bytes) return false;
  for (int64_t p = 0; p < num_planes; ++p) {
    if (d->plane_ptrs[p] == 0) return false;
    *vec = min_align(*vec, d->plane_ptrs[p]);
  }
  *vec = min_align(*vec, static_cast<uint64_t>(d->block_stride));
  *vec = min_align(*vec, static_cast<uint64_t>(d->row_stride));
  return true;
}

bool check_chunk(const kvca_chunk_desc* d, int* vec) {
  if (d == nullptr || d->base == 0) return false;
  if (d->rows_per_chunk < 1 || d->chunk_stride < 0 || d->row_stride < 0 || d->plane_stride < 0)
    return false;
  *vec = min_align(*vec, d->base);
  *vec = min_align(*vec, static_cast<uint64_t>(d->chunk_stride));
  *vec = min_align(*vec, static_cast<uint64_t>(d->row_stride));
  *vec = min_align(*vec, static_cast<uint64_t>(d->plane_stride));
  return true;
}

void to_side(const kvca_paged_desc* d, int64_t num_planes, kvca::PagedSide* s) {
  memset(s, 0, sizeof(*s));
  for (int64_t p = 0; p < num_planes; ++p) s->planes[p] = d->plane_ptrs[p];
  s->index = d->index;
  s->num_blocks = d->num_blocks;
  s->block_size = d->block_size;
  s->block_stride = d->block_stride;
  s->row_stride = d->row_stride;
}

void to_side(const kvca_chunk_desc* d, kvca::ChunkSide* s) {
  s->base = d->base;
  s->rows_per_chunk = d->rows_per_chunk;
  s->chunk_stride = d->chunk_stride;
  s->row_stride = d->row_stride;
  s->plane_stride = d->plane_stride;
}

bool common_move_args_ok(int64_t num_planes, int64_t num_rows, int64_t row_bytes) {
  return num_planes >= 1 && num_planes <= KVCA_MAX_PLANES && num_rows >= 0 && row_bytes >= 1;
}

// A device-store call whose rows total at most this many bytes runs as one
// single-CTA launch (plan, finish and row copies): its cost is launches and
// dependent round trips, not bandwidth.  Over the host link one CTA moves
// less, so the limit is lower for a pinned store.
constexpr int64_t kSmallStoreBytes = 256 * 1024;
constexpr int64_t kSmallHostStoreBytes = 64 * 1024;

bool small_store_call(int64_t count, int64_t row_bytes, int32_t move_flags) {
  const int64_t limit = (move_flags & KVCA_FLAG_HOST_MEMORY) ? kSmallHostStoreBytes : kSmallStoreBytes;
  return count <= limit / (row_bytes > 0 ? row_bytes : 1);
}

}  // namespace

extern "C" {

int kvca_abi_version(void) { return kAbiVersion; }

int kvca_device_sm_count(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return sms;
}

int kvca_inspect_load_requests(int meta_bits, const int64_t* d_l2p, int64_t num_logical,
                               const void* d_slot_meta, int64_t num_slots,
                               const int64_t* d_ids, int64_t count, int64_t* d_cur_out,
                               uint8_t* d_resident_out, int64_t* d_pin_out, void* d_usage_out,
                               int64_t* d_status, kvca_stream_t stream) {
  if (!valid_meta_bits(meta_bits) || count < 0 || num_logical < 0 || num_slots < 0)
    return KVCA_ERR_BAD_ARGUMENT;
  if (count == 0) return KVCA_OK;
  if (!d_l2p || !d_slot_meta || !d_ids || !d_cur_out || !d_resident_out || !d_pin_out ||
      !d_usage_out)
    return KVCA_ERR_BAD_ARGUMENT;
  return status_of(kvca::launch_inspect_load(meta_bits, d_l2p, num_logical, d_slot_meta,
                                             num_slots, d_ids, count, d_cur_out, d_resident_out,
                                             d_pin_out, d_usage_out, d_status, stream));
}

int kvca_inspect_save_requests(int meta_bits, const int64_t* d_l2p, int64_t num_logical,
                               const void* d_slot_meta, int64_t num_slots,
                               const int64_t* d_ids, int64_t count, int64_t* d_cur_out,
                               uint8_t* d_existing_out, void* d_usage_out, int64_t* d_status,
                               kvca_stream_t stream) {
  if (!valid_meta_bits(meta_bits) || count < 0 || num_logical < 0 || num_slots < 0)
    return KVCA_ERR_BAD_ARGUMENT;
  if (count == 0) return KVCA_OK;
  if (!d_l2p || !d_slot_meta || !d_ids || !d_cur_out || !d_existing_out || !d_usage_out)
    return KVCA_ERR_BAD_ARGUMENT;
  return status_of(kvca::launch_inspect_save(meta_bits, d_l2p, num_logical, d_slot_meta,
                                             num_slots, d_ids, count, d_cur_out, d_existing_out,
                                             d_usage_out, d_status, stream));
}

size_t kvca_pop_scratch_bytes(int64_t num_slots) { return kvca::pop_scratch_bytes(num_slots); }

int kvca_pop_reusable_slots(int meta_bits, int order, void* d_slot_meta, int64_t num_slots,
                            int64_t* d_search_start, const int64_t* d_blocked,
                            int64_t num_blocked, int64_t count, int64_t* d_out,
                            uint32_t* d_scratch_bitmap, int64_t* d_status,
                            kvca_stream_t stream) {
  if (!valid_meta_bits(meta_bits)) return KVCA_ERR_BAD_ARGUMENT;
  if (order != KVCA_POP_ORDER_GROUPED && order != KVCA_POP_ORDER_PREFIX)
    return KVCA_ERR_BAD_ARGUMENT;
  if (num_slots <= 0 || count < 0 || num_blocked < 0) return KVCA_ERR_BAD_ARGUMENT;
  if (count == 0) return KVCA_OK;
  if (!d_slot_meta || !d_search_start || !d_out || !d_scratch_bitmap) return KVCA_ERR_BAD_ARGUMENT;
  if (num_blocked > 0 && !d_blocked) return KVCA_ERR_BAD_ARGUMENT;
  return status_of(kvca::launch_pop(meta_bits, order, d_slot_meta, num_slots, d_search_start,
                                    d_blocked, num_blocked, count, d_out, d_scratch_bitmap,
                                    d_status, stream));
}

int64_t kvca_choose_pop_launch_warps(int64_t num_slots) {
  if (num_slots <= 0) return 0;
  return kvca::pop_threads_for(8, num_slots) / 32;
}

int kvca_commit_load_metadata(int meta_bits, int64_t* d_l2p, int64_t num_logical, int64_t* d_p2l,
                              void* d_slot_meta, int64_t num_slots, const int64_t* d_evicted,
                              int64_t num_evicted, const int64_t* d_miss_ids,
                              const int64_t* d_miss_slots, int64_t num_miss,
                              const int64_t* d_hit_slots, const int64_t* d_hit_pins,
                              const void* d_hit_usage, int64_t num_hit, const void* d_miss_usage,
                              int64_t* d_status, kvca_stream_t stream) {
  if (!valid_meta_bits(meta_bits) || num_evicted < 0 || num_miss < 0 || num_hit < 0 ||
      num_logical < 0 || num_slots < 0)
    return KVCA_ERR_BAD_ARGUMENT;
  if (num_evicted == 0 && num_miss == 0 && num_hit == 0) return KVCA_OK;
  if (!d_l2p || !d_p2l || !d_slot_meta) return KVCA_ERR_BAD_ARGUMENT;
  if (num_evicted > 0 && !d_evicted) return KVCA_ERR_BAD_ARGUMENT;
  if (num_miss > 0 && (!d_miss_ids || !d_miss_slots || !d_miss_usage)) return KVCA_ERR_BAD_ARGUMENT;
  if (num_hit > 0 && (!d_hit_slots || !d_hit_pins || !d_hit_usage)) return KVCA_ERR_BAD_ARGUMENT;
  return status_of(kvca::launch_commit_load(
      meta_bits, d_l2p, num_logical, d_p2l, d_slot_meta, num_slots, d_evicted, num_evicted,
      d_miss_ids, d_miss_slots, num_miss, d_hit_slots, d_hit_pins, d_hit_usage, num_hit,
      d_miss_usage, d_status, stream));
}

int kvca_commit_save_metadata(int meta_bits, int64_t* d_l2p, int64_t num_logical, int64_t* d_p2l,
                              void* d_slot_meta, int64_t num_slots, const int64_t* d_evicted,
                              int64_t num_evicted, const int64_t* d_ids, const int64_t* d_slots,
                              const void* d_final_pins, const void* d_final_usage, int64_t count,
                              int64_t* d_status, kvca_stream_t stream) {
  if (!valid_meta_bits(meta_bits) || num_evicted < 0 || count < 0 || num_logical < 0 ||
      num_slots < 0)
    return KVCA_ERR_BAD_ARGUMENT;
  if (num_evicted == 0 && count == 0) return KVCA_OK;
  if (!d_l2p || !d_p2l || !d_slot_meta) return KVCA_ERR_BAD_ARGUMENT;
  if (num_evicted > 0 && !d_evicted) return KVCA_ERR_BAD_ARGUMENT;
  if (count > 0 && (!d_ids || !d_slots || !d_final_pins || !d_final_usage))
    return KVCA_ERR_BAD_ARGUMENT;
  return status_of(kvca::launch_commit_save(meta_bits, d_l2p, num_logical, d_p2l, d_slot_meta,
                                            num_slots, d_evicted, num_evicted, d_ids, d_slots,
                                            d_final_pins, d_final_usage, count, d_status,
                                            stream));
}

int kvca_release_metadata(int meta_bits, const int64_t* d_l2p, int64_t num_logical,
                          void* d_slot_meta, int64_t num_slots, const int64_t* d_ids,
                          int64_t count, int64_t* d_status, kvca_stream_t stream) {
  if (!valid_meta_bits(meta_bits) || count < 0 || num_logical < 0 || num_slots < 0)
    return KVCA_ERR_BAD_ARGUMENT;
  if (count == 0) return KVCA_OK;
  if (!d_l2p || !d_slot_meta || !d_ids) return KVCA_ERR_BAD_ARGUMENT;
  return status_of(kvca::launch_release(meta_bits, d_l2p, num_logical, d_slot_meta, num_slots,
                                        d_ids, count, d_status, stream));
}

int kvca_clock_stream(int meta_bits, int order, void* d_slot_meta, int64_t num_slots,
                      int64_t* d_search_start, int64_t num_steps, int64_t alloc_per_step,
                      const int64_t* d_reaccess, int64_t reaccess_per_step, int64_t* d_victims,
                      int64_t* d_steps_done, int64_t* d_status, kvca_stream_t stream) {
  if (!valid_meta_bits(meta_bits)) return KVCA_ERR_BAD_ARGUMENT;
  if (order != KVCA_POP_ORDER_GROUPED && order != KVCA_POP_ORDER_PREFIX)
    return KVCA_ERR_BAD_ARGUMENT;
  if (num_slots <= 0 || num_steps < 0 || alloc_per_step < 1 || reaccess_per_step < 0 ||
      reaccess_per_step > 8192)
    return KVCA_ERR_BAD_ARGUMENT;
  if (!d_slot_meta || !d_search_start || !d_steps_done) return KVCA_ERR_BAD_ARGUMENT;
  if (num_steps == 0)  // nothing to run: no victims buffer needed
    return status_of(cudaMemsetAsync(d_steps_done, 0, sizeof(int64_t), stream));
  if (!d_victims) return KVCA_ERR_BAD_ARGUMENT;
  if (reaccess_per_step > 0 && !d_reaccess) return KVCA_ERR_BAD_ARGUMENT;
  return status_of(kvca::launch_clock_stream(meta_bits, order, d_slot_meta, num_slots,
                                             d_search_start, num_steps, alloc_per_step,
                                             d_reaccess, reaccess_per_step, d_victims,
                                             d_steps_done, d_status, stream));
}

size_t kvca_clock_stream_scratch_bytes(int64_t num_slots) {
  if (num_slots <= 0) return 0;
  return static_cast<size_t>(num_slots) * 32 + kvca::kClockStreamGridBytes;
}

int kvca_clock_stream_batched(int meta_bits, int order, void* d_slot_meta, int64_t num_slots,
                              int64_t* d_search_start, int64_t num_steps, int64_t alloc_per_step,
                              const int64_t* d_reaccess, int64_t reaccess_per_step,
                              int64_t* d_victims, int64_t* d_steps_done, void* d_scratch,
                              int ctas, int64_t* d_status, kvca_stream_t stream) {
  if (!valid_meta_bits(meta_bits) || ctas < 0) return KVCA_ERR_BAD_ARGUMENT;
  if (order != KVCA_POP_ORDER_GROUPED && order != KVCA_POP_ORDER_PREFIX)
    return KVCA_ERR_BAD_ARGUMENT;
  const int64_t limit = INT32_MAX - 2;
  if (num_slots <= 0 || num_slots > limit || num_steps < 0 || num_steps > limit ||
      alloc_per_step < 1 || alloc_per_step > limit || reaccess_per_step < 0 ||
      reaccess_per_step > 8192 || num_steps * alloc_per_step > limit)
    return KVCA_ERR_BAD_ARGUMENT;
  if (!d_slot_meta || !d_search_start || !d_steps_done || !d_scratch) return KVCA_ERR_BAD_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(d_scratch) & 7u) != 0u) return KVCA_ERR_BAD_ARGUMENT;
  if (num_steps == 0)  // nothing to run: no victims buffer needed
    return status_of(cudaMemsetAsync(d_steps_done, 0, sizeof(int64_t), stream));
  if (!d_victims) return KVCA_ERR_BAD_ARGUMENT;
  if (reaccess_per_step > 0 && !d_reaccess) return KVCA_ERR_BAD_ARGUMENT;
  return status_of(kvca::launch_clock_stream_batched(
      meta_bits, order, d_slot_meta, num_slots, d_search_start, num_steps, alloc_per_step,
      d_reaccess, reaccess_per_step, d_victims, d_steps_done,
      reinterpret_cast<unsigned char*>(d_scratch), ctas, d_status, stream));
}

static bool plan_args_ok(int meta_bits, int order, const int64_t* l2p, int64_t num_logical,
                         const int64_t* p2l, const void* meta, int64_t num_slots,
                         const int64_t* search_start, const int64_t* ids, int64_t count,
                         const uint32_t* bitmap, const int64_t* counts) {
  return valid_meta_bits(meta_bits) &&
         (order == KVCA_POP_ORDER_GROUPED || order == KVCA_POP_ORDER_PREFIX) && num_logical > 0 &&
         num_slots > 0 && count > 0 && l2p && p2l && meta && search_start && ids && bitmap && counts;
}

int kvca_plan_load(int meta_bits, int order, const int64_t* d_l2p, int64_t num_logical,
                   const int64_t* d_p2l, void* d_slot_meta, int64_t num_slots,
                   int64_t* d_search_start, const int64_t* d_ids, int64_t count,
                   uint32_t* d_scratch_bitmap, int64_t* d_result, int64_t* d_hit_slots,
                   int64_t* d_hit_pins, void* d_hit_usage, int64_t* d_miss_ids,
                   int64_t* d_victims, int64_t* d_evict_ids, int64_t* d_evict_slots,
                   int64_t* d_counts, int64_t* d_status, kvca_stream_t stream) {
  if (!plan_args_ok(meta_bits, order, d_l2p, num_logical, d_p2l, d_slot_meta, num_slots,
                    d_search_start, d_ids, count, d_scratch_bitmap, d_counts) ||
      !d_result || !d_hit_slots || !d_hit_pins || !d_hit_usage || !d_miss_ids || !d_victims ||
      !d_evict_ids || !d_evict_slots)
    return KVCA_ERR_BAD_ARGUMENT;
  return status_of(kvca::launch_plan_load(
      meta_bits, order, d_l2p, num_logical, d_p2l, d_slot_meta, num_slots, d_search_start, d_ids,
      count, d_scratch_bitmap, d_result, d_hit_slots, d_hit_pins, d_hit_usage, d_miss_ids,
      d_victims, d_evict_ids, d_evict_slots, d_counts, d_status, stream));
}

int kvca_plan_save(int meta_bits, int order, const int64_t* d_l2p, int64_t num_logical,
                   const int64_t* d_p2l, void* d_slot_meta, int64_t num_slots,
                   int64_t* d_search_start, const int64_t* d_ids, int64_t count,
                   uint32_t* d_scratch_bitmap, int64_t* d_selected, int64_t* d_move_slots,
                   void* d_final_pins, void* d_final_usage, int64_t* d_allocated,
                   int64_t* d_evict_ids, int64_t* d_evict_slots, int64_t* d_counts,
                   int64_t* d_status, kvca_stream_t stream) {
  if (!plan_args_ok(meta_bits, order, d_l2p, num_logical, d_p2l, d_slot_meta, num_slots,
                    d_search_start, d_ids, count, d_scratch_bitmap, d_counts) ||
      !d_selected || !d_move_slots || !d_final_pins || !d_final_usage || !d_allocated || !d_evict_ids ||
      !d_evict_slots)
    return KVCA_ERR_BAD_ARGUMENT;
  return status_of(kvca::launch_plan_save(
      meta_bits, order, d_l2p, num_logical, d_p2l, d_slot_meta, num_slots, d_search_start, d_ids,
      count, d_scratch_bitmap, d_selected, d_move_slots, d_final_pins, d_final_usage, d_allocated,
      d_evict_ids, d_evict_slots, d_counts, d_status, stream));
}

// One-plane paged side: slot s at base + s * row_stride.
static void one_plane(uint64_t base, int64_t rows, int64_t row_stride, const int64_t* index,
                      kvca::PagedSide* out) {
  out->planes[0] = base;
  out->index = index;
  out->num_blocks = rows;
  out->block_size = 1;
  out->block_stride = row_stride;
  out->row_stride = row_stride;
}

static bool store_ok(const kvca_device_store* store, uint64_t actual, int64_t actual_row_stride,
                     int64_t row_bytes) {
  return store && store->storage && store->present && store->scratch && actual &&
         row_bytes > 0 && actual_row_stride >= row_bytes && store->storage_row_stride >= row_bytes &&
         (store->move_flags & ~KVCA_FLAG_HOST_MEMORY) == 0;
}

int kvca_host_memory_usable(const void* p, int64_t bytes) {
  if (p == nullptr || bytes <= 0) return 0;
  const char* last = static_cast<const char*>(p) + (bytes - 1);
  for (const void* q : {p, static_cast<const void*>(last)}) {
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, q) != cudaSuccess) {
      cudaGetLastError();  // clear the sticky-free error of an unknown pointer
      return 0;
    }
    if (attr.type != cudaMemoryTypeHost || attr.devicePointer != q) return 0;
  }
  return 1;
}

// host_counts (session calls): when the call is one launch, that launch
// ends by writing the counts and seq to host_counts (*signalled = true).
static int load_device_store_impl(int meta_bits, int order, int64_t* d_l2p, int64_t num_logical,
                                  int64_t* d_p2l, void* d_slot_meta, int64_t num_slots,
                                  int64_t* d_search_start, const int64_t* d_ids, int64_t count,
                                  uint32_t* d_scratch_bitmap, const kvca_device_store* store,
                                  uint64_t d_actual, int64_t actual_row_stride, int64_t row_bytes,
                                  int64_t* d_work, void* d_work_meta, int64_t* d_result,
                                  int64_t* d_counts, int64_t* d_status, kvca_stream_t stream,
                                  int64_t* host_counts, int64_t seq, bool* signalled) {
  if (!plan_args_ok(meta_bits, order, d_l2p, num_logical, d_p2l, d_slot_meta, num_slots,
                    d_search_start, d_ids, count, d_scratch_bitmap, d_counts) ||
      !store_ok(store, d_actual, actual_row_stride, row_bytes) || !d_work || !d_work_meta ||
      !d_result)
    return KVCA_ERR_BAD_ARGUMENT;
  int vec = align_of(static_cast<uint64_t>(row_bytes));
  vec = min_align(vec, d_actual);
  vec = min_align(vec, static_cast<uint64_t>(actual_row_stride));
  vec = min_align(vec, store->storage);
  vec = min_align(vec, static_cast<uint64_t>(store->storage_row_stride));
  if (small_store_call(count, row_bytes, store->move_flags)) {
    const kvca::StoreRowArgs rows{d_actual, actual_row_stride, store->storage, store->storage_row_stride, 0,
                                  row_bytes, vec};
    *signalled = host_counts != nullptr;
    return status_of(kvca::launch_store_load_small(
        meta_bits, order, d_l2p, num_logical, d_p2l, d_slot_meta, num_slots, d_search_start, d_ids, count,
        d_scratch_bitmap, store->scratch, store->present, d_work, d_work_meta, d_result, d_counts, d_status,
        rows, stream, host_counts, seq));
  }
  int rc = status_of(kvca::launch_store_load_meta(
      meta_bits, order, d_l2p, num_logical, d_p2l, d_slot_meta, num_slots, d_search_start, d_ids,
      count, d_scratch_bitmap, store->scratch, store->present, d_work, d_work_meta, d_result,
      d_counts, d_status, stream));
  if (rc != KVCA_OK) return rc;
  const int64_t k = count;
  const int32_t flags = KVCA_FLAG_SKIP_NEGATIVE | store->move_flags;
  const int64_t* xslot = d_work + 6 * k;
  const int64_t* spill_to = d_work + 7 * k;
  const int64_t* fill_from = d_work + 8 * k;
  const int64_t* gate = d_counts + 7;
  kvca::PagedSide slots, store_out, store_in, slots_in;
  one_plane(d_actual, num_slots, actual_row_stride, xslot, &slots);
  one_plane(store->storage, num_logical, store->storage_row_stride, spill_to, &store_out);
  kvca::ExchangeArgs x{&slots, &store_out, fill_from, gate, k, row_bytes, vec, flags, d_status};
  rc = status_of(kvca::launch_exchange(x, stream));
  if (rc != KVCA_OK) return rc;
  // a miss that this call also spills is filled after every spill (gate set)
  one_plane(store->storage, num_logical, store->storage_row_stride, fill_from, &store_in);
  one_plane(d_actual, num_slots, actual_row_stride, xslot, &slots_in);
  kvca::MoveArgs fill{kvca::MoveKind::kCopyPaged, &store_in, nullptr, &slots_in, nullptr, 1, k,
                      row_bytes, vec, flags, d_status, gate};
  return status_of(kvca::launch_move(fill, stream));
}

int kvca_load_device_store(int meta_bits, int order, int64_t* d_l2p, int64_t num_logical,
                           int64_t* d_p2l, void* d_slot_meta, int64_t num_slots,
                           int64_t* d_search_start, const int64_t* d_ids, int64_t count,
                           uint32_t* d_scratch_bitmap, const kvca_device_store* store,
                           uint64_t d_actual, int64_t actual_row_stride, int64_t row_bytes,
                           int64_t* d_work, void* d_work_meta, int64_t* d_result,
                           int64_t* d_counts, int64_t* d_status, kvca_stream_t stream) {
  bool signalled = false;
  return load_device_store_impl(meta_bits, order, d_l2p, num_logical, d_p2l, d_slot_meta, num_slots,
                                d_search_start, d_ids, count, d_scratch_bitmap, store, d_actual,
                                actual_row_stride, row_bytes, d_work, d_work_meta, d_result, d_counts, d_status,
                                stream, nullptr, 0, &signalled);
}

static int save_device_store_impl(int meta_bits, int order, int64_t* d_l2p, int64_t num_logical,
                                  int64_t* d_p2l, void* d_slot_meta, int64_t num_slots,
                                  int64_t* d_search_start, const int64_t* d_ids, int64_t count,
                                  uint32_t* d_scratch_bitmap, const kvca_device_store* store,
                                  uint64_t d_actual, int64_t actual_row_stride, int64_t row_bytes,
                                  uint64_t d_block_data, int64_t* d_work, void* d_work_meta,
                                  int64_t* d_counts, int64_t* d_status, kvca_stream_t stream,
                                  int64_t* host_counts, int64_t seq, bool* signalled) {
  if (!plan_args_ok(meta_bits, order, d_l2p, num_logical, d_p2l, d_slot_meta, num_slots,
                    d_search_start, d_ids, count, d_scratch_bitmap, d_counts) ||
      !store_ok(store, d_actual, actual_row_stride, row_bytes) || !d_block_data || !d_work ||
      !d_work_meta)
    return KVCA_ERR_BAD_ARGUMENT;
  int vec = align_of(static_cast<uint64_t>(row_bytes));
  vec = min_align(vec, d_actual);
  vec = min_align(vec, static_cast<uint64_t>(actual_row_stride));
  vec = min_align(vec, store->storage);
  vec = min_align(vec, static_cast<uint64_t>(store->storage_row_stride));
  vec = min_align(vec, d_block_data);
  if (small_store_call(count, row_bytes, store->move_flags)) {
    const kvca::StoreRowArgs rows{d_actual, actual_row_stride, store->storage, store->storage_row_stride,
                                  d_block_data, row_bytes, vec};
    *signalled = host_counts != nullptr;
    return status_of(kvca::launch_store_save_small(
        meta_bits, order, d_l2p, num_logical, d_p2l, d_slot_meta, num_slots, d_search_start, d_ids, count,
        d_scratch_bitmap, store->scratch, store->present, d_work, d_work_meta, d_counts, d_status, rows,
        stream, host_counts, seq));
  }
  int rc = status_of(kvca::launch_store_save_meta(
      meta_bits, order, d_l2p, num_logical, d_p2l, d_slot_meta, num_slots, d_search_start, d_ids,
      count, d_scratch_bitmap, store->scratch, store->present, d_work, d_work_meta, d_counts,
      d_status, stream));
  if (rc != KVCA_OK) return rc;
  const int64_t k = count;
  kvca::PagedSide actual_evicted, store_evicted, actual_selected;
  one_plane(d_actual, num_slots, actual_row_stride, d_work + 3 * k, &actual_evicted);
  one_plane(store->storage, num_logical, store->storage_row_stride, d_work + 2 * k, &store_evicted);
  one_plane(d_actual, num_slots, actual_row_stride, d_work + 4 * k, &actual_selected);
  kvca::MoveArgs spill{kvca::MoveKind::kCopyPaged, &actual_evicted, nullptr, &store_evicted,
                       nullptr, 1, k, row_bytes, vec, KVCA_FLAG_SKIP_NEGATIVE | store->move_flags,
                       d_status};
  rc = status_of(kvca::launch_move(spill, stream));
  if (rc != KVCA_OK) return rc;
  kvca::ChunkSide data;
  data.base = d_block_data;
  data.rows_per_chunk = k;
  data.chunk_stride = k * row_bytes;
  data.row_stride = row_bytes;
  data.plane_stride = k * row_bytes;
  kvca::MoveArgs scatter{kvca::MoveKind::kScatter, nullptr, &data, &actual_selected, nullptr, 1,
                         k, row_bytes, vec, KVCA_FLAG_SKIP_NEGATIVE, d_status};
  return status_of(kvca::launch_move(scatter, stream));
}

int kvca_save_device_store(int meta_bits, int order, int64_t* d_l2p, int64_t num_logical,
                           int64_t* d_p2l, void* d_slot_meta, int64_t num_slots,
                           int64_t* d_search_start, const int64_t* d_ids, int64_t count,
                           uint32_t* d_scratch_bitmap, const kvca_device_store* store,
                           uint64_t d_actual, int64_t actual_row_stride, int64_t row_bytes,
                           uint64_t d_block_data, int64_t* d_work, void* d_work_meta,
                           int64_t* d_counts, int64_t* d_status, kvca_stream_t stream) {
  bool signalled = false;
  return save_device_store_impl(meta_bits, order, d_l2p, num_logical, d_p2l, d_slot_meta, num_slots,
                                d_search_start, d_ids, count, d_scratch_bitmap, store, d_actual,
                                actual_row_stride, row_bytes, d_block_data, d_work, d_work_meta, d_counts,
                                d_status, stream, nullptr, 0, &signalled);
}

// Ends a session call: when its one launch signals the host, waits for the
// sequence number in host memory (bounded; after about a second the stream's
// own synchronisation decides); otherwise copies the counts to the host and
// waits for the stream.  Either way the call returns with its work done.
static int session_finish(kvca_adapter_session* s, int rc, bool signalled) {
  if (rc != KVCA_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(s->stream);
  if (signalled) {
    volatile int64_t* done = s->counts_host + 8;
    const auto t0 = std::chrono::steady_clock::now();
    for (uint32_t spins = 0;; ++spins) {
      if (*done == s->sequence) return KVCA_OK;
      if ((spins & 4095u) == 4095u && std::chrono::steady_clock::now() - t0 > std::chrono::seconds(1)) break;
    }
    if (cudaStreamSynchronize(st) != cudaSuccess) return KVCA_ERR_CUDA;
    return *done == s->sequence ? KVCA_OK : KVCA_ERR_CUDA;
  }
  if (cudaMemcpyAsync(s->counts_host, s->counts, 8 * sizeof(int64_t), cudaMemcpyDeviceToHost, st) !=
          cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return KVCA_ERR_CUDA;
  return KVCA_OK;
}

int kvca_session_load(kvca_adapter_session* s, const int64_t* d_ids, int64_t count, int64_t* d_result) {
  if (!s || !s->counts_host || count < 0 || count > s->work_ids) return KVCA_ERR_BAD_ARGUMENT;
  bool signalled = false;
  ++s->sequence;
  const int rc = load_device_store_impl(
      s->meta_bits, s->order, s->l2p, s->num_logical, s->p2l, s->slot_meta, s->num_slots, s->search_start, d_ids,
      count, s->scratch_bitmap, &s->store, s->actual, s->actual_row_stride, s->row_bytes, s->work, s->work_meta,
      d_result, s->counts, s->status, s->stream, s->counts_host, s->sequence, &signalled);
  return session_finish(s, rc, signalled);
}

int kvca_session_save(kvca_adapter_session* s, const int64_t* d_ids, int64_t count, uint64_t d_block_data) {
  if (!s || !s->counts_host || count < 0 || count > s->work_ids) return KVCA_ERR_BAD_ARGUMENT;
  bool signalled = false;
  ++s->sequence;
  const int rc = save_device_store_impl(
      s->meta_bits, s->order, s->l2p, s->num_logical, s->p2l, s->slot_meta, s->num_slots, s->search_start, d_ids,
      count, s->scratch_bitmap, &s->store, s->actual, s->actual_row_stride, s->row_bytes, d_block_data, s->work,
      s->work_meta, s->counts, s->status, s->stream, s->counts_host, s->sequence, &signalled);
  return session_finish(s, rc, signalled);
}

int kvca_exchange(const kvca_paged_desc* slots, const kvca_paged_desc* store,
                  const int64_t* d_fill_rows, int64_t num_rows, int64_t row_bytes, int32_t flags,
                  int64_t* d_status, kvca_stream_t stream) {
  if (!common_move_args_ok(1, num_rows, row_bytes)) return KVCA_ERR_BAD_ARGUMENT;
  if (num_rows == 0) return KVCA_OK;
  if (slots == nullptr || store == nullptr || slots->index == nullptr || store->index == nullptr ||
      d_fill_rows == nullptr || slots->block_size != 1 || store->block_size != 1)
    return KVCA_ERR_BAD_ARGUMENT;
  int vec = align_of(static_cast<uint64_t>(row_bytes));
  if (!check_paged(slots, 1, row_bytes, &vec) || !check_paged(store, 1, row_bytes, &vec))
    return KVCA_ERR_BAD_ARGUMENT;
  kvca::PagedSide a, st;
  to_side(slots, 1, &a);
  to_side(store, 1, &st);
  kvca::ExchangeArgs x{&a, &st, d_fill_rows, nullptr, num_rows, row_bytes, vec, flags, d_status};
  return status_of(kvca::launch_exchange(x, stream));
}

int kvca_append_step(int meta_bits, int order, void* d_slot_meta, int64_t num_slots,
                     int64_t* d_search_start, int64_t* d_l2p, int64_t num_logical, int64_t* d_p2l,
                     const int64_t* d_need, int64_t num_need, int64_t* d_cur_block,
                     int64_t* d_cur_logical, int64_t* d_pos, int64_t num_seqs, int64_t block_size,
                     int64_t* d_next_logical, int64_t* d_victims, int64_t* d_slot_mapping,
                     uint32_t* d_scratch_bitmap, int64_t* d_status, kvca_stream_t stream) {
  if (!valid_meta_bits(meta_bits) ||
      (order != KVCA_POP_ORDER_GROUPED && order != KVCA_POP_ORDER_PREFIX) || num_slots <= 0 ||
      num_logical <= 0 || num_seqs <= 0 || block_size <= 0 || num_need < 0 ||
      num_need > num_seqs || !d_slot_meta || !d_search_start || !d_l2p || !d_p2l ||
      !d_cur_block || !d_cur_logical || !d_pos || !d_next_logical || !d_slot_mapping ||
      !d_scratch_bitmap || (num_need > 0 && (!d_need || !d_victims)))
    return KVCA_ERR_BAD_ARGUMENT;
  return status_of(kvca::launch_append_step(
      meta_bits, order, d_slot_meta, num_slots, d_search_start, d_l2p, num_logical, d_p2l, d_need,
      num_need, d_cur_block, d_cur_logical, d_pos, num_seqs, block_size, d_next_logical,
      d_scratch_bitmap, d_victims, d_slot_mapping, d_status, stream));
}

int kvca_append_steps(int meta_bits, int order, void* d_slot_meta, int64_t num_slots,
                      int64_t* d_search_start, int64_t* d_l2p, int64_t num_logical, int64_t* d_p2l,
                      const int64_t* d_need, const int64_t* d_need_offsets, int64_t num_need,
                      int64_t num_steps, int64_t* d_cur_block, int64_t* d_cur_logical,
                      int64_t* d_pos, int64_t num_seqs, int64_t block_size,
                      int64_t* d_next_logical, int64_t* d_victims, int64_t* d_slot_mapping,
                      int64_t* d_status, kvca_stream_t stream) {
  if (!valid_meta_bits(meta_bits) ||
      (order != KVCA_POP_ORDER_GROUPED && order != KVCA_POP_ORDER_PREFIX) || num_slots <= 0 ||
      num_logical <= 0 || num_seqs <= 0 || block_size <= 0 || num_need < 0 || num_steps < 0 ||
      !d_slot_meta || !d_search_start || !d_l2p || !d_p2l || !d_cur_block || !d_cur_logical ||
      !d_pos || !d_next_logical || !d_status || (num_steps > 0 && (!d_need_offsets || !d_slot_mapping)) ||
      (num_need > 0 && (!d_need || !d_victims)))
    return KVCA_ERR_BAD_ARGUMENT;
  if (num_steps == 0) return KVCA_OK;
  return status_of(kvca::launch_append_steps(
      meta_bits, order, d_slot_meta, num_slots, d_search_start, d_l2p, num_logical, d_p2l, d_need,
      d_need_offsets, num_need, num_steps, d_cur_block, d_cur_logical, d_pos, num_seqs, block_size,
      d_next_logical, d_victims, d_slot_mapping, d_status, stream));
}

int kvca_wait_selftest(const uint32_t* d_flag, uint32_t from, int64_t* d_status, kvca_stream_t stream) {
  if (!d_flag || !d_status) return KVCA_ERR_BAD_ARGUMENT;
  return status_of(kvca::launch_wait_selftest(d_flag, from, d_status, stream));
}

int kvca_gather(const kvca_paged_desc* src, const kvca_chunk_desc* dst, int64_t num_planes,
                int64_t num_rows, int64_t row_bytes, int32_t flags, int64_t* d_status,
                kvca_stream_t stream) {
  if (!common_move_args_ok(num_planes, num_rows, row_bytes)) return KVCA_ERR_BAD_ARGUMENT;
  if (num_rows == 0) return KVCA_OK;
  int vec = align_of(static_cast<uint64_t>(row_bytes));
  if (!check_paged(src, num_planes, row_bytes, &vec) || !check_chunk(dst, &vec))
    return KVCA_ERR_BAD_ARGUMENT;
  kvca::PagedSide sp;
  kvca::ChunkSide dc;
  to_side(src, num_planes, &sp);
  to_side(dst, &dc);
  kvca::MoveArgs a{kvca::MoveKind::kGather, &sp, nullptr, nullptr, &dc, num_planes, num_rows,
                   row_bytes, vec, flags, d_status};
  return status_of(kvca::launch_move(a, stream));
}

int kvca_scatter(const kvca_chunk_desc* src, const kvca_paged_desc* dst, int64_t num_planes,
                 int64_t num_rows, int64_t row_bytes, int32_t flags, int64_t* d_status,
                 kvca_stream_t stream) {
  if (!common_move_args_ok(num_planes, num_rows, row_bytes)) return KVCA_ERR_BAD_ARGUMENT;
  if (num_rows == 0) return KVCA_OK;
  int vec = align_of(static_cast<uint64_t>(row_bytes));
  if (!check_chunk(src, &vec) || !check_paged(dst, num_planes, row_bytes, &vec))
    return KVCA_ERR_BAD_ARGUMENT;
  kvca::ChunkSide sc;
  kvca::PagedSide dp;
  to_side(src, &sc);
  to_side(dst, num_planes, &dp);
  kvca::MoveArgs a{kvca::MoveKind::kScatter, nullptr, &sc, &dp, nullptr, num_planes, num_rows,
                   row_bytes, vec, flags, d_status};
  return status_of(kvca::launch_move(a, stream));
}

int kvca_scatter_gather(const kvca_chunk_desc* s_src, const kvca_paged_desc* s_dst, int64_t s_planes,
                        int64_t s_rows, int64_t s_row_bytes, const kvca_paged_desc* g_src,
                        const kvca_chunk_desc* g_dst, int64_t g_planes, int64_t g_rows,
                        int64_t g_row_bytes, int32_t s_flags, int32_t g_flags, int64_t* d_status,
                        kvca_stream_t stream) {
  if (!common_move_args_ok(s_planes, s_rows, s_row_bytes) || !common_move_args_ok(g_planes, g_rows, g_row_bytes))
    return KVCA_ERR_BAD_ARGUMENT;
  kvca::ChunkSide sc{}, gc{};
  kvca::PagedSide sp{}, gp{};
  int s_vec = align_of(static_cast<uint64_t>(s_row_bytes));
  int g_vec = align_of(static_cast<uint64_t>(g_row_bytes));
  if (s_rows > 0) {
    if (!check_chunk(s_src, &s_vec) || !check_paged(s_dst, s_planes, s_row_bytes, &s_vec))
      return KVCA_ERR_BAD_ARGUMENT;
    to_side(s_src, &sc);
    to_side(s_dst, s_planes, &sp);
  }
  if (g_rows > 0) {
    if (!check_paged(g_src, g_planes, g_row_bytes, &g_vec) || !check_chunk(g_dst, &g_vec))
      return KVCA_ERR_BAD_ARGUMENT;
    to_side(g_src, g_planes, &gp);
    to_side(g_dst, &gc);
  }
  if (s_rows == 0 && g_rows == 0) return KVCA_OK;
  kvca::MoveArgs s{kvca::MoveKind::kScatter, nullptr, &sc, &sp, nullptr, s_planes, s_rows,
                   s_row_bytes, s_vec, s_flags, d_status};
  kvca::MoveArgs g{kvca::MoveKind::kGather, &gp, nullptr, nullptr, &gc, g_planes, g_rows,
                   g_row_bytes, g_vec, g_flags, d_status};
  return status_of(kvca::launch_scatter_gather(s, g, stream));
}

int64_t kvca_move_cycle_scratch_bytes(int64_t num_blocks) {
  if (num_blocks < 0) return -1;
  return static_cast<int64_t>(kvca::move_cycle_scratch_bytes(num_blocks));
}

int kvca_move_cycle(const kvca_chunk_desc* tokens, const kvca_paged_desc* token_dst, int64_t token_row_bytes,
                    const kvca_paged_desc* block_src, int64_t num_victims, const kvca_chunk_desc* spill,
                    int64_t block_row_bytes, int64_t num_planes, const int64_t* d_offsets, int64_t num_steps,
                    int64_t num_seqs, int64_t spill_rows, int32_t flags, void* d_scratch, int64_t* d_status,
                    kvca_stream_t stream) {
  if (!common_move_args_ok(num_planes, num_seqs, token_row_bytes) || block_row_bytes < 1 || num_seqs < 1 ||
      num_steps < 1 || num_steps > kvca::kMoveCycleMaxSteps || spill_rows < 0 || num_victims < 0 ||
      d_offsets == nullptr || d_scratch == nullptr || d_status == nullptr)
    return KVCA_ERR_BAD_ARGUMENT;
  int vec = 16;
  vec = min_align(vec, static_cast<uint64_t>(token_row_bytes));
  vec = min_align(vec, static_cast<uint64_t>(block_row_bytes));
  if (!check_chunk(tokens, &vec) || !check_chunk(spill, &vec) ||
      !check_paged(token_dst, num_planes, token_row_bytes, &vec) ||
      !check_paged(block_src, num_planes, block_row_bytes, &vec) || vec != 16)
    return KVCA_ERR_BAD_ARGUMENT;
  if (token_dst->index == nullptr || (num_victims > 0 && block_src->index == nullptr) ||
      block_src->block_size != 1 || token_dst->num_blocks != block_src->num_blocks ||
      token_dst->block_stride != block_src->block_stride || block_row_bytes > block_src->block_stride ||
      (token_dst->block_size - 1) * token_dst->row_stride + token_row_bytes > token_dst->block_stride)
    return KVCA_ERR_BAD_ARGUMENT;
  for (int64_t p = 0; p < num_planes; ++p)
    if (token_dst->plane_ptrs[p] != block_src->plane_ptrs[p]) return KVCA_ERR_BAD_ARGUMENT;
  // item numbers and per-item vector counts stay below 2^31
  const int64_t s_group = kvca::move_cycle_group(token_row_bytes, num_planes);
  const int64_t g_group = kvca::move_cycle_group(block_row_bytes, num_planes);
  const int64_t items = num_steps * num_seqs * ((num_planes + s_group - 1) / s_group) *
                            kvca::move_cycle_segments(token_row_bytes) +
                        spill_rows * ((num_planes + g_group - 1) / g_group) * kvca::move_cycle_segments(block_row_bytes);
  if (num_seqs > (int64_t{1} << 26) || spill_rows > (int64_t{1} << 26) || num_victims > (int64_t{1} << 40) ||
      items >= (int64_t{1} << 31) ||
      s_group * (token_row_bytes / 16) >= (int64_t{1} << 31) || g_group * (block_row_bytes / 16) >= (int64_t{1} << 31))
    return KVCA_ERR_SIZE_LIMIT;
  kvca::PagedSide cache;
  kvca::ChunkSide src, dst;
  to_side(token_dst, num_planes, &cache);
  to_side(tokens, &src);
  to_side(spill, &dst);
  kvca::CycleArgs a{&cache, block_src->index, num_victims, d_offsets, &src, &dst, num_planes, num_steps,
                    num_seqs, spill_rows, token_row_bytes, block_row_bytes, flags,
                    static_cast<unsigned char*>(d_scratch), d_status};
  return status_of(kvca::launch_move_cycle(a, stream));
}

int kvca_copy_paged(const kvca_paged_desc* src, const kvca_paged_desc* dst, int64_t num_planes,
                    int64_t num_rows, int64_t row_bytes, int32_t flags, int64_t* d_status,
                    kvca_stream_t stream) {
  if (!common_move_args_ok(num_planes, num_rows, row_bytes)) return KVCA_ERR_BAD_ARGUMENT;
  if (num_rows == 0) return KVCA_OK;
  int vec = align_of(static_cast<uint64_t>(row_bytes));
  if (!check_paged(src, num_planes, row_bytes, &vec) ||
      !check_paged(dst, num_planes, row_bytes, &vec))
    return KVCA_ERR_BAD_ARGUMENT;
  kvca::PagedSide sp;
  kvca::PagedSide dp;
  to_side(src, num_planes, &sp);
  to_side(dst, num_planes, &dp);
  kvca::MoveArgs a{kvca::MoveKind::kCopyPaged, &sp, nullptr, &dp, nullptr, num_planes, num_rows,
                   row_bytes, vec, flags, d_status};
  return status_of(kvca::launch_move(a, stream));
}

}  // extern "C"
