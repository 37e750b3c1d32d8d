// sm_100a kernels for the paged-KV adapter hot path.
//
//  * Slot metadata ops over a packed slot_meta array (pin count in the low
//    half of each word, usage count in the high half; adapter.py:17-36,
//    adapter.py:1419-1432 of the reference).
//  * The clock sweep (pop_reusable_slots) as one CTA that scans the table in
//    16-byte vectors, ranks candidates with warp ballots / block scans and
//    stops at the first tile that completes the request when no aging is
//    needed.
//  * A device-resident clock stream that runs pop, refill and usage bumps
//    for many steps inside one launch.
//  * The row mover: whole blocks or single token rows between paged planes
//    and contiguous chunks, all planes (layers x K/V) of a call in one launch:
//    TMA bulk copies staged through shared memory for 16-byte aligned rows of
//    1 KiB or more, 16-byte vectorised coalesced loads/stores otherwise.
//
// Device-side errors never trap: they are written to a caller-owned status
// pair (code, value) with first-error-wins semantics, and the offending row
// or request is skipped.

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <atomic>
#include <utility>

#include "kvca_launch.h"

namespace kvca {
namespace {

// ---------------------------------------------------------------------------
// Status reporting
// ---------------------------------------------------------------------------

__device__ __forceinline__ void report(int64_t* status, int64_t code, int64_t value) {
  if (status == nullptr) return;
  const unsigned long long prev = atomicCAS(reinterpret_cast<unsigned long long*>(status), 0ull,
                                            static_cast<unsigned long long>(code));
  if (prev == 0ull) status[1] = value;
}

// ---------------------------------------------------------------------------
// Packed slot metadata: pin count in the low half of the word, usage count in
// the high half (adapter.py:1419-1432).
// ---------------------------------------------------------------------------

template <typename MetaT>
struct Meta {
  static constexpr int kFieldBits = static_cast<int>(sizeof(MetaT)) * 4;
  static constexpr unsigned kFieldMask = (1u << kFieldBits) - 1u;
  static constexpr int kUsageMax = static_cast<int>(kFieldMask);
  static constexpr int kSlotsPerVec = 16 / static_cast<int>(sizeof(MetaT));

  __device__ __forceinline__ static unsigned pin(unsigned w) { return w & kFieldMask; }
  __device__ __forceinline__ static unsigned usage(unsigned w) {
    return (w >> kFieldBits) & kFieldMask;
  }
  // Masks both fields exactly like _pack_slot_meta: pins above the field
  // maximum and negative pins wrap.
  __device__ __forceinline__ static MetaT pack(int64_t pin_count, int64_t usage_count) {
    const uint64_t p = static_cast<uint64_t>(pin_count) & kFieldMask;
    const uint64_t u = static_cast<uint64_t>(usage_count) & kFieldMask;
    return static_cast<MetaT>(p | (u << kFieldBits));
  }
  __device__ __forceinline__ static unsigned sat_inc(unsigned usage_count) {
    return usage_count + 1u > kFieldMask ? kFieldMask : usage_count + 1u;
  }
};

// ---------------------------------------------------------------------------
// Block-wide exclusive scan (blockDim.x a multiple of 32, at most 1024).
// `sm` holds 33 ints.  Contains three __syncthreads.
// ---------------------------------------------------------------------------

__device__ __forceinline__ int block_excl_scan(int x, int* total, int* sm) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  int incl = x;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  if (lane == 31) sm[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nwarps = static_cast<int>(blockDim.x >> 5);
    const int w = lane < nwarps ? sm[lane] : 0;
    int wi = w;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wi, d);
      if (lane >= d) wi += y;
    }
    if (lane < nwarps) sm[lane] = wi - w;
    if (lane == 31) sm[32] = wi;
  }
  __syncthreads();
  const int result = sm[warp] + incl - x;
  *total = sm[32];
  __syncthreads();
  return result;
}

// ---------------------------------------------------------------------------
// Metadata vector access: 16 bytes per thread when the table is 16-byte
// aligned, element-wise at the ragged tail.
// ---------------------------------------------------------------------------

template <typename MetaT>
union MetaVec {
  uint4 raw;
  MetaT s[Meta<MetaT>::kSlotsPerVec];
};

template <typename MetaT>
__device__ __forceinline__ void load_meta_vec(const MetaT* meta, int64_t num_slots, int64_t v,
                                              bool aligned, MetaVec<MetaT>& out) {
  constexpr int kSpv = Meta<MetaT>::kSlotsPerVec;
  const int64_t first = v * kSpv;
  // L2 loads: the batched stream's CTAs read words other CTAs wrote
  if (aligned && first + kSpv <= num_slots) {
    out.raw = __ldcg(reinterpret_cast<const uint4*>(meta + first));
  } else {
#pragma unroll
    for (int j = 0; j < kSpv; ++j) out.s[j] = first + j < num_slots ? __ldcg(meta + first + j) : MetaT(0);
  }
}

template <typename MetaT>
__device__ __forceinline__ void store_meta_vec(MetaT* meta, int64_t num_slots, int64_t v,
                                               bool aligned, const MetaVec<MetaT>& in) {
  constexpr int kSpv = Meta<MetaT>::kSlotsPerVec;
  const int64_t first = v * kSpv;
  if (aligned && first + kSpv <= num_slots) {
    *reinterpret_cast<uint4*>(meta + first) = in.raw;
  } else {
#pragma unroll
    for (int j = 0; j < kSpv; ++j)
      if (first + j < num_slots) meta[first + j] = in.s[j];
  }
}

// Vector v of a shared-memory copy of the table (padded to whole vectors).
template <typename MetaT>
__device__ __forceinline__ void load_mirror_vec(const MetaT* mirror, int64_t v, MetaVec<MetaT>& out) {
  out.raw = *reinterpret_cast<const uint4*>(mirror + v * Meta<MetaT>::kSlotsPerVec);
}

template <typename MetaT>
__device__ __forceinline__ void store_mirror_vec(MetaT* mirror, int64_t v, const MetaVec<MetaT>& in) {
  *reinterpret_cast<uint4*>(mirror + v * Meta<MetaT>::kSlotsPerVec) = in.raw;
}

// Blocked-slot bits for the kSlotsPerVec slots starting at `first` (a
// multiple of kSlotsPerVec, so they share one 32-bit bitmap word).  The
// bitmap is written with atomics earlier in the same CTA; read it through L2.
template <typename MetaT>
__device__ __forceinline__ unsigned blocked_bits(const uint32_t* bitmap, int64_t first) {
  constexpr int kSpv = Meta<MetaT>::kSlotsPerVec;
  if (bitmap == nullptr) return 0u;
  const unsigned word = __ldcg(bitmap + (first >> 5));
  return (word >> (first & 31)) & ((1u << kSpv) - 1u);
}

// ---------------------------------------------------------------------------
// Clock sweep
// ---------------------------------------------------------------------------

template <typename MetaT>
struct PopShared {
  int scan[33];
  int hist[Meta<MetaT>::kUsageMax + 1];
  long long cls_base[Meta<MetaT>::kUsageMax + 1];
  long long run[Meta<MetaT>::kUsageMax + 1];
  long long start;
  long long last_slot;
  long long need;
  int threshold;
};

// One CTA selects `count` victims (see kvca_pop_reusable_slots for the
// semantics).  Returns KVCA_OK or KVCA_ERR_INSUFFICIENT_CAPACITY, uniformly
// across the CTA.  On insufficient capacity nothing but `out` is written.
//
// Scan order from start s is split into two segments of the slot space,
// [s, N) then [0, s), each walked in aligned vectors so that loads stay
// 16-byte wide.  The vector holding s is visited by both segments, each time
// handling only its own slots.
//
// Pass 1 ranks available usage-0 slots in scan order and stops at the tile
// that completes `count`: then T = 0 and nothing ages.  Otherwise a full
// histogram fixes T, and pass 2 walks every tile once more, ranking classes
// 1..T (grouped order) or all usage <= T (prefix order) and writing the aged
// usage of every slot.
//
// start_set: the caller already put the scan start into sh.start and
// sh.last_slot (pop_start) and passed a barrier since, so the read of
// *search_start can overlap the caller's own loads.  out_sh (optional, in
// shared memory): victims 0..out_sh_cap-1 are also written there, so the
// caller reads them without a global round trip.  mirror (optional, in
// shared memory): a copy of the whole table padded to whole vectors, equal
// to it on entry; the scans read it instead of global memory and the aging
// writes go to both.
template <typename MetaT>
__device__ __forceinline__ void pop_start(const int64_t* search_start, int64_t n, PopShared<MetaT>& sh) {
  long long s = static_cast<long long>(*search_start % n);
  if (s < 0) s += n;
  sh.start = s;
  sh.last_slot = s;
}

template <typename MetaT>
__device__ int pop_cta(MetaT* meta, int64_t num_slots, int64_t* search_start,
                       const uint32_t* bitmap, int64_t count, int64_t* out, int order,
                       bool aligned, PopShared<MetaT>& sh, bool start_set = false,
                       int64_t* out_sh = nullptr, int64_t out_sh_cap = 0, MetaT* mirror = nullptr) {
  using M = Meta<MetaT>;
  constexpr int kSpv = M::kSlotsPerVec;
  const int64_t n = num_slots;

  if (!start_set) {
    if (threadIdx.x == 0) pop_start(search_start, n, sh);
    __syncthreads();
  }
  const int64_t s = sh.start;

  // ---- Pass 1: usage-0 candidates with early exit -------------------------
  int64_t found = 0;
  bool done = false;
  for (int seg = 0; seg < 2 && !done; ++seg) {
    const int64_t lo = seg == 0 ? s : 0;
    const int64_t hi = seg == 0 ? n : s;
    if (lo >= hi) continue;
    const int64_t v_begin = lo / kSpv;
    const int64_t v_end = (hi + kSpv - 1) / kSpv;
    for (int64_t tile = v_begin; tile < v_end; tile += blockDim.x) {
      const int64_t v = tile + threadIdx.x;
      unsigned mask = 0u;
      if (v < v_end) {
        MetaVec<MetaT> m;
        if (mirror != nullptr)
          load_mirror_vec(mirror, v, m);
        else
          load_meta_vec(meta, n, v, aligned, m);
        const unsigned blk = blocked_bits<MetaT>(bitmap, v * kSpv);
#pragma unroll
        for (int j = 0; j < kSpv; ++j) {
          const int64_t slot = v * kSpv + j;
          const unsigned w = m.s[j];
          const bool hit = slot >= lo && slot < hi && M::pin(w) == 0u && ((blk >> j) & 1u) == 0u &&
                           M::usage(w) == 0u;
          mask |= (hit ? 1u : 0u) << j;
        }
      }
      int total;
      const int base = block_excl_scan(__popc(mask), &total, sh.scan);
      int64_t rank = found + base;
      while (mask != 0u) {
        const int j = __ffs(mask) - 1;
        mask &= mask - 1u;
        if (rank < count) {
          out[rank] = v * kSpv + j;
          if (rank < out_sh_cap) out_sh[rank] = v * kSpv + j;
          if (rank == count - 1) sh.last_slot = v * kSpv + j;
        }
        ++rank;
      }
      found += total;
      if (found >= count) {
        done = true;
        break;
      }
    }
  }
  __syncthreads();
  if (done) {
    if (threadIdx.x == 0) *search_start = (sh.last_slot + 1) % n;
    __syncthreads();
    return KVCA_OK;
  }

  // ---- Histogram of available slots by usage ------------------------------
  for (int i = threadIdx.x; i <= M::kUsageMax; i += blockDim.x) sh.hist[i] = 0;
  __syncthreads();
  {
    const int64_t nvec = (n + kSpv - 1) / kSpv;
    const int lane = threadIdx.x & 31;
    for (int64_t tile = 0; tile < nvec; tile += blockDim.x) {
      const int64_t v = tile + threadIdx.x;
      MetaVec<MetaT> m;
      unsigned blk = 0u;
      if (v < nvec) {
        if (mirror != nullptr)
          load_mirror_vec(mirror, v, m);
        else
          load_meta_vec(meta, n, v, aligned, m);
        blk = blocked_bits<MetaT>(bitmap, v * kSpv);
      }
#pragma unroll
      for (int j = 0; j < kSpv; ++j) {
        int key = -1;
        if (v < nvec && v * kSpv + j < n) {
          const unsigned w = m.s[j];
          if (M::pin(w) == 0u && ((blk >> j) & 1u) == 0u) key = static_cast<int>(M::usage(w));
        }
        const unsigned peers = __match_any_sync(0xffffffffu, key);
        if (key >= 0 && lane == __ffs(peers) - 1) atomicAdd(&sh.hist[key], __popc(peers));
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    long long cum = 0;
    int threshold = -1;
    for (int t = 0; t <= M::kUsageMax; ++t) {
      sh.cls_base[t] = cum;
      sh.run[t] = 0;
      cum += sh.hist[t];
      if (cum >= count) {
        threshold = t;
        break;
      }
    }
    sh.threshold = threshold;
    if (threshold >= 0) sh.need = count - sh.cls_base[threshold];
  }
  __syncthreads();
  const int threshold = sh.threshold;
  if (threshold < 0) return KVCA_ERR_INSUFFICIENT_CAPACITY;

  // ---- Pass 2: ranked selection of classes <= T and aging -----------------
  const int64_t need = sh.need;
  int64_t run_prefix = 0;
  for (int seg = 0; seg < 2; ++seg) {
    const int64_t lo = seg == 0 ? s : 0;
    const int64_t hi = seg == 0 ? n : s;
    if (lo >= hi) continue;
    const int64_t v_begin = lo / kSpv;
    const int64_t v_end = (hi + kSpv - 1) / kSpv;
    for (int64_t tile = v_begin; tile < v_end; tile += blockDim.x) {
      const int64_t v = tile + threadIdx.x;
      const bool active = v < v_end;
      MetaVec<MetaT> m;
      unsigned avail_mask = 0u;  // in segment, unpinned, not blocked
      if (active) {
        if (mirror != nullptr)
          load_mirror_vec(mirror, v, m);
        else
          load_meta_vec(meta, n, v, aligned, m);
        const unsigned blk = blocked_bits<MetaT>(bitmap, v * kSpv);
        MetaVec<MetaT> aged;
#pragma unroll
        for (int j = 0; j < kSpv; ++j) {
          const int64_t slot = v * kSpv + j;
          const unsigned w = m.s[j];
          const bool in_seg = slot >= lo && slot < hi;
          if (in_seg && M::pin(w) == 0u && ((blk >> j) & 1u) == 0u) avail_mask |= 1u << j;
          const unsigned u = M::usage(w);
          const unsigned u_aged = u > static_cast<unsigned>(threshold) ? u - threshold : 0u;
          aged.s[j] = in_seg ? M::pack(M::pin(w), u_aged) : m.s[j];
        }
        store_meta_vec(meta, n, v, aligned, aged);
        if (mirror != nullptr) store_mirror_vec(mirror, v, aged);
      }
      if (order == KVCA_POP_ORDER_GROUPED) {
        for (int c = 1; c <= threshold; ++c) {
          if (sh.hist[c] == 0) continue;
          unsigned mask = 0u;
          if (active) {
#pragma unroll
            for (int j = 0; j < kSpv; ++j)
              if (((avail_mask >> j) & 1u) && M::usage(m.s[j]) == static_cast<unsigned>(c))
                mask |= 1u << j;
          }
          const long long run_c = sh.run[c];
          int total;
          const int base = block_excl_scan(__popc(mask), &total, sh.scan);
          const int64_t limit = c < threshold ? static_cast<int64_t>(sh.hist[c]) : need;
          int64_t rank = run_c + base;
          while (mask != 0u) {
            const int j = __ffs(mask) - 1;
            mask &= mask - 1u;
            if (rank < limit) {
              out[sh.cls_base[c] + rank] = v * kSpv + j;
              if (sh.cls_base[c] + rank < out_sh_cap) out_sh[sh.cls_base[c] + rank] = v * kSpv + j;
              if (c == threshold && rank == need - 1) sh.last_slot = v * kSpv + j;
            }
            ++rank;
          }
          if (threadIdx.x == 0) sh.run[c] = run_c + total;
        }
      } else {
        unsigned mask = 0u;
        if (active) {
#pragma unroll
          for (int j = 0; j < kSpv; ++j)
            if (((avail_mask >> j) & 1u) && M::usage(m.s[j]) <= static_cast<unsigned>(threshold))
              mask |= 1u << j;
        }
        int total;
        const int base = block_excl_scan(__popc(mask), &total, sh.scan);
        int64_t rank = run_prefix + base;
        while (mask != 0u) {
          const int j = __ffs(mask) - 1;
          mask &= mask - 1u;
          if (rank < count) {
            out[rank] = v * kSpv + j;
            if (rank < out_sh_cap) out_sh[rank] = v * kSpv + j;
            if (rank == count - 1) sh.last_slot = v * kSpv + j;
          }
          ++rank;
        }
        run_prefix += total;
      }
      __syncthreads();
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *search_start = (sh.last_slot + 1) % n;
  __syncthreads();
  return KVCA_OK;
}

template <typename MetaT>
__global__ void __launch_bounds__(1024)
    pop_kernel(MetaT* meta, int64_t num_slots, int64_t* search_start, const int64_t* blocked,
               int64_t num_blocked, int64_t count, int64_t* out, uint32_t* bitmap, int order,
               bool aligned, int64_t* status) {
  __shared__ PopShared<MetaT> sh;
  __shared__ int bad_blocked;
  if (threadIdx.x == 0) bad_blocked = 0;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < num_blocked; i += blockDim.x) {
    const int64_t b = blocked[i];
    if (b < 0 || b >= num_slots) {
      bad_blocked = 1;
      report(status, KVCA_ERR_BAD_INDEX, b);
    } else {
      atomicOr(bitmap + (b >> 5), 1u << (b & 31));
    }
  }
  __syncthreads();
  if (bad_blocked == 0) {
    const int rc = pop_cta<MetaT>(meta, num_slots, search_start, bitmap, count, out, order,
                                  aligned, sh);
    if (rc != KVCA_OK && threadIdx.x == 0) report(status, rc, count);
  }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < num_blocked; i += blockDim.x) {
    const int64_t b = blocked[i];
    if (b >= 0 && b < num_slots) atomicAnd(bitmap + (b >> 5), ~(1u << (b & 31)));
  }
}

constexpr int kStreamMaxReaccessPerThread = 8;

// One step of the clock stream, run by the whole CTA: pop `alloc_per_step`
// victims, refill them, bump the step's re-accessed slots.  Returns KVCA_OK
// or the pop's error (uniform).
template <typename MetaT>
__device__ int stream_step(MetaT* meta, int64_t num_slots, int64_t* search_start, int64_t step,
                           int64_t alloc_per_step, const int64_t* reaccess,
                           int64_t reaccess_per_step, int64_t* victims, int order, bool aligned,
                           int64_t* status, PopShared<MetaT>& sh) {
  using M = Meta<MetaT>;
  int64_t* out = victims + step * alloc_per_step;
  const int rc = pop_cta<MetaT>(meta, num_slots, search_start, nullptr, alloc_per_step, out, order,
                                aligned, sh);
  if (rc != KVCA_OK) return rc;
  // Victims are refilled: pin kept (it is 0), usage 1 (adapter.py:233-242
  // gives new saves usage 1; commit at adapter.py:651).
  for (int64_t i = threadIdx.x; i < alloc_per_step; i += blockDim.x) {
    const int64_t v = out[i];
    meta[v] = M::pack(M::pin(__ldcg(meta + v)), 1);
  }
  __syncthreads();
  // Usage bump of re-accessed slots: every value is read before any write,
  // so duplicates in one batch bump once, as index_put_ does.
  const int64_t* ids = reaccess + step * reaccess_per_step;
  int64_t slot_ids[kStreamMaxReaccessPerThread];
  MetaT values[kStreamMaxReaccessPerThread];
#pragma unroll
  for (int u = 0; u < kStreamMaxReaccessPerThread; ++u) {
    const int64_t i = threadIdx.x + static_cast<int64_t>(u) * blockDim.x;
    slot_ids[u] = -1;
    values[u] = MetaT(0);
    if (i < reaccess_per_step) {
      const int64_t id = ids[i];
      if (id < 0 || id >= num_slots) {
        report(status, KVCA_ERR_BAD_INDEX, id);
      } else {
        const unsigned w = __ldcg(meta + id);
        values[u] = M::pack(M::pin(w), M::sat_inc(M::usage(w)));
        slot_ids[u] = id;
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int u = 0; u < kStreamMaxReaccessPerThread; ++u)
    if (slot_ids[u] >= 0) meta[slot_ids[u]] = values[u];
  __syncthreads();
  return KVCA_OK;
}

template <typename MetaT>
__global__ void __launch_bounds__(1024)
    clock_stream_kernel(MetaT* meta, int64_t num_slots, int64_t* search_start, int64_t num_steps,
                        int64_t alloc_per_step, const int64_t* reaccess,
                        int64_t reaccess_per_step, int64_t* victims, int64_t* steps_done,
                        int order, bool aligned, int64_t* status) {
  __shared__ PopShared<MetaT> sh;
  int64_t step = 0;
  for (; step < num_steps; ++step) {
    const int rc = stream_step<MetaT>(meta, num_slots, search_start, step, alloc_per_step, reaccess,
                                      reaccess_per_step, victims, order, aligned, status, sh);
    if (rc != KVCA_OK) {
      if (threadIdx.x == 0) report(status, rc, step);
      break;
    }
  }
  if (threadIdx.x == 0) *steps_done = step;
}

// ---------------------------------------------------------------------------
// Clock stream, batched over runs of steps that need no aging
// ---------------------------------------------------------------------------
//
// While every pop finds `alloc_per_step` available usage-0 slots (T = 0) no
// usage ever decreases: refills set 1, bumps add 1.  So from a state S at
// step s0 the victims of the following steps are the available usage-0
// slots of S in scan order from search_start (the candidates), taken k per
// step, except that a candidate whose first re-access comes at a step before
// the one that would take it has usage 1 by then and is passed over.  An
// "epoch" computes all of that at once, with the whole CTA:
//   1. compact the candidates (one pass over slot_meta);
//   2. first re-access step of every slot re-accessed in the window of steps
//      the candidates can cover (atomicMax on an encoded step; the thread
//      that sets a slot first lists it, so touched slots are listed once);
//   3. candidates whose first re-access can come before the step that takes
//      them ("pending") are listed in order; one warp resolves only those,
//      32 at a time with a ballot fixed
//      point: pending candidate j is taken unless its first re-access step is
//      below s0 + (taken before j) / k, where taken before j = (candidates
//      before j that are not pending) + (pending ones taken before it);
//      every other candidate is taken while that count stays below the
//      request, so block-wide scans place all victims at once;
//   4. fold the epoch's refills and bumps into each touched slot:
//      usage = min(base + distinct bumping steps, max), base = 1 for a victim
//      (only bumps at or after its step count) and the old usage otherwise.
// The first step that cannot take k candidates needs aging (T > 0): it runs
// as one exact step (stream_step), then the next epoch starts.  After short
// epochs the kernel runs a stretch of exact steps instead.  Results equal the
// step-by-step stream bit for bit.

constexpr int kStreamThreads = 512;   // threads per CTA of the batched stream
constexpr int kStreamMaxCtas = 1024;  // CTAs of its cooperative grid, at most
constexpr int64_t kEpochMinSteps = 8;
constexpr int64_t kExactStepsAfterShortEpoch = 64;
constexpr int kCandPerThread = 16;  // candidates per thread per block-scan tile
constexpr int kHashDedupMin = 16;    // re-accesses per step deduplicated in a shared-memory set
constexpr int kHashDedupMax = 4096;  // (the set, 2 x m rounded up to a power of two, fits the pending tile)

constexpr int kPendingTile = 4096;  // pending candidates staged per round of the resolution
static_assert(kPendingTile % kStreamThreads == 0, "pending tile split evenly over the CTA");

template <typename MetaT>
struct EpochShared {
  PopShared<MetaT> pop;
  long long tile[kPendingTile];  // pending candidates staged for the one-warp pass
  int scan[33];
};

// Scratch of kvca_clock_stream_batched, carved from one buffer (byte
// offsets for num_slots = n): pending int64[n] at 0, cand int32[n] at 8n,
// cand_bump int32[n] at 12n, touched int32[n] at 16n, then the three arrays
// that are zero on entry and left zero on exit: first_bump, victim_step,
// bump_count (int32[n] each, from 20n to 32n).
struct EpochScratch {
  int64_t* pending;
  int32_t* cand;
  int32_t* cand_bump;
  int32_t* touched;
  int32_t* first_bump;
  int32_t* victim_step;
  int32_t* bump_count;
};

__device__ __forceinline__ bool slot_ok(int64_t x, int64_t n) { return x >= 0 && x < n; }

// The epoch runs on a cooperative grid (one launch, all CTAs resident): the
// passes over slots, candidates and re-access events are spread over every
// CTA, ordered compactions take a per-CTA count, a grid barrier and the
// prefix of the counts, and the one-warp resolution of the pending
// candidates and the exact aging steps run on CTA 0 while the others wait.
// With one CTA the barriers are block barriers.  StreamGrid lives in the
// scratch buffer after the per-slot arrays and is cleared before each launch.
struct StreamGrid {
  unsigned int bar_count;  // arrivals at grid barriers since the launch began
  unsigned int unused0;
  int failed;
  int nu;        // distinct slots re-accessed in the window
  int tp_total;  // pending candidates taken
  int rc;        // status of the last exact step
  long long last_victim;
  long long cnt[kStreamMaxCtas];  // per-CTA counts of the current compaction
};
static_assert(sizeof(StreamGrid) <= kClockStreamGridBytes, "grid words exceed their scratch");

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr uint32_t kGridSpinLimit = 1u << 22;  // polls of a wait: a few seconds at most

// Waits until *word differs from `from` (or *abort != 0); gives up after
// about kGridSpinLimit naps.  Returns true when the word changed.
__device__ bool bounded_wait_change(const unsigned* word, unsigned from, const int* abort) {
  uint32_t spins = 0;
  while (ld_acquire_u32(word) == from) {
    if (++spins > kGridSpinLimit || (abort != nullptr && *reinterpret_cast<const volatile int*>(abort) != 0))
      return false;
    __nanosleep(64);
  }
  return true;
}

// Grid-wide barrier with a bounded wait (counter and failure flag given by
// address; grid_barrier takes the stream's).  Every CTA's writes before the
// barrier are visible to every CTA after it: the CTA's threads meet at a
// block barrier, then one thread arrives with a release add on a counter
// that only grows (barrier j of the launch completes when it reaches
// (j + 1) x gridDim.x) and waits with acquire loads until it does; no CTA
// resets anything, so the last arrival releases the others with its one
// atomic.  The counter starts at zero with each launch.  A CTA that waits
// too long (or sees another CTA give up) marks the grid failed, reports
// KVCA_ERR_DEVICE_TIMEOUT and returns false; callers then return.
__device__ bool grid_barrier_words(unsigned* bar_count, int* failed, int64_t* status) {
  __shared__ int ok_s;
  __syncthreads();
  if (gridDim.x == 1) return true;
  if (threadIdx.x == 0) {
    const unsigned B = gridDim.x;
    unsigned old;
    asm volatile("atom.add.release.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(bar_count) : "memory");
    const unsigned target = (old / B + 1u) * B;
    int ok = 1;
    uint32_t spins = 0;
    while (static_cast<int>(ld_acquire_u32(bar_count) - target) < 0) {
      if (++spins > kGridSpinLimit || *reinterpret_cast<const volatile int*>(failed) != 0) {
        ok = 0;
        break;
      }
    }
    if (!ok) {
      atomicExch(failed, 1);
      report(status, KVCA_ERR_DEVICE_TIMEOUT, blockIdx.x);
    }
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

__device__ bool grid_barrier(StreamGrid* g, int64_t* status) {
  return grid_barrier_words(&g->bar_count, &g->failed, status);
}

// Sum over the CTAs' counts: (sum of the CTAs before this one, total).
__device__ void grid_prefix(const StreamGrid* g, int64_t* before, int64_t* total, int* scan) {
  long long b = 0, t = 0;
  for (int i = threadIdx.x; i < static_cast<int>(gridDim.x); i += blockDim.x) {
    const long long c = __ldcg(g->cnt + i);
    t += c;
    if (i < static_cast<int>(blockIdx.x)) b += c;
  }
  int tot;
  block_excl_scan(static_cast<int>(b), &tot, scan);
  *before = tot;
  block_excl_scan(static_cast<int>(t), &tot, scan);
  *total = tot;
}

template <typename MetaT>
__device__ __forceinline__ unsigned candidate_mask(const MetaT* meta, int64_t n, int64_t p0,
                                                   int64_t v0b, int64_t V0, int64_t vv,
                                                   bool aligned, int64_t* v_out) {
  using M = Meta<MetaT>;
  constexpr int kSpv = M::kSlotsPerVec;
  int64_t v, lo, hi;
  if (vv < V0) {
    v = v0b + vv;
    lo = p0;
    hi = n;
  } else {
    v = vv - V0;
    lo = 0;
    hi = p0;
  }
  *v_out = v;
  MetaVec<MetaT> mv;
  load_meta_vec(meta, n, v, aligned, mv);
  unsigned mask = 0u;
#pragma unroll
  for (int j = 0; j < kSpv; ++j) {
    const int64_t slot = v * kSpv + j;
    const unsigned wd = mv.s[j];
    if (slot >= lo && slot < hi && M::pin(wd) == 0u && M::usage(wd) == 0u) mask |= 1u << j;
  }
  return mask;
}

// One epoch from step s0 (see above); returns the first step it did not
// complete, or s0 with *ok = false when a grid barrier gave up.
template <typename MetaT>
__device__ int64_t stream_epoch(MetaT* meta, int64_t n, int64_t* search_start, int64_t s0,
                                int64_t steps, int64_t k, const int64_t* reaccess, int64_t m,
                                int64_t* victims, const EpochScratch& w, StreamGrid* g,
                                bool aligned, int64_t* status, EpochShared<MetaT>& sh, bool* ok) {
  using M = Meta<MetaT>;
  constexpr int kSpv = M::kSlotsPerVec;
  constexpr int C = kCandPerThread;
  const int64_t B = gridDim.x;
  const int64_t b = blockIdx.x;
  const int64_t T = blockDim.x;
  const int64_t gt = b * T + threadIdx.x;
  const int64_t G = B * T;
#define KVCA_GRID_SYNC()               \
  if (!grid_barrier(g, status)) {      \
    *ok = false;                       \
    return s0;                         \
  }
  int64_t p0 = __ldcg(reinterpret_cast<const long long*>(search_start)) % n;
  if (p0 < 0) p0 += n;
  if (b == 0 && threadIdx.x == 0) g->nu = 0;

  // 1. candidates: available usage-0 slots in scan order from p0; CTA b
  //    takes a contiguous range of the order's vectors (segment [p0, n),
  //    then [0, p0))
  const int64_t v0b = p0 / kSpv;
  const int64_t V0 = (n + kSpv - 1) / kSpv - v0b;
  const int64_t V = V0 + (p0 + kSpv - 1) / kSpv;
  const int64_t cb = V * b / B;
  const int64_t ce = V * (b + 1) / B;
  {
    int local = 0;
    for (int64_t t0 = cb; t0 < ce; t0 += T) {
      const int64_t vv = t0 + threadIdx.x;
      int64_t v;
      if (vv < ce) local += __popc(candidate_mask(meta, n, p0, v0b, V0, vv, aligned, &v));
    }
    int total;
    block_excl_scan(local, &total, sh.scan);
    if (threadIdx.x == 0) g->cnt[b] = total;
  }
  KVCA_GRID_SYNC();
  int64_t nc, run;
  grid_prefix(g, &run, &nc, sh.scan);
  for (int64_t t0 = cb; t0 < ce; t0 += T) {
    const int64_t vv = t0 + threadIdx.x;
    int64_t v = 0;
    unsigned mask = vv < ce ? candidate_mask(meta, n, p0, v0b, V0, vv, aligned, &v) : 0u;
    int total;
    int64_t rank = run + block_excl_scan(__popc(mask), &total, sh.scan);
    while (mask != 0u) {
      const int j = __ffs(mask) - 1;
      mask &= mask - 1u;
      w.cand[rank++] = static_cast<int32_t>(v * kSpv + j);
    }
    run += total;
  }
  // steps these candidates can serve: at most nc / k, plus the step that fails
  int64_t s_hi = s0 + nc / k + 1;
  if (s_hi > steps) s_hi = steps;
  const int64_t ev_lo = s0 * m;
  const int64_t ev_hi = s_hi * m;

  // 2. first re-access step in the window, encoded as INT_MAX - step (0 = none)
  // (the first setter of a slot lists it; one list reservation per warp)
  for (int64_t e0 = ev_lo + (gt & ~int64_t{31}); e0 < ev_hi; e0 += G) {
    const int64_t e = e0 + (threadIdx.x & 31);
    bool first = false;
    int64_t x = -1;
    if (e < ev_hi) {
      x = reaccess[e];
      if (!slot_ok(x, n)) {
        report(status, KVCA_ERR_BAD_INDEX, x);
        x = -1;
      }
    }
    // lanes holding the same slot (a popular one) send one atomic: the
    // highest lane carries the earliest step, the largest encoding
    const unsigned peers = __match_any_sync(0xffffffffu, x);
    if (x >= 0 && (threadIdx.x & 31) == 31 - __clz(peers))
      first = atomicMax(w.first_bump + x, static_cast<int32_t>(INT32_MAX - (e0 + __ffs(peers) - 1) / m)) == 0;
    const unsigned firsts = __ballot_sync(0xffffffffu, first);
    if (firsts != 0u) {
      const int lane = threadIdx.x & 31;
      int base = 0;
      if (lane == __ffs(firsts) - 1) base = atomicAdd(&g->nu, __popc(firsts));
      base = __shfl_sync(0xffffffffu, base, __ffs(firsts) - 1);
      if (first) w.touched[base + __popc(firsts & ((1u << lane) - 1u))] = static_cast<int32_t>(x);
    }
  }
  KVCA_GRID_SYNC();
  const int nu = __ldcg(&g->nu);
  // 3a. list the pending candidates in order: (index << 32) | first re-access
  //     step; CTA b takes candidates [jc0, jc1) here and in 3c.
  //     A candidate is pending only if its first re-access can come before
  //     the step that takes it.  At most j candidates are taken before
  //     candidate j, so it is taken by step s0 + j / k at the latest: a first
  //     re-access at or after that step never passes it over, and it is
  //     treated as not pending.
  const int64_t jc0 = nc * b / B;
  const int64_t jc1 = nc * (b + 1) / B;
  {
    int local = 0;
    for (int64_t j = jc0 + threadIdx.x; j < jc1; j += T) {
      const int32_t enc = __ldcg(w.first_bump + __ldcg(w.cand + j));
      const int64_t first = enc == 0 ? INT32_MAX : INT32_MAX - enc;
      const int32_t cb = first >= s0 + j / k ? INT32_MAX : static_cast<int32_t>(first);
      w.cand_bump[j] = cb;
      local += cb != INT32_MAX;
    }
    int total;
    block_excl_scan(local, &total, sh.scan);
    if (threadIdx.x == 0) g->cnt[b] = total;
  }
  KVCA_GRID_SYNC();
  int64_t pend0, np;
  grid_prefix(g, &pend0, &np, sh.scan);
  {
    int64_t p_run = pend0;
    for (int64_t tile = jc0; tile < jc1; tile += T * C) {
      const int64_t jb = tile + static_cast<int64_t>(threadIdx.x) * C;
      int32_t bb[C];
      int cnt = 0;
#pragma unroll
      for (int u = 0; u < C; ++u) {
        bb[u] = jb + u < jc1 ? __ldcg(w.cand_bump + jb + u) : INT32_MAX;
        cnt += bb[u] != INT32_MAX;
      }
      int total;
      int64_t p = p_run + block_excl_scan(cnt, &total, sh.scan);
#pragma unroll
      for (int u = 0; u < C; ++u)
        if (bb[u] != INT32_MAX)
          w.pending[p++] = (static_cast<int64_t>(jb + u) << 32) | static_cast<uint32_t>(bb[u]);
      p_run += total;
    }
  }
  KVCA_GRID_SYNC();

  // 3b. CTA 0 resolves the pending candidates; each entry becomes
  //     (pending candidates taken before it << 1) | taken.
  //     Pending entry p (candidate j, first re-access bv) is taken iff
  //     tb < max_taken and bv >= s0 + tb / k, where tb = (j - p) + (pending
  //     taken before it), i.e. iff (pending taken before it) <= c with
  //     c = min(k (bv - s0) + k - 1, max_taken - 1) - (j - p).  As
  //     (pending taken before it) >= 0, an entry with c < 0 is surely passed
  //     over; only the others (few: their first re-access falls in the short
  //     window of steps the earlier pending ones can shift) go through the
  //     one-warp sequential pass, compacted in order through shared memory.
  //     A block-wide scan then gives every entry its count.
  const int32_t kk = static_cast<int32_t>(k);
  const int32_t max_taken = static_cast<int32_t>((steps - s0) * k);
  const int32_t step0 = static_cast<int32_t>(s0);
  if (b == 0) {
    constexpr int E = kPendingTile / kStreamThreads;
    const int lane = threadIdx.x & 31;
    const unsigned below = (1u << lane) - 1u;
    int64_t tp_start = 0;  // pending taken before the tile, same in every thread
    for (int64_t t0 = 0; t0 < np; t0 += kPendingTile) {
      const int cnt = static_cast<int>(np - t0 < kPendingTile ? np - t0 : kPendingTile);
      // each thread takes E consecutive entries of the tile
      int64_t cs[E];
      int unc = 0;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int i = static_cast<int>(threadIdx.x) * E + e;
        cs[e] = -1;
        if (i < cnt) {
          const int64_t pr = __ldcg(reinterpret_cast<const long long*>(w.pending) + t0 + i);
          const int64_t nonpending_before = (pr >> 32) - (t0 + i);
          const int64_t bv = pr & 0xffffffffll;
          int64_t c = kk * (bv - step0) + kk - 1;
          if (c > max_taken - 1) c = max_taken - 1;
          cs[e] = c - nonpending_before;
        }
        unc += cs[e] >= 0;
      }
      int n_unc;
      int pos = block_excl_scan(unc, &n_unc, sh.scan);
#pragma unroll
      for (int e = 0; e < E; ++e)
        if (cs[e] >= 0) sh.tile[pos++] = cs[e];
      __syncthreads();
      if (threadIdx.x < 32) {
        int64_t tp = tp_start;
        for (int q0 = 0; q0 < n_unc; q0 += 32) {
          const int q = q0 + lane;
          const bool here = q < n_unc;
          const int64_t c = here ? sh.tile[q] : -1;
          const unsigned present = __ballot_sync(0xffffffffu, here);
          unsigned cur = present;
          for (int it = 0; it < 33; ++it) {  // converges in at most 32 rounds
            const bool take = here && tp + __popc(cur & below) <= c;
            const unsigned ok_mask = __ballot_sync(0xffffffffu, take);
            const unsigned diff = (ok_mask ^ cur) & present;
            if (diff == 0u) break;
            const unsigned keep = (1u << (__ffs(diff) - 1)) - 1u;
            cur = (cur & keep) | (ok_mask & ~keep);
          }
          if (here) sh.tile[q] = (cur >> lane) & 1u;
          tp += __popc(cur);
        }
      }
      __syncthreads();
      // taken flags in entry order, then the count before each entry
      int taken_local = 0;
      unsigned flags = 0u;
      pos -= unc;  // this thread's first compacted slot again
#pragma unroll
      for (int e = 0; e < E; ++e) {
        if (cs[e] >= 0) {
          if (sh.tile[pos++] != 0) {
            flags |= 1u << e;
            ++taken_local;
          }
        }
      }
      int tile_taken;
      int64_t before = tp_start + block_excl_scan(taken_local, &tile_taken, sh.scan);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int i = static_cast<int>(threadIdx.x) * E + e;
        if (i < cnt) {
          const unsigned t = (flags >> e) & 1u;
          w.pending[t0 + i] = (before << 1) | t;
          before += t;
        }
      }
      tp_start += tile_taken;
      __syncthreads();  // sh.tile is refilled by the next tile
    }
    if (threadIdx.x == 0) g->tp_total = static_cast<int>(tp_start);
  }
  KVCA_GRID_SYNC();
  const int32_t tp_total = __ldcg(&g->tp_total);
  int64_t total_taken = (nc - np) + tp_total;
  if (total_taken > max_taken) total_taken = max_taken;
  const int64_t full = total_taken / k;  // complete steps of this epoch
  const int64_t full_pos = full * k;
  const int64_t s_end = s0 + full;

  // 3c. place every victim of the complete steps:
  //     taken before j = (j - pending before j) + pending taken before j
  {
    int64_t np_run = pend0;
    for (int64_t tile = jc0; tile < jc1; tile += T * C) {
      const int64_t jb = tile + static_cast<int64_t>(threadIdx.x) * C;
      int32_t bb[C];
      int cnt = 0;
#pragma unroll
      for (int u = 0; u < C; ++u) {
        bb[u] = jb + u < jc1 ? __ldcg(w.cand_bump + jb + u) : INT32_MAX;
        cnt += bb[u] != INT32_MAX;
      }
      int total;
      int64_t pp = np_run + block_excl_scan(cnt, &total, sh.scan);
      int64_t cached_pp = -1;
      int64_t entry = 0;
#pragma unroll
      for (int u = 0; u < C; ++u) {
        const int64_t j = jb + u;
        if (j >= jc1) continue;
        const bool is_pending = bb[u] != INT32_MAX;
        int64_t tpb = tp_total;
        if (pp < np) {
          if (pp != cached_pp) {
            entry = __ldcg(reinterpret_cast<const long long*>(w.pending) + pp);
            cached_pp = pp;
          }
          tpb = entry >> 1;
        }
        const int64_t tb = (j - pp) + tpb;
        const bool take = is_pending ? (entry & 1) != 0 : tb < max_taken;
        if (take && tb < full_pos) {
          const int32_t x = __ldcg(w.cand + j);
          victims[s0 * k + tb] = x;
          w.victim_step[x] = static_cast<int32_t>(s0 + tb / k + 1);
          if (tb == full_pos - 1) g->last_victim = x;
        }
        if (is_pending) ++pp;
      }
      np_run += total;
    }
  }
  KVCA_GRID_SYNC();
  const int64_t v_lo = s0 * k;
  const int64_t v_hi = s_end * k;
  const int64_t cnt_hi = s_end * m;

  // 4a. distinct bumping steps per slot (only steps >= a victim's own step).
  //     16 to 4,096 re-accesses per step: each CTA takes whole steps and
  //     inserts a step's ids into an open-addressing set in shared memory;
  //     the thread that inserts an id counts it.  Otherwise each event scans
  //     its step's earlier ids in memory.
  constexpr int kWarpSet = kPendingTile * 2 / (kStreamThreads / 32);  // int32 slots per warp
  if (m >= kHashDedupMin && 2 * m <= kWarpSet) {
    // small steps: every warp takes whole steps with a set of its own
    const int lane = threadIdx.x & 31;
    int32_t* set = reinterpret_cast<int32_t*>(sh.tile) + (threadIdx.x >> 5) * kWarpSet;
    int tsz = 1;
    while (tsz < 2 * m) tsz <<= 1;
    const uint32_t mask = static_cast<uint32_t>(tsz - 1);
    // consecutive steps go to different CTAs, so a short epoch still spreads
    const int64_t warp_id = b + B * (threadIdx.x >> 5);
    for (int64_t t = s0 + warp_id; t < s_end; t += G >> 5) {
      for (int i = lane; i < tsz; i += 32) set[i] = -1;
      // the step's ids (at most kWarpSet / 64 per lane), loaded together
      constexpr int kPerLane = kWarpSet / 64;
      int32_t keys[kPerLane];
#pragma unroll
      for (int u = 0; u < kPerLane; ++u) {
        const int64_t i = lane + 32 * u;
        const int64_t x = i < m ? reaccess[t * m + i] : -1;
        keys[u] = slot_ok(x, n) ? static_cast<int32_t>(x) : -1;
      }
      __syncwarp();
#pragma unroll
      for (int u = 0; u < kPerLane; ++u) {
        const int32_t key = keys[u];
        if (key < 0) continue;
        uint32_t h = (static_cast<uint32_t>(key) * 0x9E3779B1u) & mask;
        bool first = false;
        for (int probe = 0; probe < tsz; ++probe) {  // at most half full: ends at a free slot
          const int32_t old = atomicCAS(set + h, -1, key);
          if (old == -1) {
            first = true;
            break;
          }
          if (old == key) break;
          h = (h + 1u) & mask;
        }
        if (!first) keys[u] = -1;  // a repeat within the step
      }
      int32_t vss[kPerLane];
#pragma unroll
      for (int u = 0; u < kPerLane; ++u) vss[u] = keys[u] >= 0 ? __ldcg(w.victim_step + keys[u]) : -1;
#pragma unroll
      for (int u = 0; u < kPerLane; ++u)
        if (keys[u] >= 0 && (vss[u] == 0 || vss[u] - 1 <= t)) atomicAdd(w.bump_count + keys[u], 1);
      __syncwarp();
    }
  } else if (m >= kHashDedupMin && m <= kHashDedupMax) {
    int32_t* set = reinterpret_cast<int32_t*>(sh.tile);
    int tsz = 1;
    while (tsz < 2 * m) tsz <<= 1;
    const uint32_t mask = static_cast<uint32_t>(tsz - 1);
    for (int64_t t = s0 + b; t < s_end; t += B) {
      for (int i = threadIdx.x; i < tsz; i += blockDim.x) set[i] = -1;
      __syncthreads();
      for (int64_t i = threadIdx.x; i < m; i += T) {
        const int64_t x = reaccess[t * m + i];
        if (!slot_ok(x, n)) continue;
        const int32_t key = static_cast<int32_t>(x);
        uint32_t h = (static_cast<uint32_t>(key) * 0x9E3779B1u) & mask;
        bool first = false;
        for (int probe = 0; probe < tsz; ++probe) {  // at most half full: ends at a free slot
          const int32_t old = atomicCAS(set + h, -1, key);
          if (old == -1) {
            first = true;
            break;
          }
          if (old == key) break;
          h = (h + 1u) & mask;
        }
        if (!first) continue;
        const int32_t vs = __ldcg(w.victim_step + x);
        if (vs == 0 || vs - 1 <= t) atomicAdd(w.bump_count + x, 1);
      }
      __syncthreads();
    }
  } else {
    for (int64_t e0 = ev_lo + (gt & ~int64_t{31}); e0 < cnt_hi; e0 += G) {
      const int64_t e = e0 + (threadIdx.x & 31);
      int64_t key = -1;
      if (e < cnt_hi) {
        const int64_t x = reaccess[e];
        if (slot_ok(x, n)) {
          const int64_t t = e / m;
          bool dup = false;
#pragma unroll 8
          for (int64_t i = t * m; i < e; ++i) dup |= reaccess[i] == x;
          const int32_t vs = dup ? 0 : __ldcg(w.victim_step + x);
          if (!dup && (vs == 0 || vs - 1 <= t)) key = x;
        }
      }
      // one atomic per slot per warp (popular slots are bumped by many lanes)
      const unsigned peers = __match_any_sync(0xffffffffu, key);
      if (key >= 0 && (threadIdx.x & 31) == __ffs(peers) - 1)
        atomicAdd(w.bump_count + key, __popc(peers));
    }
  }
  KVCA_GRID_SYNC();

  // 4b. final usage of every touched slot (each listed re-accessed slot once,
  //     plus the victims), computed from the epoch-start words and written
  //     straight back.  A slot listed twice (a victim that was also
  //     re-accessed) gets the same word from both: a victim's final usage
  //     does not depend on its old usage, and no pin changes, so whichever
  //     of the two reads the word first or last, both store the same value.
  const int64_t n_touched = nu + (v_hi - v_lo);
  auto touched_slot = [&](int64_t i) -> int64_t {
    return i < nu ? static_cast<int64_t>(__ldcg(w.touched + i))
                  : static_cast<int64_t>(__ldcg(reinterpret_cast<const long long*>(victims) + v_lo + (i - nu)));
  };
  constexpr int kU = 4;
  for (int64_t i0 = gt; i0 < n_touched; i0 += G * kU) {
    int64_t xs[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = i0 + static_cast<int64_t>(u) * G;
      xs[u] = i < n_touched ? touched_slot(i) : -1;
    }
    unsigned ws[kU];
    int32_t vss[kU], cts[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const bool okx = slot_ok(xs[u], n);
      ws[u] = okx ? static_cast<unsigned>(__ldcg(meta + xs[u])) : 0u;
      vss[u] = okx ? __ldcg(w.victim_step + xs[u]) : 0;
      cts[u] = okx ? __ldcg(w.bump_count + xs[u]) : 0;
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (!slot_ok(xs[u], n)) continue;
      int64_t fin = (vss[u] != 0 ? 1 : static_cast<int64_t>(M::usage(ws[u]))) + cts[u];
      if (fin > M::kUsageMax) fin = M::kUsageMax;
      meta[xs[u]] = M::pack(M::pin(ws[u]), fin);
    }
  }
  KVCA_GRID_SYNC();
  // 4c. leave the per-slot scratch words zero again
  for (int64_t i = gt; i < n_touched; i += G) {
    const int64_t x = touched_slot(i);
    if (!slot_ok(x, n)) continue;
    w.first_bump[x] = 0;
    w.victim_step[x] = 0;
    w.bump_count[x] = 0;
  }
  if (b == 0 && threadIdx.x == 0 && s_end > s0)
    *search_start = (__ldcg(&g->last_victim) + 1) % n;
  // the stream goes on: the next epoch or exact step needs the cleared
  // scratch and search_start; when it ends here, so does the launch
  if (s_end < steps) KVCA_GRID_SYNC();
#undef KVCA_GRID_SYNC
  return s_end;
}

template <typename MetaT>
__global__ void __launch_bounds__(kStreamThreads)
    clock_stream_batched_kernel(MetaT* meta, int64_t num_slots, int64_t* search_start,
                                int64_t num_steps, int64_t alloc_per_step, const int64_t* reaccess,
                                int64_t reaccess_per_step, int64_t* victims, int64_t* steps_done,
                                int order, bool aligned, unsigned char* scratch, int64_t* status) {
  __shared__ EpochShared<MetaT> sh;
  const int64_t n = num_slots;
  EpochScratch w;
  w.pending = reinterpret_cast<int64_t*>(scratch);
  w.cand = reinterpret_cast<int32_t*>(scratch + 8 * n);
  w.cand_bump = reinterpret_cast<int32_t*>(scratch + 12 * n);
  w.touched = reinterpret_cast<int32_t*>(scratch + 16 * n);
  w.first_bump = reinterpret_cast<int32_t*>(scratch + 20 * n);
  w.victim_step = reinterpret_cast<int32_t*>(scratch + 24 * n);
  w.bump_count = reinterpret_cast<int32_t*>(scratch + 28 * n);
  StreamGrid* g = reinterpret_cast<StreamGrid*>(scratch + 32 * n);
  int64_t s = 0;
  int64_t exact_until = 0;
  bool ok = true;
  while (s < num_steps) {
    if (s >= exact_until) {
      const int64_t s_end = stream_epoch<MetaT>(meta, n, search_start, s, num_steps, alloc_per_step,
                                                reaccess, reaccess_per_step, victims, w, g,
                                                aligned, status, sh, &ok);
      if (!ok) return;
      if (s_end - s < kEpochMinSteps) exact_until = s_end + 1 + kExactStepsAfterShortEpoch;
      s = s_end;
      if (s >= num_steps) break;
    }
    // an exact step (one that ages usage) on CTA 0 while the others wait
    if (blockIdx.x == 0) {
      const int rc = stream_step<MetaT>(meta, n, search_start, s, alloc_per_step, reaccess,
                                        reaccess_per_step, victims, order, aligned, status, sh.pop);
      if (threadIdx.x == 0) g->rc = rc;
    }
    if (!grid_barrier(g, status)) return;
    const int rc = __ldcg(&g->rc);
    if (rc != KVCA_OK) {
      if (blockIdx.x == 0 && threadIdx.x == 0) report(status, rc, s);
      break;
    }
    ++s;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *steps_done = s;
}

// ---------------------------------------------------------------------------
// Inspect / commit / release
// ---------------------------------------------------------------------------

template <typename MetaT>
__global__ void inspect_load_kernel(const int64_t* l2p, int64_t num_logical, const MetaT* meta,
                                    int64_t num_slots, const int64_t* ids, int64_t count,
                                    int64_t* cur_out, uint8_t* resident_out, int64_t* pin_out,
                                    MetaT* usage_out, int64_t* status) {
  using M = Meta<MetaT>;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t id = ids[i];
    int64_t cur = -1;
    if (id < 0 || id >= num_logical) {
      report(status, KVCA_ERR_BAD_INDEX, id);
    } else {
      cur = l2p[id];
    }
    bool resident = false;
    int64_t pin = 0;
    unsigned usage = 0u;
    if (cur >= num_slots) {
      report(status, KVCA_ERR_BAD_INDEX, cur);
    } else if (cur >= 0) {
      const unsigned w = meta[cur];
      resident = true;
      pin = static_cast<int64_t>(M::pin(w)) + 1;
      usage = M::sat_inc(M::usage(w));
    }
    cur_out[i] = cur;
    resident_out[i] = resident ? 1 : 0;
    pin_out[i] = pin;
    usage_out[i] = static_cast<MetaT>(usage);
  }
}

template <typename MetaT>
__global__ void inspect_save_kernel(const int64_t* l2p, int64_t num_logical, const MetaT* meta,
                                    int64_t num_slots, const int64_t* ids, int64_t count,
                                    int64_t* cur_out, uint8_t* existing_out, MetaT* usage_out,
                                    int64_t* status) {
  using M = Meta<MetaT>;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t id = ids[i];
    int64_t cur = -1;
    if (id < 0 || id >= num_logical) {
      report(status, KVCA_ERR_BAD_INDEX, id);
    } else {
      cur = l2p[id];
    }
    bool existing = false;
    unsigned usage = 1u;
    if (cur >= num_slots) {
      report(status, KVCA_ERR_BAD_INDEX, cur);
    } else if (cur >= 0) {
      existing = true;
      usage = M::sat_inc(M::usage(meta[cur]));
    }
    cur_out[i] = cur;
    existing_out[i] = existing ? 1 : 0;
    usage_out[i] = static_cast<MetaT>(usage);
  }
}

__device__ __forceinline__ bool in_range(int64_t x, int64_t n) { return x >= 0 && x < n; }

// Every id of the call must be inside its table before anything is written,
// as in the reference, whose torch indexing raises before mutating.  Returns
// true (uniformly) when all ids are valid; otherwise reports the first one.
__device__ bool all_in_range(const int64_t* ids, int64_t count, int64_t limit, int64_t* status,
                             int* flag) {
  for (int64_t i = threadIdx.x; i < count; i += blockDim.x) {
    const int64_t v = ids[i];
    if (!in_range(v, limit)) {
      *flag = 1;
      report(status, KVCA_ERR_BAD_INDEX, v);
    }
  }
  __syncthreads();
  return *flag == 0;
}

// l2p[ids[i]] = slots[i] for i in [0, count), a repeated id keeping the slot
// of its last occurrence, as a sequential index_put_ leaves it.  Every
// target is first set to a mark below any encoded position, the largest
// position per id is then elected with atomicMax, and only the elected
// thread stores its slot (the others read back either the winner's encoded
// position or the stored slot, never their own).  Ends without a barrier.
__device__ void scatter_last_wins(int64_t* l2p, const int64_t* ids, const int64_t* slots,
                                  int64_t count) {
  constexpr long long kMark = LLONG_MIN;
  for (int64_t i = threadIdx.x; i < count; i += blockDim.x) l2p[ids[i]] = kMark;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < count; i += blockDim.x)
    atomicMax(reinterpret_cast<long long*>(l2p + ids[i]), kMark + 1 + i);
  __syncthreads();
  for (int64_t i = threadIdx.x; i < count; i += blockDim.x)
    if (__ldcg(reinterpret_cast<const long long*>(l2p + ids[i])) == kMark + 1 + i)
      l2p[ids[i]] = slots[i];
}

// Commit bodies, run by one CTA, phases separated by barriers so each phase
// sees the previous one.  `bad` is a zeroed shared flag.
template <typename MetaT>
__device__ void commit_load_body(int64_t* l2p, int64_t num_logical, int64_t* p2l, MetaT* meta,
                                 int64_t num_slots, const int64_t* evicted, int64_t num_evicted,
                                 const int64_t* miss_ids, const int64_t* miss_slots,
                                 int64_t num_miss, const int64_t* hit_slots,
                                 const int64_t* hit_pins, const MetaT* hit_usage, int64_t num_hit,
                                 const MetaT* miss_usage, int64_t* status, int* bad) {
  using M = Meta<MetaT>;
  if (!all_in_range(evicted, num_evicted, num_logical, status, bad)) return;
  if (!all_in_range(miss_ids, num_miss, num_logical, status, bad)) return;
  if (!all_in_range(miss_slots, num_miss, num_slots, status, bad)) return;
  if (!all_in_range(hit_slots, num_hit, num_slots, status, bad)) return;
  for (int64_t i = threadIdx.x; i < num_evicted; i += blockDim.x) l2p[evicted[i]] = -1;
  __syncthreads();
  scatter_last_wins(l2p, miss_ids, miss_slots, num_miss);
  for (int64_t i = threadIdx.x; i < num_miss; i += blockDim.x) p2l[miss_slots[i]] = miss_ids[i];
  __syncthreads();
  for (int64_t i = threadIdx.x; i < num_hit; i += blockDim.x)
    meta[hit_slots[i]] = M::pack(hit_pins[i], hit_usage[i]);
  __syncthreads();
  // no miss_usage: every miss takes usage 1, as KVCacheAdapter.load passes it
  for (int64_t i = threadIdx.x; i < num_miss; i += blockDim.x)
    meta[miss_slots[i]] = M::pack(1, miss_usage != nullptr ? miss_usage[i] : MetaT(1));
}

template <typename MetaT>
__device__ void commit_save_body(int64_t* l2p, int64_t num_logical, int64_t* p2l, MetaT* meta,
                                 int64_t num_slots, const int64_t* evicted, int64_t num_evicted,
                                 const int64_t* ids, const int64_t* slots, const MetaT* final_pins,
                                 const MetaT* final_usage, int64_t count, int64_t* status,
                                 int* bad) {
  using M = Meta<MetaT>;
  if (!all_in_range(evicted, num_evicted, num_logical, status, bad)) return;
  if (!all_in_range(ids, count, num_logical, status, bad)) return;
  if (!all_in_range(slots, count, num_slots, status, bad)) return;
  for (int64_t i = threadIdx.x; i < num_evicted; i += blockDim.x) l2p[evicted[i]] = -1;
  __syncthreads();
  scatter_last_wins(l2p, ids, slots, count);
  // a repeated slot is repeated with its id, pins and usage: any store wins
  for (int64_t i = threadIdx.x; i < count; i += blockDim.x) {
    p2l[slots[i]] = ids[i];
    meta[slots[i]] = M::pack(final_pins[i], final_usage[i]);
  }
}

template <typename MetaT>
__global__ void __launch_bounds__(1024)
    commit_load_kernel(int64_t* l2p, int64_t num_logical, int64_t* p2l, MetaT* meta,
                       int64_t num_slots, const int64_t* evicted, int64_t num_evicted,
                       const int64_t* miss_ids, const int64_t* miss_slots, int64_t num_miss,
                       const int64_t* hit_slots, const int64_t* hit_pins, const MetaT* hit_usage,
                       int64_t num_hit, const MetaT* miss_usage, int64_t* status) {
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  __syncthreads();
  commit_load_body<MetaT>(l2p, num_logical, p2l, meta, num_slots, evicted, num_evicted, miss_ids,
                          miss_slots, num_miss, hit_slots, hit_pins, hit_usage, num_hit,
                          miss_usage, status, &bad);
}

template <typename MetaT>
__global__ void __launch_bounds__(1024)
    commit_save_kernel(int64_t* l2p, int64_t num_logical, int64_t* p2l, MetaT* meta,
                       int64_t num_slots, const int64_t* evicted, int64_t num_evicted,
                       const int64_t* ids, const int64_t* slots, const MetaT* final_pins,
                       const MetaT* final_usage, int64_t count, int64_t* status) {
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  __syncthreads();
  commit_save_body<MetaT>(l2p, num_logical, p2l, meta, num_slots, evicted, num_evicted, ids,
                          slots, final_pins, final_usage, count, status, &bad);
}

constexpr int kReleasePerThread = 8;

// One CTA.  All ids are checked first; then every new word is computed from
// the words as they were on entry and only then written, so an id listed
// twice releases one pin, as the reference's index_select + index_put_ does.
// Batches above 1024 * kReleasePerThread ids run in rounds of that size.
template <typename MetaT>
__global__ void __launch_bounds__(1024)
    release_kernel(const int64_t* l2p, int64_t num_logical, MetaT* meta, int64_t num_slots,
                   const int64_t* ids, int64_t count, int64_t* status) {
  using M = Meta<MetaT>;
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  __syncthreads();
  if (!all_in_range(ids, count, num_logical, status, &bad)) return;
  for (int64_t i = threadIdx.x; i < count; i += blockDim.x) {
    const int64_t slot = l2p[ids[i]];
    if (!in_range(slot, num_slots)) {
      bad = 1;
      report(status, KVCA_ERR_BAD_INDEX, slot);
    }
  }
  __syncthreads();
  if (bad) return;
  const int64_t round = static_cast<int64_t>(blockDim.x) * kReleasePerThread;
  for (int64_t base = 0; base < count; base += round) {
    int64_t slot[kReleasePerThread];
    MetaT next[kReleasePerThread];
#pragma unroll
    for (int u = 0; u < kReleasePerThread; ++u) {
      const int64_t i = base + threadIdx.x + static_cast<int64_t>(u) * blockDim.x;
      slot[u] = -1;
      next[u] = MetaT(0);
      if (i < count) {
        slot[u] = l2p[ids[i]];
        const unsigned w = meta[slot[u]];
        next[u] = M::pack(static_cast<int64_t>(M::pin(w)) - 1, M::usage(w));
      }
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < kReleasePerThread; ++u)
      if (slot[u] >= 0) meta[slot[u]] = next[u];
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Load / save planning: everything of KVCacheAdapter.load / save that decides
// slots, in one CTA, so the host synchronises once per call (to size the
// backend calls) instead of at every step.
// ---------------------------------------------------------------------------
//
// counts[0..4] = n_hit (load) or n_existing (save), n_miss, n_evict, error
// code, error value.  On an error nothing but the outputs is written (a bad
// id is found before anything changes; too few reusable slots leave the
// table as the pop found it).

constexpr int kPackShift = 16;  // hit/miss tile counts packed in one scan word

constexpr int kPlanThreads = 1024;

template <typename MetaT>
struct PlanShared {
  PopShared<MetaT> pop;
  int bad;
  int repeated;
  long long bad_value;
  long long rkeys[2 * kPlanThreads];  // slot -> largest position in the tile (repeated saves)
  int rvals[2 * kPlanThreads];
};

__device__ __forceinline__ void plan_fail(int64_t* counts, int64_t* status, int code, int64_t value) {
  counts[3] = code;
  counts[4] = value;
  report(status, code, value);
}

// counts[5..6] take the status word as the plan finds it, so that the one
// read of counts also reports an error latched by an earlier unchecked launch.
__device__ __forceinline__ void plan_begin(int64_t* counts, const int64_t* status) {
  counts[3] = counts[4] = 0;
  counts[5] = status[0];
  counts[6] = status[1];
}

// Validates ids and their current slots; returns false (uniformly) on a bad id.
template <typename MetaT>
__device__ bool plan_validate(const int64_t* l2p, int64_t n_logical, int64_t n, const int64_t* ids,
                              int64_t k, int64_t* counts, int64_t* status, PlanShared<MetaT>& sh) {
  if (threadIdx.x == 0) sh.bad = 0;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
    const int64_t id = ids[i];
    bool bad = !in_range(id, n_logical);
    int64_t v = id;
    if (!bad) {
      const int64_t cur = l2p[id];
      if (cur >= n) {
        bad = true;
        v = cur;
      }
    }
    if (bad && atomicCAS(&sh.bad, 0, 1) == 0) sh.bad_value = v;
  }
  __syncthreads();
  if (sh.bad) {
    if (threadIdx.x == 0) plan_fail(counts, status, KVCA_ERR_BAD_INDEX, sh.bad_value);
    return false;
  }
  return true;
}

// KVCacheAdapter.load up to the backend calls (adapter.py:264-305):
// inspect (hits: pin + 1, usage + 1 saturating), hit / miss compaction in
// request order, pop(#miss) with the hit slots blocked, the eviction plan of
// the popped slots, the hits' usage re-read after the pop's aging, and the
// returned slots.
template <typename MetaT>
__device__ void plan_load_body(const int64_t* l2p, int64_t n_logical, const int64_t* p2l, MetaT* meta, int64_t n,
                               int64_t* search_start, const int64_t* ids, int64_t k, uint32_t* bitmap,
                               int order, bool aligned, int64_t* result, int64_t* hit_slots,
                               int64_t* hit_pins, MetaT* hit_usage, int64_t* miss_ids, int64_t* victims,
                               int64_t* evict_ids, int64_t* evict_slots, int64_t* counts, int64_t* status,
                               PlanShared<MetaT>& sh) {
  using M = Meta<MetaT>;
  if (threadIdx.x == 0) plan_begin(counts, status);
  if (!plan_validate<MetaT>(l2p, n_logical, n, ids, k, counts, status, sh)) return;
  // hits and misses in request order
  int64_t nh = 0, nm = 0;
  for (int64_t tile = 0; tile < k; tile += blockDim.x) {
    const int64_t i = tile + threadIdx.x;
    const int64_t cur = i < k ? l2p[ids[i]] : -1;
    const bool hit = i < k && cur >= 0;
    const bool miss = i < k && cur < 0;
    int total;
    const int base = block_excl_scan((hit ? 1 : 0) | ((miss ? 1 : 0) << kPackShift), &total, sh.pop.scan);
    if (hit) {
      const int64_t r = nh + (base & ((1 << kPackShift) - 1));
      const unsigned w = meta[cur];
      hit_slots[r] = cur;
      hit_pins[r] = static_cast<int64_t>(M::pin(w)) + 1;
      hit_usage[r] = static_cast<MetaT>(M::sat_inc(M::usage(w)));
      result[i] = cur;
    }
    if (miss) miss_ids[nm + (base >> kPackShift)] = ids[i];
    nh += total & ((1 << kPackShift) - 1);
    nm += total >> kPackShift;
  }
  if (nm == 0) {  // every request hit: no pop, no eviction plan (nm is uniform across the CTA)
    if (threadIdx.x == 0) {
      counts[0] = nh;
      counts[1] = 0;
      counts[2] = 0;
    }
    return;
  }
  __syncthreads();  // this thread's hit slots were written by others
  // the hit slots are blocked for the pop
  for (int64_t j = threadIdx.x; j < nh; j += blockDim.x) {
    const int64_t b = hit_slots[j];
    atomicOr(bitmap + (b >> 5), 1u << (b & 31));
  }
  __syncthreads();
  const int rc = pop_cta<MetaT>(meta, n, search_start, bitmap, nm, victims, order, aligned, sh.pop);
  __syncthreads();
  for (int64_t j = threadIdx.x; j < nh; j += blockDim.x) {
    const int64_t b = hit_slots[j];
    atomicAnd(bitmap + (b >> 5), ~(1u << (b & 31)));
  }
  if (rc != KVCA_OK) {
    if (threadIdx.x == 0) plan_fail(counts, status, rc, nm);
    return;
  }
  // returned slots at the miss positions; the eviction plan of the victims
  int64_t mi = 0, ne = 0;
  for (int64_t tile = 0; tile < k; tile += blockDim.x) {
    const int64_t i = tile + threadIdx.x;
    const bool miss = i < k && l2p[ids[i]] < 0;
    int total;
    const int base = block_excl_scan(miss ? 1 : 0, &total, sh.pop.scan);
    if (miss) result[i] = victims[mi + base];
    mi += total;
  }
  for (int64_t tile = 0; tile < nm; tile += blockDim.x) {
    const int64_t j = tile + threadIdx.x;
    int64_t prev = -1;
    if (j < nm) prev = p2l[victims[j]];
    const bool ev = j < nm && prev >= 0 && prev != miss_ids[j];
    int total;
    const int base = block_excl_scan(ev ? 1 : 0, &total, sh.pop.scan);
    if (ev) {
      evict_ids[ne + base] = prev;
      evict_slots[ne + base] = victims[j];
    }
    ne += total;
  }
  // the pop may have aged usage: hits take usage + 1 of what is left
  for (int64_t j = threadIdx.x; j < nh; j += blockDim.x)
    hit_usage[j] = static_cast<MetaT>(M::sat_inc(M::usage(meta[hit_slots[j]])));
  if (threadIdx.x == 0) {
    counts[0] = nh;
    counts[1] = nm;
    counts[2] = ne;
  }
}

template <typename MetaT>
__global__ void __launch_bounds__(1024)
    plan_load_kernel(const int64_t* l2p, int64_t n_logical, const int64_t* p2l, MetaT* meta, int64_t n,
                     int64_t* search_start, const int64_t* ids, int64_t k, uint32_t* bitmap,
                     int order, bool aligned, int64_t* result, int64_t* hit_slots, int64_t* hit_pins,
                     MetaT* hit_usage, int64_t* miss_ids, int64_t* victims, int64_t* evict_ids,
                     int64_t* evict_slots, int64_t* counts, int64_t* status) {
  __shared__ PlanShared<MetaT> sh;
  plan_load_body<MetaT>(l2p, n_logical, p2l, meta, n, search_start, ids, k, bitmap, order, aligned, result,
                        hit_slots, hit_pins, hit_usage, miss_ids, victims, evict_ids, evict_slots, counts,
                        status, sh);
}

// KVCacheAdapter.save up to the backend call (adapter.py:221-243): existing /
// missing compaction, pop(#missing) with the existing slots blocked, the
// selected slots, final pins and usage read after the pop, and the eviction
// plan over every selected slot in request order.
template <typename MetaT>
__device__ void plan_save_body(const int64_t* l2p, int64_t n_logical, const int64_t* p2l, MetaT* meta, int64_t n,
                               int64_t* search_start, const int64_t* ids, int64_t k, uint32_t* bitmap,
                               int order, bool aligned, int64_t* selected, int64_t* move_slots,
                               MetaT* final_pins, MetaT* final_usage, int64_t* allocated, int64_t* evict_ids,
                               int64_t* evict_slots, int64_t* counts, int64_t* status, PlanShared<MetaT>& sh) {
  using M = Meta<MetaT>;
  if (threadIdx.x == 0) {
    plan_begin(counts, status);
    sh.repeated = 0;
  }
  if (!plan_validate<MetaT>(l2p, n_logical, n, ids, k, counts, status, sh)) return;
  int64_t nx = 0, nm = 0;
  for (int64_t tile = 0; tile < k; tile += blockDim.x) {
    const int64_t i = tile + threadIdx.x;
    const int64_t cur = i < k ? l2p[ids[i]] : -1;
    const bool ex = i < k && cur >= 0;
    const bool miss = i < k && cur < 0;
    int total;
    block_excl_scan((ex ? 1 : 0) | ((miss ? 1 : 0) << kPackShift), &total, sh.pop.scan);
    if (ex) {
      const unsigned bit = 1u << (cur & 31);
      if (atomicOr(bitmap + (cur >> 5), bit) & bit) sh.repeated = 1;  // an existing id asked twice
      selected[i] = cur;
    }
    nx += total & ((1 << kPackShift) - 1);
    nm += total >> kPackShift;
  }
  __syncthreads();
  int rc = KVCA_OK;
  if (nm > 0) rc = pop_cta<MetaT>(meta, n, search_start, bitmap, nm, allocated, order, aligned, sh.pop);
  __syncthreads();
  const bool repeated = sh.repeated != 0;
  if (!repeated) {
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
      const int64_t cur = l2p[ids[i]];
      if (cur >= 0) atomicAnd(bitmap + (cur >> 5), ~(1u << (cur & 31)));
    }
  } else {
    // Rows for the data scatter: an existing slot named more than once takes
    // the row of its last occurrence (index_copy_ applied in order), the
    // earlier ones are dropped (-1).  Tiles from the last to the first: in a
    // tile, a shared-memory map elects each slot's largest position, and that
    // position is the last occurrence overall if the slot's blocked bit is
    // still set; clearing the bit tells earlier tiles.  Every bit ends clear.
    const int tsz = 2 * static_cast<int>(blockDim.x);
    for (int64_t tile = ((k - 1) / blockDim.x) * blockDim.x; tile >= 0; tile -= blockDim.x) {
      for (int h = threadIdx.x; h < tsz; h += blockDim.x) {
        sh.rkeys[h] = -1;
        sh.rvals[h] = -1;
      }
      __syncthreads();
      const int64_t i = tile + threadIdx.x;
      const int64_t cur = i < k ? l2p[ids[i]] : -1;
      int h = -1;
      if (cur >= 0) {
        h = static_cast<int>((static_cast<uint64_t>(cur) * 0x9E3779B97F4A7C15ull) >> 40) & (tsz - 1);
        for (int probe = 0; probe < tsz; ++probe) {  // at most half full
          const long long old = atomicCAS(reinterpret_cast<unsigned long long*>(sh.rkeys + h),
                                          static_cast<unsigned long long>(-1ll),
                                          static_cast<unsigned long long>(cur));
          if (old == -1ll || old == cur) break;
          h = (h + 1) & (tsz - 1);
        }
        atomicMax(sh.rvals + h, static_cast<int>(threadIdx.x));
      }
      __syncthreads();
      if (cur >= 0) {
        bool last = false;
        if (sh.rvals[h] == static_cast<int>(threadIdx.x)) {
          const unsigned bit = 1u << (cur & 31);
          last = (atomicAnd(bitmap + (cur >> 5), ~bit) & bit) != 0u;
        }
        if (rc == KVCA_OK) move_slots[i] = last ? cur : -1;
      }
      __syncthreads();
    }
  }
  if (rc != KVCA_OK) {
    if (threadIdx.x == 0) plan_fail(counts, status, rc, nm);
    return;
  }
  int64_t mi = 0, ne = 0;
  for (int64_t tile = 0; tile < k; tile += blockDim.x) {
    const int64_t i = tile + threadIdx.x;
    const int64_t cur = i < k ? l2p[ids[i]] : -1;
    const bool miss = i < k && cur < 0;
    int total;
    const int base = block_excl_scan(miss ? 1 : 0, &total, sh.pop.scan);
    int64_t slot = cur;
    if (miss) {
      slot = allocated[mi + base];
      selected[i] = slot;
    }
    if (i < k && (miss || !repeated)) move_slots[i] = slot;
    bool ev = false;
    int64_t prev = -1;
    if (i < k) {
      const unsigned w = meta[slot];
      final_pins[i] = static_cast<MetaT>(M::pin(w));
      final_usage[i] = static_cast<MetaT>(miss ? 1u : M::sat_inc(M::usage(w)));
      prev = p2l[slot];
      ev = prev >= 0 && prev != ids[i];
    }
    mi += total;
    __syncthreads();
    int etotal;
    const int ebase = block_excl_scan(ev ? 1 : 0, &etotal, sh.pop.scan);
    if (ev) {
      evict_ids[ne + ebase] = prev;
      evict_slots[ne + ebase] = slot;
    }
    ne += etotal;
  }
  if (threadIdx.x == 0) {
    counts[0] = nx;
    counts[1] = nm;
    counts[2] = ne;
  }
}

template <typename MetaT>
__global__ void __launch_bounds__(1024)
    plan_save_kernel(const int64_t* l2p, int64_t n_logical, const int64_t* p2l, MetaT* meta, int64_t n,
                     int64_t* search_start, const int64_t* ids, int64_t k, uint32_t* bitmap,
                     int order, bool aligned, int64_t* selected, int64_t* move_slots,
                     MetaT* final_pins, MetaT* final_usage, int64_t* allocated, int64_t* evict_ids,
                     int64_t* evict_slots, int64_t* counts, int64_t* status) {
  __shared__ PlanShared<MetaT> sh;
  plan_save_body<MetaT>(l2p, n_logical, p2l, meta, n, search_start, ids, k, bitmap, order, aligned, selected,
                        move_slots, final_pins, final_usage, allocated, evict_ids, evict_slots, counts, status,
                        sh);
}

// ---------------------------------------------------------------------------
// Decode append: one step of a paged cache's block bookkeeping
// ---------------------------------------------------------------------------
//
// Sequences append one token per step into their current block.  The c
// sequences need[0..c) whose block is full get a new one in one CTA: pop(c)
// (victims, in order), each victim's previous logical id unmapped (l2p = -1),
// the victim committed as logical id next_logical + j, pinned, usage 1 (a
// fresh save, as commit_save_metadata with pins and usage 1), the full block
// released (pin - 1), and the sequence's block, logical id and position
// reset.  Then every sequence's slot_mapping entry for this step is
// cur_block * block_size + pos and its position advances.  The sequence is
// the composition pop_reusable_slots -> commit_save_metadata ->
// release_metadata of those ops (adapter.py:472-525, :647-651, :309-336).
// Ids are checked before anything changes; too few reusable slots change
// nothing.
// A small CTA: the step is a chain of short dependent phases, and block
// barriers of 8 warps are cheaper than of 32 (decode mix, B200: 16.1 us per
// decode step at 256 threads, 16.7 at 512, 18.5 at 1024, 16.3 at 128).
//
// The step is latency-bound: its cost is the number of dependent global
// round trips.  Every read that does not depend on another is issued at
// the start (the id checks' need -> cur_logical -> l2p chain, the scan
// start, the sequences' blocks and positions), the pop's scan reads the
// metadata right after the checks, and the victims stay in shared memory,
// so the chain is: ids (3 deep) -> metadata tile -> p2l of the victims and
// the full blocks' words -> stores.  Nothing is written before the checks
// pass.  The step blocks no slot, so the pop reads no bitmap.
constexpr int kAppendThreads = 256;
constexpr int kAppendMaxSteps = 256;  // steps of one append_steps launch (offsets staged in shared memory)

template <typename MetaT>
struct AppendShared {
  PopShared<MetaT> pop;
  int64_t victims[kAppendThreads];
  long long bad_value;
};

// One step (see above) for need[0..c), victims[0..c) and slot_mapping[0..seqs).
// Returns KVCA_OK or the reported error code, uniformly across the CTA.  On
// an error the step has changed nothing.  Every thread's global writes of
// the step are visible to the CTA after its next block barrier.
template <typename MetaT>
__device__ int append_step_body(MetaT* meta, int64_t n, int64_t* search_start, int64_t* l2p,
                                int64_t n_logical, int64_t* p2l, const int64_t* need, int64_t c,
                                int64_t* cur_block, int64_t* cur_logical, int64_t* pos,
                                int64_t seqs, int64_t block_size, int64_t* next_logical, int order,
                                bool aligned, int64_t* victims, int64_t* slot_mapping,
                                int64_t* status, AppendShared<MetaT>& sh, MetaT* mirror = nullptr) {
  using M = Meta<MetaT>;
  const int64_t base = *next_logical;
  if (c > 0 && threadIdx.x == 0) pop_start(search_start, n, sh.pop);
  // this thread's sequence for the slot_mapping pass
  int64_t my_block = 0, my_pos = 0;
  if (threadIdx.x < seqs) {
    my_block = cur_block[threadIdx.x];
    my_pos = pos[threadIdx.x];
  }
  // Thread t keeps what it reads for need entry t (the common case: at most
  // one entry per thread); entries beyond the block size are read again.
  int64_t my_q = -1, my_full = -1;
  bool bad = false;
  for (int64_t j = threadIdx.x; j < c; j += blockDim.x) {
    const int64_t q = need[j];
    int64_t v = q;
    int64_t full = -1;
    bool ok = in_range(q, seqs);
    if (ok) {
      v = cur_logical[q];
      ok = in_range(v, n_logical);
      if (ok) {
        full = l2p[v];
        ok = in_range(full, n);
        if (!ok) v = full;
      }
    }
    if (!ok) {
      bad = true;
      sh.bad_value = v;  // any one of the bad values
    }
    if (j == threadIdx.x) {
      my_q = q;
      my_full = full;
    }
  }
  if (threadIdx.x == 0 && c > 0 && (base < 0 || base + c > n_logical)) {
    bad = true;
    sh.bad_value = base + c;
  }
  if (__syncthreads_or(bad)) {
    if (threadIdx.x == 0) report(status, KVCA_ERR_BAD_INDEX, sh.bad_value);
    return KVCA_ERR_BAD_INDEX;
  }
  if (c > 0) {
    const int rc = pop_cta<MetaT>(meta, n, search_start, nullptr, c, victims, order, aligned, sh.pop,
                                  true, sh.victims, kAppendThreads, mirror);
    if (rc != KVCA_OK) {
      if (threadIdx.x == 0) report(status, rc, c);
      return rc;
    }
    // Unmap the victims' previous ids, commit the new ones, release the full
    // blocks.  The writes of different entries never meet: evicted ids are
    // older than base, the full blocks are pinned (never victims) and each
    // sequence appears once.  The full blocks' words are read after the pop,
    // which may have aged them.
    for (int64_t j = threadIdx.x; j < c; j += blockDim.x) {
      const int64_t q = j == threadIdx.x ? my_q : need[j];
      const int64_t full = j == threadIdx.x ? my_full : l2p[cur_logical[q]];
      const int64_t v = j < kAppendThreads ? sh.victims[j] : victims[j];
      const int64_t prev = p2l[v];
      const unsigned w = mirror != nullptr ? mirror[full] : meta[full];
      if (prev >= 0) l2p[prev] = -1;
      l2p[base + j] = v;
      p2l[v] = base + j;
      const MetaT fresh = M::pack(1, 1);
      const MetaT released = M::pack(static_cast<int64_t>(M::pin(w)) - 1, M::usage(w));
      meta[v] = fresh;
      meta[full] = released;
      if (mirror != nullptr) {
        mirror[v] = fresh;
        mirror[full] = released;
      }
      cur_block[q] = v;
      cur_logical[q] = base + j;
    }
    if (threadIdx.x == 0) *next_logical = base + c;
  }
  // this step's token slots; the sequences that got a new block are
  // rewritten below (block v, position 0)
  for (int64_t q = threadIdx.x; q < seqs; q += blockDim.x) {
    const int64_t b = q == threadIdx.x ? my_block : cur_block[q];
    const int64_t p = q == threadIdx.x ? my_pos : pos[q];
    slot_mapping[q] = b * block_size + p;
    pos[q] = p + 1;
  }
  if (c > 0) {
    __syncthreads();
    for (int64_t j = threadIdx.x; j < c; j += blockDim.x) {
      const int64_t q = j == threadIdx.x ? my_q : need[j];
      const int64_t v = j < kAppendThreads ? sh.victims[j] : victims[j];
      slot_mapping[q] = v * block_size;
      pos[q] = 1;
    }
  }
  return KVCA_OK;
}

template <typename MetaT>
__global__ void __launch_bounds__(kAppendThreads)
    append_step_kernel(MetaT* meta, int64_t n, int64_t* search_start, int64_t* l2p,
                       int64_t n_logical, int64_t* p2l, const int64_t* need, int64_t c,
                       int64_t* cur_block, int64_t* cur_logical, int64_t* pos, int64_t seqs,
                       int64_t block_size, int64_t* next_logical, int order, bool aligned,
                       int64_t* victims, int64_t* slot_mapping, int64_t* status) {
  __shared__ AppendShared<MetaT> sh;
  append_step_body<MetaT>(meta, n, search_start, l2p, n_logical, p2l, need, c, cur_block,
                          cur_logical, pos, seqs, block_size, next_logical, order, aligned,
                          victims, slot_mapping, status, sh);
}

// Per-sequence state (block, logical id, position) of up to kAppendSmemSeqs
// sequences, and up to kAppendSmemNeed need entries, live in shared memory
// for the whole launch: a step's dependent chain is then l2p of the full
// blocks -> metadata tile -> p2l / full-block words, three global round
// trips instead of five.
constexpr int64_t kAppendSmemSeqs = 4096;
constexpr int64_t kAppendSmemNeed = 4096;
constexpr size_t kAppendSmemBytes = (3 * kAppendSmemSeqs + kAppendSmemNeed) * sizeof(int64_t);
// The slot table itself is mirrored in shared memory after that state when
// both fit in kAppendDynMax bytes (a 65,536-slot 8-bit table is 64 KiB): it
// is read once per launch, every pop scans the copy, and every metadata
// write goes to both, so a step's chain loses the round trip of the pop's
// table reads (B200, decode mix with one KV head and a 65,536-block pool:
// the 16-step booking launch takes 84 us without the copy).
constexpr size_t kAppendDynMax = 200 * 1024;
#ifndef KVCA_APPEND_MIRROR
#define KVCA_APPEND_MIRROR 1
#endif
constexpr bool kAppendMirror = KVCA_APPEND_MIRROR != 0;

// num_steps steps in a row in one CTA: step s takes need[off[s]..off[s+1]),
// writes its victims to victims[off[s]..] and its slot_mapping to
// slot_mapping[s * seqs..], exactly as num_steps append_step launches would.
// The offsets are checked first (non-decreasing, at most seqs per step,
// within [0, num_need]); an error at step s leaves steps 0..s-1 done and
// stops there.  Steps after the first read the state the previous one wrote
// (same CTA, ordered by a block barrier).
// Minimum resident CTAs per SM the booking kernel is compiled for (a build
// knob for sweeps).  At 4 (64 registers) its CTA fits beside a pair-kernel
// CTA on one SM; B200, decode mix with the full pool: 8 KV heads 24.46
// against 24.65 us per step (one-launch cycles 24.64 against 27.03), but one
// KV head 5.11 against 4.62, where the slower booking shows; 1 is kept.
#ifndef KVCA_APPEND_MIN_CTAS
#define KVCA_APPEND_MIN_CTAS 1
#endif
template <typename MetaT>
__global__ void __launch_bounds__(kAppendThreads, KVCA_APPEND_MIN_CTAS)
    append_steps_kernel(MetaT* meta, int64_t n, int64_t* search_start, int64_t* l2p,
                        int64_t n_logical, int64_t* p2l, const int64_t* need,
                        const int64_t* need_offsets, int64_t num_need, int64_t num_steps,
                        int64_t* cur_block, int64_t* cur_logical, int64_t* pos, int64_t seqs,
                        int64_t block_size, int64_t* next_logical, int order, bool aligned,
                        int64_t* victims, int64_t* slot_mapping, int64_t* status, bool staged,
                        int64_t mirror_off) {
  __shared__ AppendShared<MetaT> sh;
  __shared__ int64_t off[kAppendMaxSteps + 1];
  // staged: block | logical id | position (seqs each), need entries; then,
  // from byte mirror_off (16-byte aligned; -1: none), the table's copy
  extern __shared__ __align__(16) int64_t dyn[];
  MetaT* mirror = mirror_off >= 0 ? reinterpret_cast<MetaT*>(reinterpret_cast<char*>(dyn) + mirror_off) : nullptr;
  if (mirror != nullptr) {  // issued first: its loads overlap the offset checks
    const int64_t nvec = (n + Meta<MetaT>::kSlotsPerVec - 1) / Meta<MetaT>::kSlotsPerVec;
    constexpr int kBatch = 8;  // vectors in flight per thread
    for (int64_t v0 = threadIdx.x; v0 < nvec; v0 += kBatch * static_cast<int64_t>(blockDim.x)) {
      MetaVec<MetaT> m[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int64_t v = v0 + u * static_cast<int64_t>(blockDim.x);
        if (v < nvec) load_meta_vec(meta, n, v, aligned, m[u]);
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int64_t v = v0 + u * static_cast<int64_t>(blockDim.x);
        if (v < nvec) store_mirror_vec(mirror, v, m[u]);
      }
    }
  }
  bool bad = false;
  for (int64_t s = threadIdx.x; s <= num_steps; s += blockDim.x) {
    const int64_t o = need_offsets[s];
    off[s] = o;
    if (o < 0 || o > num_need) {
      bad = true;
      sh.bad_value = o;
    }
  }
  __syncthreads();
  for (int64_t s = threadIdx.x; s < num_steps; s += blockDim.x) {
    const int64_t c = off[s + 1] - off[s];
    if (c < 0 || c > seqs) {
      bad = true;
      sh.bad_value = off[s + 1];
    }
  }
  if (__syncthreads_or(bad)) {
    if (threadIdx.x == 0) report(status, KVCA_ERR_BAD_INDEX, sh.bad_value);
    return;
  }
  int64_t* cb = cur_block;
  int64_t* cl = cur_logical;
  int64_t* ps = pos;
  const int64_t* nd = need;
  int64_t nd_base = 0;
  if (staged) {  // seqs <= kAppendSmemSeqs: the launch sized dyn for it
    cb = dyn;
    cl = dyn + seqs;
    ps = dyn + 2 * seqs;
    for (int64_t q = threadIdx.x; q < seqs; q += blockDim.x) {
      cb[q] = cur_block[q];
      cl[q] = cur_logical[q];
      ps[q] = pos[q];
    }
    const int64_t total = off[num_steps] - off[0];
    if (total <= kAppendSmemNeed) {
      int64_t* sn = dyn + 3 * seqs;
      for (int64_t j = threadIdx.x; j < total; j += blockDim.x) sn[j] = need[off[0] + j];
      nd = sn;
      nd_base = off[0];
    }
    __syncthreads();
  }
  for (int64_t s = 0; s < num_steps; ++s) {
    const int64_t o = off[s];
    const int rc = append_step_body<MetaT>(meta, n, search_start, l2p, n_logical, p2l,
                                           nd + (o - nd_base), off[s + 1] - o, cb, cl, ps, seqs,
                                           block_size, next_logical, order, aligned, victims + o,
                                           slot_mapping + s * seqs, status, sh, mirror);
    __syncthreads();
    if (rc != KVCA_OK) break;  // uniform across the CTA
  }
  if (staged) {
    for (int64_t q = threadIdx.x; q < seqs; q += blockDim.x) {
      cur_block[q] = cb[q];
      cur_logical[q] = cl[q];
      pos[q] = ps[q];
    }
  }
}

// ---------------------------------------------------------------------------
// Device-resident block store: the metadata half of a load / save after the
// plan, with no host round trip in between
// ---------------------------------------------------------------------------
//
// The store is the in-memory backend's (adapter.py:679-833) with its storage
// on this GPU: row l of `storage` holds logical block l, present[l] != 0 once
// it was saved.  A fused load runs plan_load, then store_load_finish, then
// the spill copy (actual[evict_slots] -> storage[evict_ids]) and the fill
// copy (storage[miss_ids] -> actual[load_slots]); a fused save runs
// plan_save, store_save_finish, the spill copy and the data scatter.  The
// finish kernels read the plan's counts from device memory.

// Spill preparation: among repeated evicted ids only the last occurrence
// keeps its slot (the others get -1, so the spill copy skips them and leaves
// the payload index_copy_ applied in order leaves), and every evicted id is
// marked present.  `scratch` (one int per logical id) is zero on entry and
// left zero.  Ends with a barrier.
__device__ void store_spill_prepare(const int64_t* evict_ids, int64_t* evict_slots, int64_t ne,
                                    int32_t* scratch, uint8_t* present) {
  for (int64_t j = threadIdx.x; j < ne; j += blockDim.x)
    atomicMax(scratch + evict_ids[j], static_cast<int32_t>(j + 1));
  __syncthreads();
  for (int64_t j = threadIdx.x; j < ne; j += blockDim.x)
    if (__ldcg(scratch + evict_ids[j]) != static_cast<int32_t>(j + 1)) evict_slots[j] = -1;
  __syncthreads();
  for (int64_t j = threadIdx.x; j < ne; j += blockDim.x) {
    scratch[evict_ids[j]] = 0;
    present[evict_ids[j]] = 1;
  }
  __syncthreads();
}

// After plan_load: the per-victim rows of the exchange, the backend's
// presence check of the misses (adapter.py:801-806) and the commit.
//   xslot[j]     = victims[j] for every miss j (the slot spilled and filled);
//   spill_to[j]  = the victim's previous logical id when it is evicted and j
//                  is the last victim evicting that id (index_copy_ applied in
//                  order keeps the last payload), else -1;
//   fill_from[j] = miss_ids[j] when every miss is present in the store.
// Evicted ids are marked present first, as the backend's save precedes its
// load.  A miss that is also spilled by this call must be filled after the
// spill: counts[7] (the gate) is set and the fill moves to a second launch.
// A missing block sets counts[3..4] = KVCA_ERR_BLOCK_NOT_FOUND, id; the
// spill still runs, nothing is filled or committed, as when the backend
// raises.  `scratch` (one int per logical id) is zero on entry and left zero.
// Nothing runs when the plan failed.
struct FinishShared {
  int bad;
  int missing;
  int conflict;
  long long missing_id;
};

template <typename MetaT>
__device__ void store_load_finish_body(int64_t* l2p, int64_t n_logical, int64_t* p2l, MetaT* meta, int64_t n,
                                       int64_t* counts, const int64_t* hit_slots, const int64_t* hit_pins,
                                       const MetaT* hit_usage, const int64_t* miss_ids,
                                       const int64_t* victims, const int64_t* evict_ids, int32_t* scratch,
                                       uint8_t* present, int64_t* xslot, int64_t* spill_to,
                                       int64_t* fill_from, int64_t* status, FinishShared& fs) {
  int& bad = fs.bad;
  int& missing = fs.missing;
  int& conflict = fs.conflict;
  long long& missing_id = fs.missing_id;
  if (counts[3] != 0) return;  // written by the plan (an earlier launch, or before a barrier): uniform
  const int64_t nh = counts[0], nm = counts[1], ne = counts[2];
  if (threadIdx.x == 0) bad = missing = conflict = 0;
  for (int64_t j = threadIdx.x; j < nm; j += blockDim.x) {
    const int64_t prev = p2l[victims[j]];
    const bool ev = prev >= 0 && prev != miss_ids[j];
    spill_to[j] = ev ? prev : -1;
    xslot[j] = victims[j];
    if (ev) atomicMax(scratch + prev, static_cast<int32_t>(j + 1));
  }
  __syncthreads();
  for (int64_t j = threadIdx.x; j < nm; j += blockDim.x) {
    const int64_t sp = spill_to[j];
    if (sp >= 0 && __ldcg(scratch + sp) != static_cast<int32_t>(j + 1)) spill_to[j] = -1;
    if (__ldcg(scratch + miss_ids[j]) != 0) conflict = 1;
  }
  __syncthreads();
  for (int64_t j = threadIdx.x; j < nm; j += blockDim.x) {
    const int64_t prev = p2l[victims[j]];
    if (prev >= 0 && prev != miss_ids[j]) {
      scratch[prev] = 0;
      present[prev] = 1;
    }
  }
  __syncthreads();
  for (int64_t j = threadIdx.x; j < nm; j += blockDim.x)
    if (present[miss_ids[j]] == 0 && atomicCAS(&missing, 0, 1) == 0) missing_id = miss_ids[j];
  __syncthreads();
  if (missing) {
    if (threadIdx.x == 0) {
      counts[3] = KVCA_ERR_BLOCK_NOT_FOUND;
      counts[4] = missing_id;
    }
    return;
  }
  for (int64_t j = threadIdx.x; j < nm; j += blockDim.x) fill_from[j] = miss_ids[j];
  if (threadIdx.x == 0) counts[7] = conflict;
  commit_load_body<MetaT>(l2p, n_logical, p2l, meta, n, evict_ids, ne, miss_ids, victims, nm,
                          hit_slots, hit_pins, hit_usage, nh, nullptr, status, &bad);
}

template <typename MetaT>
__global__ void __launch_bounds__(1024)
    store_load_finish_kernel(int64_t* l2p, int64_t n_logical, int64_t* p2l, MetaT* meta, int64_t n,
                             int64_t* counts, const int64_t* hit_slots, const int64_t* hit_pins,
                             const MetaT* hit_usage, const int64_t* miss_ids,
                             const int64_t* victims, const int64_t* evict_ids, int32_t* scratch,
                             uint8_t* present, int64_t* xslot, int64_t* spill_to,
                             int64_t* fill_from, int64_t* status) {
  __shared__ FinishShared fs;
  store_load_finish_body<MetaT>(l2p, n_logical, p2l, meta, n, counts, hit_slots, hit_pins, hit_usage, miss_ids,
                                victims, evict_ids, scratch, present, xslot, spill_to, fill_from, status, fs);
}

// After plan_save: spill preparation and the commit.  Nothing runs when the
// plan failed.
template <typename MetaT>
__device__ void store_save_finish_body(int64_t* l2p, int64_t n_logical, int64_t* p2l, MetaT* meta, int64_t n,
                                       int64_t* counts, const int64_t* ids, int64_t k,
                                       const int64_t* selected, const MetaT* final_pins,
                                       const MetaT* final_usage, const int64_t* evict_ids,
                                       int64_t* evict_slots, int32_t* scratch, uint8_t* present,
                                       int64_t* status, FinishShared& fs) {
  if (counts[3] != 0) return;
  const int64_t ne = counts[2];
  if (threadIdx.x == 0) fs.bad = 0;
  store_spill_prepare(evict_ids, evict_slots, ne, scratch, present);
  commit_save_body<MetaT>(l2p, n_logical, p2l, meta, n, evict_ids, ne, ids, selected, final_pins,
                          final_usage, k, status, &fs.bad);
}

template <typename MetaT>
__global__ void __launch_bounds__(1024)
    store_save_finish_kernel(int64_t* l2p, int64_t n_logical, int64_t* p2l, MetaT* meta, int64_t n,
                             int64_t* counts, const int64_t* ids, int64_t k,
                             const int64_t* selected, const MetaT* final_pins,
                             const MetaT* final_usage, const int64_t* evict_ids,
                             int64_t* evict_slots, int32_t* scratch, uint8_t* present,
                             int64_t* status) {
  __shared__ FinishShared fs;
  store_save_finish_body<MetaT>(l2p, n_logical, p2l, meta, n, counts, ids, k, selected, final_pins, final_usage,
                                evict_ids, evict_slots, scratch, present, status, fs);
}

// ---------------------------------------------------------------------------
// Small device-store calls in one launch
// ---------------------------------------------------------------------------
//
// A load or save whose rows total at most a few hundred KiB (an adapter call
// of tens of blocks) spends its time in launches, not in moving bytes.  Then
// one CTA runs the whole call: plan, finish (spill preparation, presence
// check, commit) and the row copies, each phase behind a block barrier, with
// the same results as the multi-launch sequence: spill rows are read before
// any fill or data row is written (the exchange's gate is the barrier).

// Row j: dst[dst_idx[j]] = src[src_idx[j]] (a null index array means row j
// itself), rows with a negative index skipped; one warp per row, vectors of
// `vec` bytes (the widest every address and stride allows).  Plain loads and
// stores, so either side may be pinned host memory.
template <typename V>
__device__ void copy_rows_cta_typed(uint64_t dst, int64_t dst_stride, const int64_t* dst_idx, uint64_t src,
                                    int64_t src_stride, const int64_t* src_idx, int64_t rows, int64_t row_bytes) {
  const int lane = threadIdx.x & 31;
  const int64_t nv = row_bytes / static_cast<int64_t>(sizeof(V));
  for (int64_t j = threadIdx.x >> 5; j < rows; j += blockDim.x >> 5) {
    const int64_t di = dst_idx != nullptr ? dst_idx[j] : j;
    const int64_t si = src_idx != nullptr ? src_idx[j] : j;
    if (di < 0 || si < 0) continue;
    const V* s = reinterpret_cast<const V*>(src + si * src_stride);
    V* d = reinterpret_cast<V*>(dst + di * dst_stride);
    for (int64_t v = lane; v < nv; v += 32) d[v] = s[v];
  }
}

__device__ void copy_rows_cta(uint64_t dst, int64_t dst_stride, const int64_t* dst_idx, uint64_t src,
                              int64_t src_stride, const int64_t* src_idx, int64_t rows, int64_t row_bytes,
                              int vec) {
  switch (vec) {
    case 16: copy_rows_cta_typed<uint4>(dst, dst_stride, dst_idx, src, src_stride, src_idx, rows, row_bytes); break;
    case 8: copy_rows_cta_typed<uint2>(dst, dst_stride, dst_idx, src, src_stride, src_idx, rows, row_bytes); break;
    case 4: copy_rows_cta_typed<unsigned>(dst, dst_stride, dst_idx, src, src_stride, src_idx, rows, row_bytes); break;
    case 2:
      copy_rows_cta_typed<unsigned short>(dst, dst_stride, dst_idx, src, src_stride, src_idx, rows, row_bytes);
      break;
    default:
      copy_rows_cta_typed<unsigned char>(dst, dst_stride, dst_idx, src, src_stride, src_idx, rows, row_bytes);
  }
}

// The slot rows and store rows of a small call.
struct StoreRows {
  uint64_t actual;
  int64_t actual_stride;
  uint64_t storage;
  int64_t storage_stride;
  uint64_t data;  // save: the caller's block_data rows
  int64_t row_bytes;
  int vec;
};

// work as in launch_store_load_meta (9 x k int64): hit_slots, hit_pins,
// miss_ids, victims, evict_ids, evict_slots, xslot, spill_to, fill_from.
// The last action of a one-launch store call made for a session: the
// call's 8 counts and then its sequence number go to pinned host memory, so
// the host learns that the call is done (and its outcome) by reading host
// memory instead of copying the counts and synchronising the stream.  The
// block barrier orders every thread's writes of the call before thread 0's
// system-scope fence and the sequence store.
__device__ __forceinline__ void signal_host(const int64_t* counts, int64_t* host_counts, int64_t seq) {
  if (host_counts == nullptr) return;
  __syncthreads();
  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) host_counts[i] = counts[i];
    __threadfence_system();
    *reinterpret_cast<volatile int64_t*>(host_counts + 8) = seq;
  }
}

template <typename MetaT>
__global__ void __launch_bounds__(1024)
    store_load_small_kernel(int64_t* l2p, int64_t n_logical, int64_t* p2l, MetaT* meta, int64_t n,
                            int64_t* search_start, const int64_t* ids, int64_t k, uint32_t* bitmap, int order,
                            bool aligned, int32_t* scratch, uint8_t* present, int64_t* work, MetaT* hit_usage,
                            int64_t* result, int64_t* counts, int64_t* status, StoreRows rows,
                            int64_t* host_counts, int64_t seq) {
  __shared__ PlanShared<MetaT> sh;
  __shared__ FinishShared fs;
  int64_t* hit_slots = work;
  int64_t* hit_pins = work + k;
  int64_t* miss_ids = work + 2 * k;
  int64_t* victims = work + 3 * k;
  int64_t* evict_ids = work + 4 * k;
  int64_t* evict_slots = work + 5 * k;
  int64_t* xslot = work + 6 * k;
  int64_t* spill_to = work + 7 * k;
  int64_t* fill_from = work + 8 * k;
  if (threadIdx.x == 0) {
    counts[7] = 0;
    fs.bad = 0;
  }
  plan_load_body<MetaT>(l2p, n_logical, p2l, meta, n, search_start, ids, k, bitmap, order, aligned, result,
                        hit_slots, hit_pins, hit_usage, miss_ids, victims, evict_ids, evict_slots, counts, status,
                        sh);
  __syncthreads();
  if (counts[1] == 0 && counts[3] == 0) {  // every request hit: commit the hits' pins and usage, no rows move
    const int64_t nh = counts[0];
    if (all_in_range(hit_slots, nh, n, status, &fs.bad))
      for (int64_t i = threadIdx.x; i < nh; i += blockDim.x)
        meta[hit_slots[i]] = Meta<MetaT>::pack(hit_pins[i], hit_usage[i]);
    signal_host(counts, host_counts, seq);
    return;
  }
  for (int64_t i = threadIdx.x; i < 3 * k; i += blockDim.x) xslot[i] = -1;  // xslot, spill_to, fill_from
  __syncthreads();
  store_load_finish_body<MetaT>(l2p, n_logical, p2l, meta, n, counts, hit_slots, hit_pins, hit_usage, miss_ids,
                                victims, evict_ids, scratch, present, xslot, spill_to, fill_from, status, fs);
  __syncthreads();
  // spill the victims' old rows, then fill them
  copy_rows_cta(rows.storage, rows.storage_stride, spill_to, rows.actual, rows.actual_stride, xslot, k,
                rows.row_bytes, rows.vec);
  __syncthreads();
  copy_rows_cta(rows.actual, rows.actual_stride, xslot, rows.storage, rows.storage_stride, fill_from, k,
                rows.row_bytes, rows.vec);
  signal_host(counts, host_counts, seq);
}

// work as in launch_store_save_meta (5 x k int64): selected, allocated,
// evict_ids, evict_slots, move_slots; work_meta: final pins, final usage.
template <typename MetaT>
__global__ void __launch_bounds__(1024)
    store_save_small_kernel(int64_t* l2p, int64_t n_logical, int64_t* p2l, MetaT* meta, int64_t n,
                            int64_t* search_start, const int64_t* ids, int64_t k, uint32_t* bitmap, int order,
                            bool aligned, int32_t* scratch, uint8_t* present, int64_t* work, MetaT* work_meta,
                            int64_t* counts, int64_t* status, StoreRows rows, int64_t* host_counts, int64_t seq) {
  __shared__ PlanShared<MetaT> sh;
  __shared__ FinishShared fs;
  int64_t* selected = work;
  int64_t* allocated = work + k;
  int64_t* evict_ids = work + 2 * k;
  int64_t* evict_slots = work + 3 * k;
  int64_t* move_slots = work + 4 * k;
  MetaT* final_pins = work_meta;
  MetaT* final_usage = work_meta + k;
  for (int64_t i = threadIdx.x; i < 3 * k; i += blockDim.x) evict_ids[i] = -1;  // evict_ids, evict_slots, move_slots
  __syncthreads();
  plan_save_body<MetaT>(l2p, n_logical, p2l, meta, n, search_start, ids, k, bitmap, order, aligned, selected,
                        move_slots, final_pins, final_usage, allocated, evict_ids, evict_slots, counts, status, sh);
  __syncthreads();
  store_save_finish_body<MetaT>(l2p, n_logical, p2l, meta, n, counts, ids, k, selected, final_pins, final_usage,
                                evict_ids, evict_slots, scratch, present, status, fs);
  __syncthreads();
  // spill the evicted rows, then scatter the data rows
  copy_rows_cta(rows.storage, rows.storage_stride, evict_ids, rows.actual, rows.actual_stride, evict_slots, k,
                rows.row_bytes, rows.vec);
  __syncthreads();
  copy_rows_cta(rows.actual, rows.actual_stride, move_slots, rows.data, rows.row_bytes, nullptr, k, rows.row_bytes,
                rows.vec);
  signal_host(counts, host_counts, seq);
}

// ---------------------------------------------------------------------------
// Row mover
// ---------------------------------------------------------------------------

struct MoveParams {
  PagedSide src_paged;
  PagedSide dst_paged;
  ChunkSide src_chunk;
  ChunkSide dst_chunk;
  int64_t num_planes;
  int64_t num_rows;
  int64_t row_vecs;
  int64_t seg_vecs;      // vectors per work item: rows longer than this are split
  int64_t segs_per_row;  // ceil(row_vecs / seg_vecs)
  int tpr_log2;  // threads per work item = 1 << tpr_log2 (a power of two <= 32)
  int32_t flags;
  int64_t* status;
  const int64_t* gate;  // non-null: the launch moves nothing unless *gate != 0
  int rows_per_batch;   // move_rows_stream_kernel: rows a warp moves per batch
};

template <typename V>
__device__ __forceinline__ V ld_stream(const V* p) {
  return __ldcs(p);
}
template <>
__device__ __forceinline__ uint4 ld_stream<uint4>(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

template <typename V>
__device__ __forceinline__ void st_stream(V* p, const V& v) {
  __stcs(p, v);
}

// Offset of row r (without the plane term) on a paged side, or -1 when the
// row is skipped.  Reports ids outside the table.
__device__ __forceinline__ int64_t paged_row_offset(const PagedSide& side, int64_t r,
                                                    int32_t flags, int64_t* status, bool lead) {
  const int64_t idx = side.index != nullptr ? side.index[r] : r;
  if (idx < 0) {
    if (!(flags & KVCA_FLAG_SKIP_NEGATIVE) && lead) report(status, KVCA_ERR_BAD_INDEX, idx);
    return -1;
  }
  int64_t blk = idx;
  int64_t off = 0;
  if (side.block_size != 1) {
    blk = idx / side.block_size;
    off = idx - blk * side.block_size;
  }
  if (blk >= side.num_blocks) {
    if (lead) report(status, KVCA_ERR_BAD_INDEX, idx);
    return -1;
  }
  return blk * side.block_stride + off * side.row_stride;
}

__device__ __forceinline__ int64_t chunk_row_offset(const ChunkSide& side, int64_t r) {
  const int64_t c = r / side.rows_per_chunk;
  return c * side.chunk_stride + (r - c * side.rows_per_chunk) * side.row_stride;
}

constexpr int kMoverThreads = 512;
// Moves over the host link saturate it with a few CTAs; a full grid only
// adds contention (B200, random 64 KiB rows: exchange 80 GB/s at 8-16 CTAs,
// 79 at 32, 73 at 148; one way 52 vs 51 GB/s; 256 B rows device->host 47 at
// 16 CTAs vs 38 at 148).
constexpr int kHostMoverCtas = 16;
constexpr int kMoverUnroll = 8;
constexpr int64_t kMoverSegmentBytes = 16384;

// Work item g = (r * num_planes + p) * segs_per_row + segment: a row of one
// plane, split into segments of at most seg_vecs vectors so that every group
// of lanes gets the same number of bytes however long the rows are.  Each
// group of 2^tpr_log2 lanes takes one contiguous range of items, so
// consecutive items share a row: the row's index is loaded and its offset
// computed once per row, not once per plane or segment.  Each lane keeps
// kMoverUnroll vectors in flight.
// kHost: one side is pinned, mapped host memory reached over the host link;
// rows move with plain loads and stores there (no non-coherent cache path).
// The movers' bodies take the CTA's index and the CTA count of the work
// split (blockIdx.x and gridDim.x for a launch of their own), so that one
// launch can also split its CTAs between two moves (move_pair_kernel).
// kEarly (pair mover, inputs ready): the body itself waits for the launch's
// programmatic predecessor (grid_dependency_wait) after its index loads and
// before any load of paged rows or any store; loads of a chunk source may
// come before it too (stream and small-row bodies).
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <bool kSrcPaged, bool kDstPaged, typename V, bool kHost, bool kEarly = false, int kUnroll = kMoverUnroll>
__device__ __forceinline__ void move_rows_body(const MoveParams& p, int64_t cta, int64_t ctas) {
  if (p.gate != nullptr && *p.gate == 0) return;
  const int tpr = 1 << p.tpr_log2;
  const int64_t gtid = cta * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int lane = static_cast<int>(gtid & (tpr - 1));
  const int64_t group = gtid >> p.tpr_log2;
  const int64_t num_groups = (ctas * blockDim.x) >> p.tpr_log2;
  const int64_t planes = p.num_planes;
  const int64_t segs = p.segs_per_row;
  const int64_t per_row = planes * segs;
  const int64_t items = per_row * p.num_rows;
  const int64_t per = items / num_groups;
  const int64_t rem = items - per * num_groups;
  const int64_t begin = group * per + (group < rem ? group : rem);
  const int64_t end = begin + per + (group < rem ? 1 : 0);
  if (begin >= end) return;

  int64_t r = begin / per_row;
  int64_t pl = (begin - r * per_row) / segs;
  int64_t sg = begin - r * per_row - pl * segs;
  int64_t src_row = 0;
  int64_t dst_row = 0;
  bool row_ready = false;
  const bool lead = lane == 0;
  const int64_t row_vecs = p.row_vecs;
  const int64_t seg_vecs = p.seg_vecs;

  for (int64_t g = begin; g < end; ++g) {
    if (!row_ready) {
      row_ready = true;
      src_row = kSrcPaged ? paged_row_offset(p.src_paged, r, p.flags, p.status, lead)
                          : chunk_row_offset(p.src_chunk, r);
      dst_row = kDstPaged ? paged_row_offset(p.dst_paged, r, p.flags, p.status, lead)
                          : chunk_row_offset(p.dst_chunk, r);
    }
    if constexpr (kEarly) grid_dependency_wait();
    if (src_row >= 0 && dst_row >= 0) {
      const V* src = reinterpret_cast<const V*>(
          kSrcPaged ? p.src_paged.planes[pl] + src_row
                    : p.src_chunk.base + src_row + pl * p.src_chunk.plane_stride);
      V* dst = reinterpret_cast<V*>(kDstPaged
                                        ? p.dst_paged.planes[pl] + dst_row
                                        : p.dst_chunk.base + dst_row + pl * p.dst_chunk.plane_stride);
      const int64_t v_begin = sg * seg_vecs;
      const int64_t v_end = v_begin + seg_vecs < row_vecs ? v_begin + seg_vecs : row_vecs;
      for (int64_t b = v_begin + lane; b < v_end; b += static_cast<int64_t>(tpr) * kUnroll) {
        V buf[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int64_t i = b + static_cast<int64_t>(u) * tpr;
          if (i < v_end) buf[u] = kHost ? src[i] : ld_stream(src + i);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int64_t i = b + static_cast<int64_t>(u) * tpr;
          if (i < v_end) {
            if (kHost)
              dst[i] = buf[u];
            else
              st_stream(dst + i, buf[u]);
          }
        }
      }
    }
    if (++sg == segs) {
      sg = 0;
      if (++pl == planes) {
        pl = 0;
        ++r;
        row_ready = false;
      }
    }
  }
}

// Entry of a kernel launched as a programmatic dependent of the kernel
// before it on its stream (launch_dependent): its CTAs may be dispatched
// while that kernel drains, wait for it (griddepcontrol.wait: the grid
// complete, its writes visible) before touching memory, and then let the
// next launch start dispatching.  Without a programmatic predecessor the
// wait returns at once.  Only the pair mover launches this way: its
// consecutive launches are short and latency-bound (a decode step), while
// early-resident CTAs of large moves took the SMs that a concurrent kernel
// on another stream needed (decode mix, 8 KV heads: 39.6 against 29.6 us
// per step, the cycle booking starved).
__device__ __forceinline__ void dependent_launch_entry() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <bool kSrcPaged, bool kDstPaged, typename V, bool kHost>
__global__ void __launch_bounds__(kMoverThreads) move_rows_kernel(const __grid_constant__ MoveParams p) {
  move_rows_body<kSrcPaged, kDstPaged, V, kHost>(p, blockIdx.x, gridDim.x);
}

// Rows of at most kSmallRowMaxVecs 16-byte vectors (256 bytes).
constexpr int64_t kSmallRowMaxVecs = 16;
// In the pair kernel, rows of 97 to 128 vectors (1.5 to 2 KiB) take the
// short-row body with a whole warp per row, 4 vectors per lane and
// kMediumRows rows per warp and iteration: a decode step's token scatter
// with 8 KV heads (2 KiB rows) keeps 8 vectors per lane in flight over every
// row of its short launch (B200, a step's scatter with the next step's spill
// gather, 134 MB: 24.4 us per step against 28.2 on the SIMT body; 4 rows per
// iteration: 25.8 us).  Moves of their own keep the SIMT body for these rows
// (random 2 KiB token rows, 1 GiB: 5.75 / 5.88 TB/s gather / scatter
// against 5.65 / 5.63 on this body).
constexpr int kMediumRows = 2;
constexpr int64_t kMediumRowMinVecs = 96;
constexpr int64_t kMediumRowMaxVecs = 128;


// Offset of slot id idx on a paged side (shift = log2 of the block size when
// that is a power of two, else -1), or -1 when the row is skipped; the same
// checks and reports as paged_row_offset.
__device__ __forceinline__ int64_t paged_slot_offset(const PagedSide& side, int64_t idx, int shift,
                                                     int32_t flags, int64_t* status, bool lead) {
  if (idx < 0) {
    if (!(flags & KVCA_FLAG_SKIP_NEGATIVE) && lead) report(status, KVCA_ERR_BAD_INDEX, idx);
    return -1;
  }
  int64_t blk;
  int64_t off;
  if (shift >= 0) {
    blk = idx >> shift;
    off = idx & ((int64_t{1} << shift) - 1);
  } else {
    blk = idx / side.block_size;
    off = idx - blk * side.block_size;
  }
  if (blk >= side.num_blocks) {
    if (lead) report(status, KVCA_ERR_BAD_INDEX, idx);
    return -1;
  }
  return blk * side.block_stride + off * side.row_stride;
}

__device__ __forceinline__ int pow2_shift(int64_t v) {
  return v > 0 && (v & (v - 1)) == 0 ? __ffsll(static_cast<long long>(v)) - 1 : -1;
}

// Small rows (at most 256 bytes) of 16-byte vectors, several rows per lane
// group and iteration: 2^k <= 8 lanes share a row, kVpl vectors each, so
// that every load or store instruction covers whole 128-byte lines of its
// rows, and each group moves kRows rows per iteration (all loads, then all
// stores).  Work items in plane-major order, g = plane * num_rows + row: a
// group walks consecutive rows of one plane, which are consecutive rows of
// a chunk and, for slot mappings made from block tables, runs of
// consecutive rows of a block.  Every item loads its own index;
// power-of-two block sizes divide by shifting, and the chunk position
// advances by counting instead of dividing.  Same work items, index checks
// and gate as move_rows_kernel; rows are never split into segments.
// Used for rows under 128 bytes (the stream mover covers 128 B to 1.5 KiB).
// B200, random 256-byte token rows over 64 planes: gather / scatter
// 5.7 / 5.7 TB/s, against 4.9 / 4.7 for the SIMT mover's shape (four lanes
// of four vectors, one row at a time: every instruction touches half-lines
// of eight rows).
template <bool kSrcPaged, bool kDstPaged, int kVpl, int kRows, bool kEarly = false>
__device__ __forceinline__ void move_short_rows_pm_body(const MoveParams& p, int64_t cta, int64_t ctas) {
  if (p.gate != nullptr && *p.gate == 0) return;
  const int tpr = 1 << p.tpr_log2;
  const int64_t gtid = cta * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int lane = static_cast<int>(gtid & (tpr - 1));
  const int64_t group = gtid >> p.tpr_log2;
  const int64_t num_groups = (ctas * blockDim.x) >> p.tpr_log2;
  const int64_t rows = p.num_rows;
  const int64_t items = p.num_planes * rows;
  const int64_t per = items / num_groups;
  const int64_t rem = items - per * num_groups;
  const int64_t begin = group * per + (group < rem ? group : rem);
  const int64_t end = begin + per + (group < rem ? 1 : 0);
  if (begin >= end) return;

  constexpr bool kChunk = !(kSrcPaged && kDstPaged);
  const ChunkSide& cs = kSrcPaged ? p.dst_chunk : p.src_chunk;  // the chunk side, when there is one
  int64_t pl = begin / rows;
  int64_t r = begin - pl * rows;
  int64_t c = 0;
  int64_t cr = 0;
  if (kChunk) {
    c = r / cs.rows_per_chunk;
    cr = r - c * cs.rows_per_chunk;
  }
  const int s_shift = kSrcPaged ? pow2_shift(p.src_paged.block_size) : 0;
  const int d_shift = kDstPaged ? pow2_shift(p.dst_paged.block_size) : 0;
  const bool lead = lane == 0;
  const int row_vecs = static_cast<int>(p.row_vecs);

  // Slot indices are loaded one iteration ahead, before the current rows'
  // loads, so that an iteration waits for its row loads only (the index and
  // the rows it names no longer form one chain).
  int64_t sidx[kRows];
  int64_t didx[kRows];
  {
    int64_t rr = r;
#pragma unroll
    for (int u = 0; u < kRows; ++u) {
      sidx[u] = 0;
      didx[u] = 0;
      if (begin + u < end) {
        if (kSrcPaged) sidx[u] = p.src_paged.index != nullptr ? p.src_paged.index[rr] : rr;
        if (kDstPaged) didx[u] = p.dst_paged.index != nullptr ? p.dst_paged.index[rr] : rr;
      }
      if (++rr == rows) rr = 0;
    }
  }

  for (int64_t g = begin; g < end; g += kRows) {
    int64_t plane[kRows];
    int64_t coff[kRows];
#pragma unroll
    for (int u = 0; u < kRows; ++u) {
      plane[u] = pl;
      coff[u] = kChunk ? c * cs.chunk_stride + cr * cs.row_stride + pl * cs.plane_stride : 0;
      if (++r == rows) {
        r = 0;
        ++pl;
        c = 0;
        cr = 0;
      } else if (kChunk && ++cr == cs.rows_per_chunk) {
        cr = 0;
        ++c;
      }
    }
    const uint4* src[kRows];
    uint4* dst[kRows];
#pragma unroll
    for (int u = 0; u < kRows; ++u) {
      src[u] = nullptr;
      dst[u] = nullptr;
      if (g + u < end) {
        const int64_t so = kSrcPaged ? paged_slot_offset(p.src_paged, sidx[u], s_shift, p.flags, p.status, lead)
                                     : coff[u];
        const int64_t dso = kDstPaged ? paged_slot_offset(p.dst_paged, didx[u], d_shift, p.flags, p.status, lead)
                                      : coff[u];
        if (so >= 0 && dso >= 0) {
          src[u] = reinterpret_cast<const uint4*>(kSrcPaged ? p.src_paged.planes[plane[u]] + so
                                                            : p.src_chunk.base + so);
          dst[u] = reinterpret_cast<uint4*>(kDstPaged ? p.dst_paged.planes[plane[u]] + dso
                                                      : p.dst_chunk.base + dso);
        }
      }
    }
    {  // the next iteration's indices: rows r, r + 1, ... of the position reached
      int64_t rr = r;
#pragma unroll
      for (int u = 0; u < kRows; ++u) {
        if (g + kRows + u < end) {
          if (kSrcPaged) sidx[u] = p.src_paged.index != nullptr ? p.src_paged.index[rr] : rr;
          if (kDstPaged) didx[u] = p.dst_paged.index != nullptr ? p.dst_paged.index[rr] : rr;
        }
        if (++rr == rows) rr = 0;
      }
    }
    uint4 buf[kRows][kVpl];
    if constexpr (kEarly && kSrcPaged) grid_dependency_wait();
#pragma unroll
    for (int u = 0; u < kRows; ++u)
#pragma unroll
      for (int j = 0; j < kVpl; ++j) {
        const int i = lane + j * tpr;
        if (src[u] != nullptr && i < row_vecs) buf[u][j] = ld_stream(src[u] + i);
      }
    if constexpr (kEarly && !kSrcPaged) grid_dependency_wait();
#pragma unroll
    for (int u = 0; u < kRows; ++u)
#pragma unroll
      for (int j = 0; j < kVpl; ++j) {
        const int i = lane + j * tpr;
        if (dst[u] != nullptr && i < row_vecs) st_stream(dst[u] + i, buf[u][j]);
      }
  }
}

template <bool kSrcPaged, bool kDstPaged, int kVpl, int kRows>
__global__ void __launch_bounds__(kMoverThreads) move_short_rows_pm_kernel(const __grid_constant__ MoveParams p) {
  move_short_rows_pm_body<kSrcPaged, kDstPaged, kVpl, kRows>(p, blockIdx.x, gridDim.x);
}

// Warp-cooperative mover for rows of 128 bytes to 1.5 KiB in 16-byte
// vectors: each warp takes a contiguous range of work items in plane-major
// order (consecutive rows of one plane) and moves them in batches of
// rows_per_batch rows.  Lane r computes the source and destination
// addresses of the batch's row r (one index load per row, coalesced across
// the warp), and the warp's 32 x kRowStreamSlots vector slots tile the
// batch's rows back to back: slot k of lane l is vector l + 32k of the
// batch, and takes its row's address from the lane that computed it by a
// shuffle.  Nearly every slot does useful work whatever the row length
// (9 slots per lane: 8 rows of 576 bytes or 4 of 1,152 fill all 288), so
// each lane keeps 9 vectors in flight and consecutive lanes cover
// consecutive bytes.  B200, token rows through a product-path gather /
// scatter: 576-byte rows under a block-table slot mapping 5.8 / 5.8 TB/s
// (5.3 / 5.4 with 32 lanes of 3 vectors, 2 rows per iteration), 1,152-byte
// rows 5.9 / 5.9 (5.6 / 5.6), random 128-byte rows 4.7 / 4.8 (3.7 / 3.7 with
// the small-row shape).  Above 1.5 KiB a batch holds one or two rows and
// the SIMT mover is as fast or faster (3 KiB rows: 5.6 against 6.0).
constexpr int kRowStreamThreads = 512;
constexpr int kRowStreamSlots = 9;

template <bool kSrcPaged, bool kDstPaged, bool kEarly = false>
__device__ __forceinline__ void move_rows_stream_body(const MoveParams& p, int64_t cta, int64_t ctas) {
  if (p.gate != nullptr && *p.gate == 0) return;
  const int lane = static_cast<int>(threadIdx.x & 31);
  const int64_t warp = (cta * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t num_warps = (ctas * blockDim.x) >> 5;
  const int64_t rows = p.num_rows;
  const int64_t items = p.num_planes * rows;
  const int64_t per = items / num_warps;
  const int64_t rem = items - per * num_warps;
  const int64_t begin = warp * per + (warp < rem ? warp : rem);
  const int64_t end = begin + per + (warp < rem ? 1 : 0);
  if (begin >= end) return;  // the whole warp

  const int rpb = p.rows_per_batch;
  const int rv = static_cast<int>(p.row_vecs);
  constexpr bool kChunk = !(kSrcPaged && kDstPaged);
  const ChunkSide& cs = kSrcPaged ? p.dst_chunk : p.src_chunk;  // the chunk side, when there is one
  const int s_shift = kSrcPaged ? pow2_shift(p.src_paged.block_size) : 0;
  const int d_shift = kDstPaged ? pow2_shift(p.dst_paged.block_size) : 0;

  // This lane's item (begin + lane), advanced by rpb per batch, and its
  // position in the chunk side; 32-bit (the launcher checks the row count).
  int pl = static_cast<int>((begin + lane) / rows);
  int r = static_cast<int>((begin + lane) - static_cast<int64_t>(pl) * rows);
  const int rows32 = static_cast<int>(rows);
  const int rpc = kChunk ? static_cast<int>(cs.rows_per_chunk) : 1;
  int c = r / rpc;
  int cr = r - c * rpc;
  const int qc = rpb / rpc;
  const int mc = rpb - qc * rpc;

  // Slot k of this lane is vector f = lane + 32k of a batch: row f / rv,
  // vector f % rv; successive slots step by 32 = q32 * rv + m32.
  const int row0 = lane / rv;
  const int vec0 = lane - row0 * rv;
  const int q32 = 32 / rv;
  const int m32 = 32 - q32 * rv;

  // The batch's slot indices are loaded one batch ahead, before the previous
  // batch's row loads, so that a batch waits for its row loads only, not for
  // an index load and then its row loads (random 128-byte rows: the index
  // latency took half of each batch).
  int64_t cur_s = 0;
  int64_t cur_d = 0;
  if (lane < (end - begin < rpb ? end - begin : rpb)) {
    if (kSrcPaged) cur_s = p.src_paged.index != nullptr ? p.src_paged.index[r] : r;
    if (kDstPaged) cur_d = p.dst_paged.index != nullptr ? p.dst_paged.index[r] : r;
  }
  for (int64_t g = begin; g < end; g += rpb) {
    const int nrows = end - g < rpb ? static_cast<int>(end - g) : rpb;
    uint64_t my_src = 0;
    uint64_t my_dst = 0;
    if (lane < nrows) {
      const int64_t coff = kChunk ? c * cs.chunk_stride + cr * cs.row_stride + pl * cs.plane_stride : 0;
      int64_t so = coff;
      int64_t dso = coff;
      if (kSrcPaged) so = paged_slot_offset(p.src_paged, cur_s, s_shift, p.flags, p.status, true);
      if (kDstPaged) dso = paged_slot_offset(p.dst_paged, cur_d, d_shift, p.flags, p.status, true);
      if (so >= 0 && dso >= 0) {
        my_src = kSrcPaged ? p.src_paged.planes[pl] + so : p.src_chunk.base + so;
        my_dst = kDstPaged ? p.dst_paged.planes[pl] + dso : p.dst_chunk.base + dso;
      }
    }
    r += rpb;
    cr += mc;
    c += qc;
    if (cr >= rpc) {
      cr -= rpc;
      ++c;
    }
    if (r >= rows32) {
      do {
        r -= rows32;
        ++pl;
      } while (r >= rows32);
      c = r / rpc;
      cr = r - c * rpc;
    }
    {  // the next batch's indices (its lane's row is now r of plane pl)
      const int64_t gn = g + rpb;
      if (gn < end && lane < (end - gn < rpb ? end - gn : rpb)) {
        if (kSrcPaged) cur_s = p.src_paged.index != nullptr ? p.src_paged.index[r] : r;
        if (kDstPaged) cur_d = p.dst_paged.index != nullptr ? p.dst_paged.index[r] : r;
      }
    }

    // my_src and my_dst are both set or both zero (a skipped row).
    uint4 buf[kRowStreamSlots];
    int row = row0;
    int vec = vec0;
    if constexpr (kEarly && kSrcPaged) grid_dependency_wait();
#pragma unroll
    for (int k = 0; k < kRowStreamSlots; ++k) {
      const uint64_t sb = __shfl_sync(0xffffffffu, my_src, row & 31);
      if (row < nrows && sb != 0) buf[k] = ld_stream(reinterpret_cast<const uint4*>(sb) + vec);
      vec += m32;
      row += q32;
      if (vec >= rv) {
        vec -= rv;
        ++row;
      }
    }
    if constexpr (kEarly && !kSrcPaged) grid_dependency_wait();
    row = row0;
    vec = vec0;
#pragma unroll
    for (int k = 0; k < kRowStreamSlots; ++k) {
      const uint64_t db = __shfl_sync(0xffffffffu, my_dst, row & 31);
      if (row < nrows && db != 0) st_stream(reinterpret_cast<uint4*>(db) + vec, buf[k]);
      vec += m32;
      row += q32;
      if (vec >= rv) {
        vec -= rv;
        ++row;
      }
    }
  }
}

template <bool kSrcPaged, bool kDstPaged>
__global__ void __launch_bounds__(kRowStreamThreads) move_rows_stream_kernel(const __grid_constant__ MoveParams p) {
  move_rows_stream_body<kSrcPaged, kDstPaged>(p, blockIdx.x, gridDim.x);
}

// Two independent moves in one launch: CTAs [0, split) run move a, the
// others move b, each with the body its rows take on their own (the bulk
// mover's rows take the SIMT body: one CTA shape for both).  For moves that
// are each too small to fill the GPU for long (a decode step's token scatter
// and the next step's spill gather), one launch instead of two saves a
// launch's latency, ramp and tail.  The two moves must not touch the same
// bytes.
// Vectors per lane and iteration of the pair kernel's SIMT body (a build
// knob for sweeps; B200, decode step pairs: 16 was slower than 8, 25.3 against
// 24.4 us per step with 8 KV heads and 7.8 against 4.7 with one).
// Rows of a multiple of kSplitVecs 16-byte vectors (the bulk mover's rows, in
// the pair kernel) as sub-rows of kSplitVecs vectors: a warp per sub-row, 4
// vectors per lane, two sub-rows per warp and iteration, so each lane keeps
// 8 vectors in flight as on the short-row body.  Work items g = (row *
// planes + plane) * sub-rows + sub-row: a warp walks the sub-rows of one
// row's plane (32 KiB of a decode step's victim block) before the next, and
// loads each row's index once.  A skipped or refused row leaves its
// destination as it was.
constexpr int64_t kSplitVecs = 128;

template <bool kSrcPaged, bool kDstPaged, bool kEarly>
__device__ __forceinline__ void move_split_rows_body(const MoveParams& p, int64_t cta, int64_t ctas) {
  if (p.gate != nullptr && *p.gate == 0) return;
  const int lane = static_cast<int>(threadIdx.x & 31);
  const int64_t warp = (cta * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t warps = (ctas * static_cast<int64_t>(blockDim.x)) >> 5;
  const int64_t subs = p.row_vecs / kSplitVecs;
  const int64_t planes = p.num_planes;
  const int64_t per_row = planes * subs;
  const int64_t items = per_row * p.num_rows;
  const int64_t per = items / warps;
  const int64_t rem = items - per * warps;
  const int64_t begin = warp * per + (warp < rem ? warp : rem);
  const int64_t end = begin + per + (warp < rem ? 1 : 0);
  if (begin >= end) return;
  int64_t r = begin / per_row;
  int64_t pl = (begin - r * per_row) / subs;
  int64_t j = begin - r * per_row - pl * subs;
  int64_t row_r = -1;
  int64_t src_row = 0;
  int64_t dst_row = 0;
  const bool lead = lane == 0;
  if constexpr (kEarly) grid_dependency_wait();
  for (int64_t g = begin; g < end; g += 2) {
    const uint4* src[2];
    uint4* dst[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      src[u] = nullptr;
      dst[u] = nullptr;
      if (g + u < end) {
        if (r != row_r) {
          row_r = r;
          src_row = kSrcPaged ? paged_row_offset(p.src_paged, r, p.flags, p.status, lead)
                              : chunk_row_offset(p.src_chunk, r);
          dst_row = kDstPaged ? paged_row_offset(p.dst_paged, r, p.flags, p.status, lead)
                              : chunk_row_offset(p.dst_chunk, r);
        }
        if (src_row >= 0 && dst_row >= 0) {
          const uint64_t sub = static_cast<uint64_t>(j) * kSplitVecs * 16;
          src[u] = reinterpret_cast<const uint4*>(
              (kSrcPaged ? p.src_paged.planes[pl] + src_row
                         : p.src_chunk.base + src_row + pl * p.src_chunk.plane_stride) + sub);
          dst[u] = reinterpret_cast<uint4*>(
              (kDstPaged ? p.dst_paged.planes[pl] + dst_row
                         : p.dst_chunk.base + dst_row + pl * p.dst_chunk.plane_stride) + sub);
        }
        if (++j == subs) {
          j = 0;
          if (++pl == planes) {
            pl = 0;
            ++r;
          }
        }
      }
    }
    uint4 buf[2][4];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int v = 0; v < 4; ++v)
        if (src[u] != nullptr) buf[u][v] = ld_stream(src[u] + lane + 32 * v);
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int v = 0; v < 4; ++v)
        if (dst[u] != nullptr) st_stream(dst[u] + lane + 32 * v, buf[u][v]);
  }
}

#ifndef KVCA_PAIR_SIMT_UNROLL
#define KVCA_PAIR_SIMT_UNROLL 8
#endif
constexpr int kPairSimtUnroll = KVCA_PAIR_SIMT_UNROLL;
// The pair kernel moves the bulk mover's rows as 2 KiB sub-rows (a build
// knob for sweeps; 0 keeps them on the SIMT body).  B200, decode step pairs
// replayed alone: 8 KV heads (32 KiB victim rows) 23.7 against 24.6 us per
// step; one KV head (4 KiB rows) 4.71 against 4.72.
#ifndef KVCA_PAIR_SPLIT_ROWS
#define KVCA_PAIR_SPLIT_ROWS 1
#endif
constexpr bool kPairSplitRows = KVCA_PAIR_SPLIT_ROWS != 0;

enum class MoverBody : int { kSimt = 0, kStream = 1, kSmall = 2, kMedium = 3, kSplit = 4 };

template <MoverBody kBody, bool kSrcPaged, bool kDstPaged, bool kEarly>
__device__ __forceinline__ void run_mover_body(const MoveParams& p, int64_t cta, int64_t ctas) {
  if constexpr (kBody == MoverBody::kStream)
    move_rows_stream_body<kSrcPaged, kDstPaged, kEarly>(p, cta, ctas);
  else if constexpr (kBody == MoverBody::kSmall)
    move_short_rows_pm_body<kSrcPaged, kDstPaged, 2, 4, kEarly>(p, cta, ctas);
  else if constexpr (kBody == MoverBody::kMedium)  // a warp per row of at most 128 vectors
    move_short_rows_pm_body<kSrcPaged, kDstPaged, 4, kMediumRows, kEarly>(p, cta, ctas);
  else if constexpr (kBody == MoverBody::kSplit)  // a warp per 2 KiB sub-row of longer rows
    move_split_rows_body<kSrcPaged, kDstPaged, kEarly>(p, cta, ctas);
  else
    move_rows_body<kSrcPaged, kDstPaged, uint4, false, kEarly, kPairSimtUnroll>(p, cta, ctas);
}

static_assert(kMoverThreads == kRowStreamThreads, "the pair kernel runs every body at one CTA size");

// a: a scatter (chunk -> paged), b: a gather (paged -> chunk); launched as a
// programmatic dependent.  kEarly (KVCA_FLAG_INPUTS_READY: the index arrays
// and the scatter's source rows were complete before the previous kernel on
// the stream started): the next launch is let in at once, and the bodies
// load indices and chunk rows before waiting for the previous grid, so only
// the paged loads and the stores wait.  Otherwise everything waits.
template <MoverBody kA, MoverBody kB, bool kEarly>
__global__ void __launch_bounds__(kMoverThreads)
    move_pair_kernel(const __grid_constant__ MoveParams a, const __grid_constant__ MoveParams b, int split) {
  if constexpr (kEarly)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  else
    dependent_launch_entry();
  if (static_cast<int>(blockIdx.x) < split)
    run_mover_body<kA, false, true, kEarly>(a, blockIdx.x, split);
  else
    run_mover_body<kB, true, false, kEarly>(b, static_cast<int64_t>(blockIdx.x) - split,
                                            static_cast<int64_t>(gridDim.x) - split);
}

// Build knobs of the all-CTA pair kernel (sweeps): KVCA_PAIR_ALL_PDL=1
// launches it as a programmatic dependent (with KVCA_FLAG_INPUTS_READY the
// next launch is let in at once and only paged loads and stores wait);
// KVCA_PAIR_ALL_MIN_CTAS=2 bounds its registers so that two 512-thread CTAs
// (or one beside another kernel's CTA of up to 32K registers) fit on an SM;
// KVCA_PAIR_ALL_GRID_PER_SM sets the CTAs launched per SM.  B200, decode
// step with 8 KV heads (64 MiB each way), live decode mix / the cycle's 16
// pair launches replayed alone: plain launch 24.7 / 23.4 us per step,
// programmatic dependent 23.2 / 21.6 us; 64 registers (spills) 25.9 / 25.4
// with one CTA per SM, 26.7 / 25.9 with two, 24.8 / 23.8 with two and the
// programmatic launch.
#ifndef KVCA_PAIR_ALL_PDL
#define KVCA_PAIR_ALL_PDL 1
#endif
#ifndef KVCA_PAIR_ALL_MIN_CTAS
#define KVCA_PAIR_ALL_MIN_CTAS 1
#endif
#ifndef KVCA_PAIR_ALL_GRID_PER_SM
#define KVCA_PAIR_ALL_GRID_PER_SM 1
#endif
// The pair kernel's grid leaves KVCA_PAIR_SPARE_SMS SMs out.  Its CTAs
// split the work statically and fill every SM with one 512-thread CTA, so a
// kernel holding one SM meanwhile (a decode loop's one-CTA booking launch on
// another stream) would leave one CTA waiting for a whole share: the step
// then takes up to twice as long.  B200, decode mix with 8 KV heads, booking
// beside the moves: 23.2 us per step with every SM, 21.8 with one spare, 21.7
// with two; the pair launches alone 21.6 / 21.7 / 21.7 us; one KV head 5.3 us
// live and 4.6 alone either way.
#ifndef KVCA_PAIR_SPARE_SMS
#define KVCA_PAIR_SPARE_SMS 1
#endif
constexpr bool kPairAllPdl = KVCA_PAIR_ALL_PDL != 0;
constexpr int kPairAllGridPerSm = KVCA_PAIR_ALL_GRID_PER_SM;

// Two large independent moves in one launch: every CTA moves its share of
// the scatter, then its share of the gather, so the two share one ramp and
// one tail and every SM carries both.  kEarly as in move_pair_kernel (only
// when launched as a programmatic dependent).
template <MoverBody kA, MoverBody kB, bool kEarly>
__global__ void __launch_bounds__(kMoverThreads, KVCA_PAIR_ALL_MIN_CTAS)
    move_pair_all_kernel(const __grid_constant__ MoveParams a, const __grid_constant__ MoveParams b) {
  if constexpr (kPairAllPdl) {
    if constexpr (kEarly)
      asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    else
      dependent_launch_entry();
  }
  run_mover_body<kA, false, true, kEarly>(a, blockIdx.x, gridDim.x);
  run_mover_body<kB, true, false, kEarly>(b, blockIdx.x, gridDim.x);
}

// Launch as a programmatic dependent of the kernel before it on the stream
// (the kernel must begin with dependent_launch_entry()).
template <typename... Params, typename... Args>
cudaError_t launch_dependent(void (*kernel)(Params...), unsigned grid, unsigned block, size_t smem,
                             cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  return e != cudaSuccess ? e : cudaGetLastError();
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return sms;
}

// Function attributes (the dynamic shared-memory limit, the carve-out)
// belong to the current device's context, so a launcher sets them once per
// device: `done` records the ordinals done (devices past the table are set
// up on every call).
constexpr int kTrackedDevices = 64;
using DeviceFlags = std::atomic<bool>[kTrackedDevices];

bool needs_setup(const DeviceFlags& done, int* dev) {
  *dev = -1;
  if (cudaGetDevice(dev) != cudaSuccess) return true;
  return *dev < 0 || *dev >= kTrackedDevices || !done[*dev].load(std::memory_order_acquire);
}

void mark_setup(DeviceFlags& done, int dev) {
  if (dev >= 0 && dev < kTrackedDevices) done[dev].store(true, std::memory_order_release);
}

template <bool kSrcPaged, bool kDstPaged, typename V, bool kHost = false>
cudaError_t launch_move_typed(const MoveParams& p, cudaStream_t stream) {
  auto kernel = move_rows_kernel<kSrcPaged, kDstPaged, V, kHost>;
  static int blocks_per_sm = 0;
  if (blocks_per_sm == 0) {
    int b = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, kMoverThreads, 0);
    if (e != cudaSuccess) return e;
    blocks_per_sm = b > 0 ? b : 1;
  }
  const int sms = device_sm_count();
  const int64_t items = p.num_planes * p.num_rows * p.segs_per_row;
  const int64_t threads_needed = items << p.tpr_log2;
  int64_t blocks = (threads_needed + kMoverThreads - 1) / kMoverThreads;
  const int64_t resident = static_cast<int64_t>(sms > 0 ? sms : 1) * blocks_per_sm;
  if (blocks > resident) blocks = resident;
  if (kHost && blocks > kHostMoverCtas) blocks = kHostMoverCtas;
  if (blocks < 1) blocks = 1;
  kernel<<<static_cast<unsigned>(blocks), kMoverThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

// Rows of at most kSmallRowMaxVecs 16-byte vectors in device memory: 2^k
// lanes per row with 2^k >= the row's vectors, at most 8, 2 vectors each,
// 4 rows per iteration.
template <bool kSrcPaged, bool kDstPaged>
cudaError_t launch_move_small(MoveParams p, cudaStream_t stream) {
  auto kernel = move_short_rows_pm_kernel<kSrcPaged, kDstPaged, 2, 4>;
  static int blocks_per_sm = 0;
  if (blocks_per_sm == 0) {
    int b = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, kMoverThreads, 0);
    if (e != cudaSuccess) return e;
    blocks_per_sm = b > 0 ? b : 1;
  }
  p.tpr_log2 = 0;
  while (p.tpr_log2 < 3 && (int64_t{1} << p.tpr_log2) < p.row_vecs) ++p.tpr_log2;
  p.seg_vecs = p.row_vecs;
  p.segs_per_row = 1;
  const int sms = device_sm_count();
  const int64_t items = p.num_planes * p.num_rows;
  const int64_t threads_needed = ((items + 3) / 4) << p.tpr_log2;
  int64_t blocks = (threads_needed + kMoverThreads - 1) / kMoverThreads;
  const int64_t resident = static_cast<int64_t>(sms > 0 ? sms : 1) * blocks_per_sm;
  if (blocks > resident) blocks = resident;
  if (blocks < 1) blocks = 1;
  kernel<<<static_cast<unsigned>(blocks), kMoverThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

// Rows of kRowStreamMinVecs to kRowStreamMaxVecs 16-byte vectors in device
// memory (and fewer than 2^30 rows: the kernel keeps row positions in 32
// bits): the warp-cooperative stream mover.
constexpr int64_t kRowStreamMinVecs = 8;
constexpr int64_t kRowStreamMaxVecs = 96;

template <bool kSrcPaged, bool kDstPaged>
cudaError_t launch_move_stream(MoveParams p, cudaStream_t stream) {
  auto kernel = move_rows_stream_kernel<kSrcPaged, kDstPaged>;
  static int blocks_per_sm = 0;
  if (blocks_per_sm == 0) {
    int b = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, kRowStreamThreads, 0);
    if (e != cudaSuccess) return e;
    blocks_per_sm = b > 0 ? b : 1;
  }
  int64_t rpb = (int64_t{32} * kRowStreamSlots) / p.row_vecs;
  if (rpb > 32) rpb = 32;
  if (rpb < 1) rpb = 1;
  p.rows_per_batch = static_cast<int>(rpb);
  p.seg_vecs = p.row_vecs;
  p.segs_per_row = 1;
  const int sms = device_sm_count();
  const int64_t items = p.num_planes * p.num_rows;
  const int64_t warps_needed = (items + rpb - 1) / rpb;
  int64_t blocks = (warps_needed * 32 + kRowStreamThreads - 1) / kRowStreamThreads;
  const int64_t resident = static_cast<int64_t>(sms > 0 ? sms : 1) * blocks_per_sm;
  if (blocks > resident) blocks = resident;
  if (blocks < 1) blocks = 1;
  kernel<<<static_cast<unsigned>(blocks), kRowStreamThreads, 0, stream>>>(p);
  return cudaGetLastError();
}



// ---------------------------------------------------------------------------
// Exchange: spill and fill of the same slots in one pass
// ---------------------------------------------------------------------------
//
// Row j: a.index[j] is a slot of the blocks; its row goes out to store row
// store.index[j] (spill, when >= 0) and store row fill_from[j] comes in
// (fill, when >= 0), so that one launch moves both directions and, with the
// store in host memory, both directions of the host link are busy at once.
// Each lane loads its vectors of the slot and of the fill row before it
// stores either, so a spill always reads the slot's old bytes.  All loads are
// plain: the slot rows are written by this launch.  With *gate != 0 the
// launch only spills (a fill that must wait for every spill follows it).

struct ExchangeParams {
  PagedSide a;
  PagedSide store;
  const int64_t* fill_from;
  const int64_t* gate;
  int64_t num_rows;
  int64_t row_vecs;
  int64_t seg_vecs;
  int64_t segs_per_row;
  int tpr_log2;
  int32_t flags;
  int64_t* status;
};

template <typename V>
__global__ void __launch_bounds__(kMoverThreads) exchange_rows_kernel(const __grid_constant__ ExchangeParams p) {
  const bool fill_open = p.gate == nullptr || *p.gate == 0;
  const int tpr = 1 << p.tpr_log2;
  const int64_t gtid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int lane = static_cast<int>(gtid & (tpr - 1));
  const int64_t group = gtid >> p.tpr_log2;
  const int64_t num_groups = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> p.tpr_log2;
  const int64_t segs = p.segs_per_row;
  const int64_t items = segs * p.num_rows;
  const int64_t per = items / num_groups;
  const int64_t rem = items - per * num_groups;
  const int64_t begin = group * per + (group < rem ? group : rem);
  const int64_t end = begin + per + (group < rem ? 1 : 0);
  const bool lead = lane == 0;
  int64_t cur_row = -1;
  int64_t a_row = -1, out_row = -1, in_row = -1;
  for (int64_t g = begin; g < end; ++g) {
    const int64_t r = g / segs;
    const int64_t sg = g - r * segs;
    if (r != cur_row) {
      cur_row = r;
      a_row = paged_row_offset(p.a, r, p.flags, p.status, lead);
      out_row = paged_row_offset(p.store, r, p.flags, p.status, lead);
      in_row = -1;
      if (fill_open) {
        const int64_t idx = p.fill_from[r];
        if (idx >= p.store.num_blocks) {
          if (lead) report(p.status, KVCA_ERR_BAD_INDEX, idx);
        } else if (idx >= 0) {
          in_row = idx * p.store.block_stride;
        }
      }
    }
    if (a_row < 0 || (out_row < 0 && in_row < 0)) continue;
    V* slot = reinterpret_cast<V*>(p.a.planes[0] + a_row);
    V* out = reinterpret_cast<V*>(p.store.planes[0] + (out_row >= 0 ? out_row : 0));
    const V* in = reinterpret_cast<const V*>(p.store.planes[0] + (in_row >= 0 ? in_row : 0));
    const int64_t v_begin = sg * p.seg_vecs;
    const int64_t v_end = v_begin + p.seg_vecs < p.row_vecs ? v_begin + p.seg_vecs : p.row_vecs;
    for (int64_t b = v_begin + lane; b < v_end; b += static_cast<int64_t>(tpr) * kMoverUnroll) {
      V old_bytes[kMoverUnroll];
      V new_bytes[kMoverUnroll];
      // the incoming row's loads (the long ones, over the host link for a
      // host store) go out first, then the slot's
#pragma unroll
      for (int u = 0; u < kMoverUnroll; ++u) {
        const int64_t i = b + static_cast<int64_t>(u) * tpr;
        if (i < v_end && in_row >= 0) new_bytes[u] = in[i];
      }
#pragma unroll
      for (int u = 0; u < kMoverUnroll; ++u) {
        const int64_t i = b + static_cast<int64_t>(u) * tpr;
        if (i < v_end && out_row >= 0) old_bytes[u] = slot[i];
      }
#pragma unroll
      for (int u = 0; u < kMoverUnroll; ++u) {
        const int64_t i = b + static_cast<int64_t>(u) * tpr;
        if (i < v_end) {
          if (out_row >= 0) out[i] = old_bytes[u];
          if (in_row >= 0) slot[i] = new_bytes[u];
        }
      }
    }
  }
}

template <typename V>
cudaError_t launch_exchange_typed(const ExchangeParams& p, cudaStream_t stream) {
  auto kernel = exchange_rows_kernel<V>;
  static int blocks_per_sm = 0;
  if (blocks_per_sm == 0) {
    int b = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, kMoverThreads, 0);
    if (e != cudaSuccess) return e;
    blocks_per_sm = b > 0 ? b : 1;
  }
  const int sms = device_sm_count();
  const int64_t threads_needed = (p.num_rows * p.segs_per_row) << p.tpr_log2;
  int64_t blocks = (threads_needed + kMoverThreads - 1) / kMoverThreads;
  const int64_t resident = static_cast<int64_t>(sms > 0 ? sms : 1) * blocks_per_sm;
  if (blocks > resident) blocks = resident;
  if ((p.flags & KVCA_FLAG_HOST_MEMORY) && blocks > kHostMoverCtas) blocks = kHostMoverCtas;
  if (blocks < 1) blocks = 1;
  kernel<<<static_cast<unsigned>(blocks), kMoverThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Row mover on the TMA bulk-copy engine (16-byte aligned rows of >= 1 KiB)
// ---------------------------------------------------------------------------
//
// One warp per CTA; lane 0 streams its range of work items through a ring of
// shared-memory stages: cp.async.bulk global->shared completes on the stage's
// mbarrier, then cp.async.bulk shared->global writes it out, and the stage is
// reused once that store has read it (cp.async.bulk.wait_group.read).  Every
// copy stays within this CTA and this GPU's memory.  Rows are cut into segments of at most kBulkSegmentBytes;
// the stage count makes stages x segment = kBulkStageBytes, and the grid holds
// kBulkCtasPerSm CTAs per SM, so about 48 KiB are in flight per SM, the
// amount that measured fastest on B200 (more in flight per SM was slower).

constexpr int kBulkMaxStages = 16;
constexpr int64_t kBulkSegmentBytes = 4096;
constexpr int64_t kBulkStageBytes = 16384;
constexpr int kBulkCtasPerSm = 3;
constexpr int64_t kBulkMinRowBytes = 4096;
constexpr uint32_t kBulkSpinLimit = 1u << 24;  // bounded mbarrier waits

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Waits until at most n of this thread's most recent bulk store groups are
// still reading shared memory (the immediate must be a constant).
__device__ __forceinline__ void bulk_wait_read(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.bulk.wait_group.read 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.bulk.wait_group.read 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.bulk.wait_group.read 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.bulk.wait_group.read 5;" ::: "memory"); break;
    case 6: asm volatile("cp.async.bulk.wait_group.read 6;" ::: "memory"); break;
    case 7: asm volatile("cp.async.bulk.wait_group.read 7;" ::: "memory"); break;
    case 8: asm volatile("cp.async.bulk.wait_group.read 8;" ::: "memory"); break;
    case 9: asm volatile("cp.async.bulk.wait_group.read 9;" ::: "memory"); break;
    case 10: asm volatile("cp.async.bulk.wait_group.read 10;" ::: "memory"); break;
    case 11: asm volatile("cp.async.bulk.wait_group.read 11;" ::: "memory"); break;
    case 12: asm volatile("cp.async.bulk.wait_group.read 12;" ::: "memory"); break;
    case 13: asm volatile("cp.async.bulk.wait_group.read 13;" ::: "memory"); break;
    case 14: asm volatile("cp.async.bulk.wait_group.read 14;" ::: "memory"); break;
    default: asm volatile("cp.async.bulk.wait_group.read 15;" ::: "memory"); break;
  }
}

// Bounded wait for the completion of phase `parity` of an mbarrier.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done = 0;
  for (uint32_t tries = 0; tries < kBulkSpinLimit && !done; ++tries) {
    asm volatile(
        "{ .reg .pred q; mbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2; selp.u32 %0, 1, 0, q; }"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
  }
  return done != 0;
}

template <bool kSrcPaged, bool kDstPaged>
__global__ void __launch_bounds__(32) move_rows_bulk_kernel(const __grid_constant__ MoveParams p,
                                                            int stages) {
  extern __shared__ __align__(128) unsigned char stage_buf[];
  __shared__ __align__(8) uint64_t full[kBulkMaxStages];
  if (threadIdx.x != 0) return;
  const int64_t planes = p.num_planes;
  const int64_t segs = p.segs_per_row;
  const int64_t per_row = planes * segs;
  const int64_t items = per_row * p.num_rows;
  const int64_t groups = gridDim.x;
  const int64_t per = items / groups;
  const int64_t rem = items - per * groups;
  const int64_t group = blockIdx.x;
  const int64_t begin = group * per + (group < rem ? group : rem);
  const int64_t end = begin + per + (group < rem ? 1 : 0);
  if (begin >= end) return;
  for (int s = 0; s < stages; ++s)
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&full[s])));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

  const int64_t seg_bytes = p.seg_vecs * 16;
  const int64_t row_bytes = p.row_vecs * 16;
  int64_t r = begin / per_row;
  int64_t pl = (begin - r * per_row) / segs;
  int64_t sg = begin - r * per_row - pl * segs;
  int64_t g = begin;
  int64_t src_row = 0;
  int64_t dst_row = 0;
  bool row_ready = false;
  uint64_t dst_q[kBulkMaxStages];
  uint32_t bytes_q[kBulkMaxStages];
  int64_t loaded = 0;  // loads issued
  int64_t stored = 0;  // stores issued; item k uses stage k % stages
  bool timed_out = false;
  while (true) {
    while (loaded < stored + stages && g < end) {
      if (!row_ready) {
        row_ready = true;
        src_row = kSrcPaged ? paged_row_offset(p.src_paged, r, p.flags, p.status, true)
                            : chunk_row_offset(p.src_chunk, r);
        dst_row = kDstPaged ? paged_row_offset(p.dst_paged, r, p.flags, p.status, true)
                            : chunk_row_offset(p.dst_chunk, r);
      }
      const bool valid = src_row >= 0 && dst_row >= 0;
      const int64_t off = sg * seg_bytes;
      const int64_t bytes = off + seg_bytes < row_bytes ? seg_bytes : row_bytes - off;
      const uint64_t src = (kSrcPaged ? p.src_paged.planes[pl] + src_row
                                      : p.src_chunk.base + src_row + pl * p.src_chunk.plane_stride) +
                           off;
      const uint64_t dst = (kDstPaged ? p.dst_paged.planes[pl] + dst_row
                                      : p.dst_chunk.base + dst_row + pl * p.dst_chunk.plane_stride) +
                           off;
      ++g;
      if (++sg == segs) {
        sg = 0;
        if (++pl == planes) {
          pl = 0;
          ++r;
          row_ready = false;
        }
      }
      if (!valid) continue;
      const int stage = static_cast<int>(loaded % stages);
      // the store of item loaded - stages used this stage: let it finish reading
      if (loaded >= stages) bulk_wait_read(static_cast<int>(stored - 1 - (loaded - stages)));
      unsigned char* buf = stage_buf + stage * seg_bytes;
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                       smem_u32(&full[stage])),
                   "r"(static_cast<uint32_t>(bytes))
                   : "memory");
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
              smem_u32(buf)),
          "l"(src), "r"(static_cast<uint32_t>(bytes)), "r"(smem_u32(&full[stage]))
          : "memory");
      dst_q[stage] = dst;
      bytes_q[stage] = static_cast<uint32_t>(bytes);
      ++loaded;
    }
    if (stored == loaded) break;
    const int stage = static_cast<int>(stored % stages);
    if (!mbar_wait(&full[stage], static_cast<uint32_t>((stored / stages) & 1))) {
      timed_out = true;
      break;
    }
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst_q[stage]),
                 "r"(smem_u32(stage_buf + stage * seg_bytes)), "r"(bytes_q[stage])
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    ++stored;
  }
  if (timed_out) {
    report(p.status, KVCA_ERR_DEVICE_TIMEOUT, blockIdx.x);
    // let the loads still in flight land before shared memory is released
    for (int64_t k = stored; k < loaded; ++k)
      mbar_wait(&full[k % stages], static_cast<uint32_t>((k / stages) & 1));
  }
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

template <bool kSrcPaged, bool kDstPaged>
cudaError_t launch_move_bulk(const MoveParams& base, cudaStream_t stream) {
  MoveParams p = base;
  p.seg_vecs = kBulkSegmentBytes / 16;
  if (p.seg_vecs >= p.row_vecs) p.seg_vecs = p.row_vecs;
  p.segs_per_row = (p.row_vecs + p.seg_vecs - 1) / p.seg_vecs;
  const int64_t seg_bytes = p.seg_vecs * 16;
  int stages = static_cast<int>(kBulkStageBytes / seg_bytes);
  if (stages > kBulkMaxStages) stages = kBulkMaxStages;
  if (stages < 2) stages = 2;
  const int smem = static_cast<int>(stages * seg_bytes);
  auto kernel = move_rows_bulk_kernel<kSrcPaged, kDstPaged>;
  static DeviceFlags configured;
  int dev = -1;
  if (needs_setup(configured, &dev)) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(kBulkMaxStages * kBulkSegmentBytes));
    if (e != cudaSuccess) return e;
    mark_setup(configured, dev);
  }
  const int sms = device_sm_count();
  const int64_t items = p.num_planes * p.num_rows * p.segs_per_row;
  int64_t blocks = static_cast<int64_t>(sms > 0 ? sms : 1) * kBulkCtasPerSm;
  if (blocks > items) blocks = items;
  if (blocks < 1) blocks = 1;
  kernel<<<static_cast<unsigned>(blocks), 32, smem, stream>>>(p, stages);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Staged token-row gather: shared-memory tiles between random rows and chunks
// ---------------------------------------------------------------------------
//
// For a gather of rows of 128 to 576 bytes into a dense chunk side (rows
// back to back), a (chunk, plane) run of rows is one contiguous range of the
// chunk, cut into tiles of at most kStagedTileBytes.  A CTA owns a
// contiguous range of tiles and a ring of kStagedStages tiles in shared
// memory: every thread copies its 16-byte vectors of a tile's random source
// rows into the tile with cp.async (no register holds the bytes while they
// travel), and once the tile has landed one thread writes it to the chunk
// with one bulk store; kStagedLookahead tiles are in flight behind the one
// being stored, and two CTAs share an SM.  The register-bound stream mover
// keeps at most 9 vectors per lane in flight.  A row whose index is skipped
// (negative with KVCA_FLAG_SKIP_NEGATIVE, or reported as bad) is copied
// from its own chunk row, so the tile store writes its bytes back unchanged.

constexpr int kStagedThreads = 256;
constexpr int kStagedStages = 5;
constexpr int kStagedLookahead = kStagedStages - 2;  // one tile stored, one being refilled
constexpr int64_t kStagedTileBytes = 16384;
constexpr int64_t kStagedMinVecs = 8;   // 128 bytes
constexpr int64_t kStagedMaxVecs = 36;  // 576 bytes
constexpr int kStagedVecsPerThread = static_cast<int>(kStagedTileBytes / 16 / kStagedThreads);
static_assert(kStagedVecsPerThread * kStagedThreads * 16 == kStagedTileBytes, "a tile is whole vectors per thread");

struct StagedGeom {
  int64_t rows_per_tile;
  int64_t tiles_per_unit;
  int64_t units;  // chunks x planes
};

// Tile position advanced one tile at a time (no divisions per tile).
struct TileCursor {
  int64_t c, pl, k;
  __device__ __forceinline__ void init(const MoveParams& p, const StagedGeom& g, int64_t t) {
    const int64_t unit = t / g.tiles_per_unit;
    k = t - unit * g.tiles_per_unit;
    c = unit / p.num_planes;
    pl = unit - c * p.num_planes;
  }
  __device__ __forceinline__ void next(const MoveParams& p, const StagedGeom& g) {
    if (++k == g.tiles_per_unit) {
      k = 0;
      if (++pl == p.num_planes) {
        pl = 0;
        ++c;
      }
    }
  }
  // first row of the tile and its row count (<= 0 past a short last chunk)
  __device__ __forceinline__ void rows(const MoveParams& p, const ChunkSide& cs, const StagedGeom& g, int64_t* r0,
                                       int64_t* n) const {
    const int64_t chunk_row0 = c * cs.rows_per_chunk;
    const int64_t unit_rows =
        p.num_rows - chunk_row0 < cs.rows_per_chunk ? p.num_rows - chunk_row0 : cs.rows_per_chunk;
    *r0 = chunk_row0 + k * g.rows_per_tile;
    const int64_t left = chunk_row0 + unit_rows - *r0;
    *n = left < g.rows_per_tile ? left : g.rows_per_tile;
  }
};

__device__ __forceinline__ uint64_t staged_chunk_addr(const ChunkSide& cs, int64_t c, int64_t pl, int64_t r) {
  return cs.base + c * cs.chunk_stride + pl * cs.plane_stride + (r - c * cs.rows_per_chunk) * cs.row_stride;
}

__device__ __forceinline__ void cp_async16(uint32_t smem, uint64_t gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem), "l"(gmem) : "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(kStagedThreads, 1) move_rows_staged_gather_kernel(const __grid_constant__ MoveParams p,
                                                                                 StagedGeom g) {
  extern __shared__ __align__(128) unsigned char tiles[];
  const ChunkSide& cs = p.dst_chunk;
  const PagedSide& ps = p.src_paged;
  const int64_t total = g.units * g.tiles_per_unit;
  const int64_t tb = total * blockIdx.x / gridDim.x;
  const int64_t te = total * (blockIdx.x + 1) / gridDim.x;
  const int64_t n_tiles = te - tb;
  if (n_tiles <= 0) return;
  const int rv = static_cast<int>(p.row_vecs);
  const int64_t row_bytes = p.row_vecs * 16;
  const int shift = pow2_shift(ps.block_size);
  const uint32_t base = smem_u32(tiles);
  // vector v = threadIdx.x + u * kStagedThreads of every tile is row v / rv,
  // vector v % rv of that row: the same for every tile, so computed once
  int rr[kStagedVecsPerThread];
  int64_t voff[kStagedVecsPerThread];
#pragma unroll
  for (int u = 0; u < kStagedVecsPerThread; ++u) {
    const int v = threadIdx.x + u * kStagedThreads;
    rr[u] = v / rv;
    voff[u] = static_cast<int64_t>(v - rr[u] * rv) * 16;
  }
  TileCursor ld, st;  // the tile loaded next and the tile stored next
  ld.init(p, g, tb);
  st = ld;
  int stage_ld = 0, stage_st = 0;
  for (int64_t k = 0; k < n_tiles + kStagedLookahead; ++k) {
    if (k < n_tiles) {
      const int stage = stage_ld;
      stage_ld = stage_ld + 1 == kStagedStages ? 0 : stage_ld + 1;
      // the store that last read this stage was issued two iterations ago
      if (k >= kStagedStages && threadIdx.x == 0) bulk_wait_read(1);
      __syncthreads();
      int64_t r0, n;
      ld.rows(p, cs, g, &r0, &n);
      const int64_t c = ld.c, pl = ld.pl;
      ld.next(p, g);
      const uint64_t plane = ps.planes[pl];
      const uint64_t chunk0 = staged_chunk_addr(cs, c, pl, r0);
      const uint32_t sbase = base + static_cast<uint32_t>(stage * kStagedTileBytes);
      const int vecs = static_cast<int>(n) * rv;
      int64_t idx[kStagedVecsPerThread];  // all index loads first, then all copies
#pragma unroll
      for (int u = 0; u < kStagedVecsPerThread; ++u) {
        const int v = threadIdx.x + u * kStagedThreads;
        const int64_t r = r0 + rr[u];
        idx[u] = v < vecs ? (ps.index != nullptr ? __ldg(ps.index + r) : r) : 0;
      }
#pragma unroll
      for (int u = 0; u < kStagedVecsPerThread; ++u) {
        const int v = threadIdx.x + u * kStagedThreads;
        if (v < vecs) {
          const int64_t off = paged_slot_offset(ps, idx[u], shift, p.flags, p.status, voff[u] == 0);
          const uint64_t src = off >= 0 ? plane + off + voff[u] : chunk0 + rr[u] * row_bytes + voff[u];
          cp_async16(sbase + static_cast<uint32_t>(v) * 16u, src);
        }
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (k >= kStagedLookahead) {              // store tile k - kStagedLookahead
      cp_async_wait<kStagedLookahead>();       // this thread's copies of that tile have landed
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncthreads();
      int64_t r0, n;
      st.rows(p, cs, g, &r0, &n);
      if (threadIdx.x == 0 && n > 0) {
        const uint32_t src = base + static_cast<uint32_t>(stage_st * kStagedTileBytes);
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                         staged_chunk_addr(cs, st.c, st.pl, r0)),
                     "r"(src), "r"(static_cast<uint32_t>(n * row_bytes))
                     : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      }
      st.next(p, g);
      stage_st = stage_st + 1 == kStagedStages ? 0 : stage_st + 1;
    }
  }
  if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// The staged mover takes gathers of 16-byte-aligned rows of 128 to 576
// bytes in device memory whose chunk side is dense.  B200, random token rows,
// 1 GiB per move: 128 B 5.25 TB/s (the stream mover 4.87), 576 B 5.60 (5.48),
// 256 B 5.76 (5.79); 1,152 B 5.64 (5.78) and every scatter width were
// slower staged (bulk-loaded chunk tiles stored row by row: 128 B 5.01
// against 5.06, 576 B 4.69 against 5.05), so those stay on the stream mover.
bool staged_applies(const MoveParams& p) {
  return p.gate == nullptr && !(p.flags & KVCA_FLAG_HOST_MEMORY) && p.row_vecs >= kStagedMinVecs &&
         p.row_vecs <= kStagedMaxVecs && p.dst_chunk.row_stride == p.row_vecs * 16 &&
         p.dst_chunk.rows_per_chunk > 0 && p.num_rows > 0;
}

cudaError_t launch_move_staged(const MoveParams& p, cudaStream_t stream) {
  const int64_t row_bytes = p.row_vecs * 16;
  const ChunkSide& cs = p.dst_chunk;
  StagedGeom g;
  g.rows_per_tile = kStagedTileBytes / row_bytes;
  const int64_t unit_rows = cs.rows_per_chunk < p.num_rows ? cs.rows_per_chunk : p.num_rows;
  if (g.rows_per_tile > unit_rows) g.rows_per_tile = unit_rows;
  g.tiles_per_unit = (unit_rows + g.rows_per_tile - 1) / g.rows_per_tile;
  g.units = (p.num_rows + cs.rows_per_chunk - 1) / cs.rows_per_chunk * p.num_planes;
  const void* kernel = reinterpret_cast<const void*>(move_rows_staged_gather_kernel);
  const size_t smem = static_cast<size_t>(kStagedStages) * kStagedTileBytes;
  static int blocks_per_sm = 0;
  static DeviceFlags configured;
  int dev = -1;
  if (needs_setup(configured, &dev)) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int b = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, kStagedThreads, smem);
    if (e != cudaSuccess) return e;
    blocks_per_sm = b > 0 ? b : 1;
    mark_setup(configured, dev);
  }
  const int sms = device_sm_count();
  int64_t blocks = static_cast<int64_t>(sms > 0 ? sms : 1) * blocks_per_sm;
  const int64_t tiles = g.units * g.tiles_per_unit;
  if (blocks > tiles) blocks = tiles;
  move_rows_staged_gather_kernel<<<static_cast<unsigned>(blocks), kStagedThreads, smem, stream>>>(p, g);
  return cudaGetLastError();
}

template <bool kSrcPaged, bool kDstPaged>
cudaError_t launch_move_vec(const MoveParams& p, int vec_bytes, cudaStream_t stream) {
  if (p.flags & KVCA_FLAG_HOST_MEMORY) {  // SIMT only: no bulk copies to or from host memory
    switch (vec_bytes) {
      case 16: return launch_move_typed<kSrcPaged, kDstPaged, uint4, true>(p, stream);
      case 8: return launch_move_typed<kSrcPaged, kDstPaged, uint2, true>(p, stream);
      case 4: return launch_move_typed<kSrcPaged, kDstPaged, unsigned int, true>(p, stream);
      case 2: return launch_move_typed<kSrcPaged, kDstPaged, unsigned short, true>(p, stream);
      default: return launch_move_typed<kSrcPaged, kDstPaged, unsigned char, true>(p, stream);
    }
  }
  switch (vec_bytes) {
    case 16:
      if (p.row_vecs * 16 >= kBulkMinRowBytes) return launch_move_bulk<kSrcPaged, kDstPaged>(p, stream);
      if constexpr (kSrcPaged && !kDstPaged) {
        if (staged_applies(p)) return launch_move_staged(p, stream);
      }
      if (p.row_vecs >= kRowStreamMinVecs && p.row_vecs <= kRowStreamMaxVecs && p.num_rows < (int64_t{1} << 30))
        return launch_move_stream<kSrcPaged, kDstPaged>(p, stream);
      if (p.row_vecs <= kSmallRowMaxVecs) return launch_move_small<kSrcPaged, kDstPaged>(p, stream);
      return launch_move_typed<kSrcPaged, kDstPaged, uint4>(p, stream);
    case 8: return launch_move_typed<kSrcPaged, kDstPaged, uint2>(p, stream);
    case 4: return launch_move_typed<kSrcPaged, kDstPaged, unsigned int>(p, stream);
    case 2: return launch_move_typed<kSrcPaged, kDstPaged, unsigned short>(p, stream);
    default: return launch_move_typed<kSrcPaged, kDstPaged, unsigned char>(p, stream);
  }
}

int grid_for(int64_t count, int threads) {
  const int sms = device_sm_count();
  int64_t blocks = (count + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sms > 0 ? sms : 1) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

}  // namespace

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------

namespace {

MoveParams make_move_params(const MoveArgs& a) {
  MoveParams p;
  memset(&p, 0, sizeof(p));
  if (a.src_paged) p.src_paged = *a.src_paged;
  if (a.dst_paged) p.dst_paged = *a.dst_paged;
  if (a.src_chunk) p.src_chunk = *a.src_chunk;
  if (a.dst_chunk) p.dst_chunk = *a.dst_chunk;
  p.num_planes = a.num_planes;
  p.num_rows = a.num_rows;
  p.row_vecs = a.row_bytes / a.vec_bytes;
  // Work items of at most kMoverSegmentBytes; each gets the largest power of
  // two lanes (at most 32) that leaves every lane at least four vectors.
  p.seg_vecs = kMoverSegmentBytes / a.vec_bytes;
  if (p.seg_vecs < 1) p.seg_vecs = 1;
  if (p.seg_vecs >= p.row_vecs) p.seg_vecs = p.row_vecs;
  p.segs_per_row = (p.row_vecs + p.seg_vecs - 1) / p.seg_vecs;
  int64_t lanes = p.seg_vecs / 4;
  if (lanes > 32) lanes = 32;
  p.tpr_log2 = 0;
  while ((int64_t{2} << p.tpr_log2) <= lanes) ++p.tpr_log2;
  p.flags = a.flags;
  p.status = a.status;
  p.gate = a.gate;
  return p;
}

// The body a 16-byte-vector move in device memory takes in the pair kernel
// (the rules of launch_move_vec, with the bulk mover's rows on the SIMT
// body), its parameters adjusted for that body, and the CTAs it can use.
MoverBody pair_body(MoveParams* p, int64_t* ctas_wanted) {
  const int64_t items = p->num_planes * p->num_rows;
  if (p->row_vecs * 16 < kBulkMinRowBytes && p->row_vecs >= kRowStreamMinVecs &&
      p->row_vecs <= kRowStreamMaxVecs && p->num_rows < (int64_t{1} << 30)) {
    int64_t rpb = (int64_t{32} * kRowStreamSlots) / p->row_vecs;
    if (rpb > 32) rpb = 32;
    if (rpb < 1) rpb = 1;
    p->rows_per_batch = static_cast<int>(rpb);
    p->seg_vecs = p->row_vecs;
    p->segs_per_row = 1;
    *ctas_wanted = (((items + rpb - 1) / rpb) * 32 + kMoverThreads - 1) / kMoverThreads;
    return MoverBody::kStream;
  }
  if (p->row_vecs <= kSmallRowMaxVecs) {
    p->tpr_log2 = 0;
    while (p->tpr_log2 < 3 && (int64_t{1} << p->tpr_log2) < p->row_vecs) ++p->tpr_log2;
    p->seg_vecs = p->row_vecs;
    p->segs_per_row = 1;
    *ctas_wanted = ((((items + 3) / 4) << p->tpr_log2) + kMoverThreads - 1) / kMoverThreads;
    return MoverBody::kSmall;
  }
  if (kPairSplitRows && p->row_vecs * 16 >= kBulkMinRowBytes && p->row_vecs % kSplitVecs == 0) {
    const int64_t subs = items * (p->row_vecs / kSplitVecs);
    *ctas_wanted = (((subs + 1) / 2) * 32 + kMoverThreads - 1) / kMoverThreads;
    return MoverBody::kSplit;
  }
  if (p->row_vecs > kMediumRowMinVecs && p->row_vecs <= kMediumRowMaxVecs) {
    p->tpr_log2 = 5;
    p->seg_vecs = p->row_vecs;
    p->segs_per_row = 1;
    *ctas_wanted = ((((items + kMediumRows - 1) / kMediumRows) << 5) + kMoverThreads - 1) / kMoverThreads;
    return MoverBody::kMedium;
  }
  *ctas_wanted = (((items * p->segs_per_row) << p->tpr_log2) + kMoverThreads - 1) / kMoverThreads;
  return MoverBody::kSimt;
}

template <MoverBody kA, MoverBody kB>
cudaError_t launch_pair_typed(const MoveParams& a, const MoveParams& b, int split, int grid, bool early,
                              cudaStream_t stream) {
  if (split < 0) {  // large: every CTA takes part in both moves
    if constexpr (kPairAllPdl) {
      if (early)
        return launch_dependent(move_pair_all_kernel<kA, kB, true>, static_cast<unsigned>(grid), kMoverThreads,
                                0, stream, a, b);
      return launch_dependent(move_pair_all_kernel<kA, kB, false>, static_cast<unsigned>(grid), kMoverThreads, 0,
                              stream, a, b);
    }
    move_pair_all_kernel<kA, kB, false><<<static_cast<unsigned>(grid), kMoverThreads, 0, stream>>>(a, b);
    return cudaGetLastError();
  }
  if (early)
    return launch_dependent(move_pair_kernel<kA, kB, true>, static_cast<unsigned>(grid), kMoverThreads, 0,
                            stream, a, b, split);
  return launch_dependent(move_pair_kernel<kA, kB, false>, static_cast<unsigned>(grid), kMoverThreads, 0,
                          stream, a, b, split);
}

template <MoverBody kA>
cudaError_t launch_pair_b(MoverBody b_body, const MoveParams& a, const MoveParams& b, int split, int grid,
                          bool early, cudaStream_t stream) {
  switch (b_body) {
    case MoverBody::kStream: return launch_pair_typed<kA, MoverBody::kStream>(a, b, split, grid, early, stream);
    case MoverBody::kSmall: return launch_pair_typed<kA, MoverBody::kSmall>(a, b, split, grid, early, stream);
    case MoverBody::kMedium: return launch_pair_typed<kA, MoverBody::kMedium>(a, b, split, grid, early, stream);
    case MoverBody::kSplit: return launch_pair_typed<kA, MoverBody::kSplit>(a, b, split, grid, early, stream);
    default: return launch_pair_typed<kA, MoverBody::kSimt>(a, b, split, grid, early, stream);
  }
}

}  // namespace

cudaError_t launch_move(const MoveArgs& a, cudaStream_t stream) {
  MoveParams p = make_move_params(a);
  if (a.gate != nullptr && a.kind == MoveKind::kCopyPaged) {  // gated moves stay on the SIMT kernel
    switch (a.vec_bytes) {
      case 16:
        return (a.flags & KVCA_FLAG_HOST_MEMORY) ? launch_move_typed<true, true, uint4, true>(p, stream)
                                                 : launch_move_typed<true, true, uint4>(p, stream);
      case 8:
        return (a.flags & KVCA_FLAG_HOST_MEMORY) ? launch_move_typed<true, true, uint2, true>(p, stream)
                                                 : launch_move_typed<true, true, uint2>(p, stream);
      case 4:
        return (a.flags & KVCA_FLAG_HOST_MEMORY) ? launch_move_typed<true, true, unsigned int, true>(p, stream)
                                                 : launch_move_typed<true, true, unsigned int>(p, stream);
      case 2:
        return (a.flags & KVCA_FLAG_HOST_MEMORY) ? launch_move_typed<true, true, unsigned short, true>(p, stream)
                                                 : launch_move_typed<true, true, unsigned short>(p, stream);
      default:
        return (a.flags & KVCA_FLAG_HOST_MEMORY) ? launch_move_typed<true, true, unsigned char, true>(p, stream)
                                                 : launch_move_typed<true, true, unsigned char>(p, stream);
    }
  }
  switch (a.kind) {
    case MoveKind::kGather: return launch_move_vec<true, false>(p, a.vec_bytes, stream);
    case MoveKind::kScatter: return launch_move_vec<false, true>(p, a.vec_bytes, stream);
    default: return launch_move_vec<true, true>(p, a.vec_bytes, stream);
  }
}

// Up to this many bytes moved by the two together, the CTAs are split
// between the moves (each move's chain of loads runs once, side by side);
// above it every CTA takes part in both, one after the other (a decode step
// with 8 KV heads, 64 MiB each way, B200, both on the SIMT body and as
// plain launches: 32.2 us per step split, 29.3 all CTAs in both, 29.6 as
// two launches; with 1 KV head, 4 MiB each way: 6.0 us split against 10.4
// as two launches).  KVCA_PAIR_MAX_MIB sets it for sweeps.
#ifndef KVCA_PAIR_MAX_MIB
#define KVCA_PAIR_MAX_MIB 32
#endif
constexpr double kPairMaxBytes = static_cast<double>(KVCA_PAIR_MAX_MIB) * 1024 * 1024;

cudaError_t launch_scatter_gather(const MoveArgs& scatter, const MoveArgs& gather, cudaStream_t stream) {
  const double bytes_a = static_cast<double>(scatter.num_planes) * scatter.num_rows * scatter.row_bytes;
  const double bytes_b = static_cast<double>(gather.num_planes) * gather.num_rows * gather.row_bytes;
  const bool pairable = scatter.kind == MoveKind::kScatter && gather.kind == MoveKind::kGather &&
                        scatter.vec_bytes == 16 && gather.vec_bytes == 16 && scatter.gate == nullptr &&
                        gather.gate == nullptr && !((scatter.flags | gather.flags) & KVCA_FLAG_HOST_MEMORY) &&
                        scatter.num_rows > 0 && gather.num_rows > 0;
  if (!pairable) {  // two launches, in this order
    if (scatter.num_rows > 0) {
      const cudaError_t e = launch_move(scatter, stream);
      if (e != cudaSuccess) return e;
    }
    return gather.num_rows > 0 ? launch_move(gather, stream) : cudaSuccess;
  }
  MoveParams a = make_move_params(scatter);
  MoveParams b = make_move_params(gather);
  int64_t want_a = 1, want_b = 1;
  const MoverBody body_a = pair_body(&a, &want_a);
  const MoverBody body_b = pair_body(&b, &want_b);
  const bool early = ((scatter.flags & gather.flags) & KVCA_FLAG_INPUTS_READY) != 0;
  if (bytes_a + bytes_b > kPairMaxBytes) {  // every CTA takes part in both
    const int sms_all = device_sm_count();
    const int grid_all =
        sms_all > KVCA_PAIR_SPARE_SMS ? (sms_all - KVCA_PAIR_SPARE_SMS) * kPairAllGridPerSm : 1;
    switch (body_a) {
      case MoverBody::kStream: return launch_pair_b<MoverBody::kStream>(body_b, a, b, -1, grid_all, early, stream);
      case MoverBody::kSmall: return launch_pair_b<MoverBody::kSmall>(body_b, a, b, -1, grid_all, early, stream);
      case MoverBody::kMedium: return launch_pair_b<MoverBody::kMedium>(body_b, a, b, -1, grid_all, early, stream);
      case MoverBody::kSplit: return launch_pair_b<MoverBody::kSplit>(body_b, a, b, -1, grid_all, early, stream);
      default: return launch_pair_b<MoverBody::kSimt>(body_b, a, b, -1, grid_all, early, stream);
    }
  }
  // CTAs split by bytes over the resident grid (one CTA of 512 threads per SM)
  const int sms = device_sm_count();
  const int64_t grid_max = sms - KVCA_PAIR_SPARE_SMS > 1 ? sms - KVCA_PAIR_SPARE_SMS : 2;
  int64_t ca = static_cast<int64_t>(grid_max * bytes_a / (bytes_a + bytes_b) + 0.5);
  if (ca < 1) ca = 1;
  if (ca > grid_max - 1) ca = grid_max - 1;
  int64_t cb = grid_max - ca;
  if (ca > want_a) ca = want_a > 0 ? want_a : 1;
  if (cb > want_b) cb = want_b > 0 ? want_b : 1;
  const int split = static_cast<int>(ca);
  const int grid = static_cast<int>(ca + cb);
  switch (body_a) {
    case MoverBody::kStream: return launch_pair_b<MoverBody::kStream>(body_b, a, b, split, grid, early, stream);
    case MoverBody::kSmall: return launch_pair_b<MoverBody::kSmall>(body_b, a, b, split, grid, early, stream);
    case MoverBody::kMedium: return launch_pair_b<MoverBody::kMedium>(body_b, a, b, split, grid, early, stream);
    case MoverBody::kSplit: return launch_pair_b<MoverBody::kSplit>(body_b, a, b, split, grid, early, stream);
    default: return launch_pair_b<MoverBody::kSimt>(body_b, a, b, split, grid, early, stream);
  }
}

namespace {

// ---------------------------------------------------------------------------
// The moves of a booked decode cycle in one launch
// ---------------------------------------------------------------------------
//
// Step q of the cycle (q < num_steps <= 32) is the spill gather of its victims
// (block rows of the cache to spill rows offsets[q] .. offsets[q + 1]) and
// then the token scatter of its slot-mapping row (num_seqs token rows); the
// result equals running the steps one after the other.  The work is cut into
// warp items of at most kMoveCycleItemBytes (a victim's block rows of a few
// planes, or a sequence's token rows of a few planes; rows longer than that
// in pieces), numbered step by step with a step's gathers before its
// scatters, and warps take item numbers from one counter: every SM streams
// until the cycle's last item, with no launch, ramp or barrier between steps.
// A warp moves an item through its own shared-memory buffer: each lane issues
// 16-byte cp.async loads for its share of the item (all of them in flight at
// once, no registers held), waits, and stores from the buffer.
//
// Items wait only where steps depend on each other.  Before the moves, every
// CTA marks in two per-block words which steps evict the block (victims) and
// which steps write a token row into it (slot mapping); one grid barrier
// later those marks say, for each item, which earlier items it needs:
//   - a token row whose block is a victim of this step or an earlier one
//     waits until all gathers of that step are done (the spill reads the old
//     bytes before the first token of the new owner lands);
//   - a gather of a block that an earlier step's scatter wrote waits until
//     all scatters of that step are done.
// In a decode cycle that is the first token of every new block and, rarely, a
// block released and evicted again within the cycle.  Each wait is for items
// with smaller numbers, and item numbers are taken in order by resident CTAs
// (cooperative launch), so the smallest number in flight never waits on
// anything unfinished.  Token rows written twice in one call (the same slot at
// two steps) end with either row: the slots of a decode cycle are distinct.
//
// The per-block words carry a launch generation in their high half, so words
// of earlier launches read as empty and nothing has to clear them; the last
// CTA to leave resets the counters and advances the generation.

// Warps per CTA (a build knob for sweeps, as is KVCA_CYCLE_ITEM_BYTES; B200,
// a booked 8-KV-head cycle measured alone with 8 items per ticket: 5 warps of
// 16 KiB items 542 us, 3, 5 or 10 warps of 8 KiB items 704-739 us; with 2
// items per ticket, 5 warps of 16 KiB: 368 us under the profiler).
#ifndef KVCA_CYCLE_WARPS
#define KVCA_CYCLE_WARPS 5
#endif
constexpr int kCycleWarps = KVCA_CYCLE_WARPS;
constexpr int kCycleThreads = kCycleWarps * 32;
constexpr int kCycleMaxSteps = static_cast<int>(kMoveCycleMaxSteps);
constexpr uint32_t kCycleItemVecs = static_cast<uint32_t>(kMoveCycleItemBytes / 16);
// Rows of at least this many bytes move as bulk copies (one lane issues a
// copy per row into the item's buffer, and one per row out of it); shorter
// rows move as 16-byte cp.async loads and stores by all lanes.
constexpr int64_t kCycleBulkMinRowBytes = 1024;
constexpr unsigned kCycleItemsPerTicket = 2;
// two items per warp: one landing while the other is stored
constexpr size_t kCycleSmemBytes = static_cast<size_t>(kCycleWarps) * 2 * kMoveCycleItemBytes;

struct CycleWords {
  unsigned int bar_count;  // grid-barrier arrivals
  int failed;              // a wait gave up
  unsigned int ticket;     // next item number
  unsigned int exits;      // CTAs that have left
  unsigned int gen;        // launch generation of the per-block words
  unsigned int pad[3];
  unsigned int g_done[kCycleMaxSteps];  // finished gather items per step
  unsigned int s_done[kCycleMaxSteps];  // finished scatter items per step
};
static_assert(sizeof(CycleWords) <= kCycleHeaderBytes, "cycle words exceed their header");

// n / d for 0 <= n < 2^31 and 1 <= d < 2^31 by a multiply-high, an add and a
// shift (Granlund and Montgomery, "Division by invariant integers using
// multiplication", 1994): with 2^s >= d > 2^(s-1) and
// m = floor(2^32 (2^s - d) / d) + 1, n / d = (mulhi(n, m) + n) >> s.
struct FastDiv {
  uint32_t mul;
  uint32_t shift;
};

FastDiv make_fast_div(uint32_t d) {
  uint32_t s = 0;
  while ((uint64_t{1} << s) < d) ++s;
  const uint64_t m = ((uint64_t{1} << 32) * ((uint64_t{1} << s) - d)) / d + 1;
  return FastDiv{static_cast<uint32_t>(m), s};
}

__device__ __forceinline__ uint32_t fast_div(uint32_t n, FastDiv f) { return (__umulhi(n, f.mul) + n) >> f.shift; }

// How one kind of row (token rows, block rows) is cut into items: `group`
// planes of a unit (a sequence, a victim) per item, rows longer than an item
// in `segs` pieces of kCycleItemVecs vectors (then group = 1).
struct CycleKind {
  uint32_t vecs;      // 16-byte vectors per row
  FastDiv div;        // division by vecs
  int group;
  int segs;
  unsigned per_unit;  // items per unit: ceil(planes / group) * segs
  bool bulk;          // rows of kCycleBulkMinRowBytes or more: one bulk copy per row and item
};

struct CycleParams {
  uint64_t planes[KVCA_MAX_PLANES];  // the cache's planes (layer x K/V)
  int64_t num_blocks;
  int64_t block_stride;      // bytes between blocks of a plane
  int64_t tokens_per_block;  // token rows of a block
  int64_t token_stride;      // bytes between token rows of a block
  const int64_t* slot_mapping;  // num_steps x num_seqs token slots
  const int64_t* victims;       // offsets[num_steps] block ids
  const int64_t* offsets;       // num_steps + 1: victims of step q
  ChunkSide src;                // token rows: row q * num_seqs + s
  ChunkSide spill;              // victim entry e's block rows: row e
  int64_t num_seqs;
  int64_t spill_rows;  // offsets[num_steps] may not pass this
  int num_planes;
  int num_steps;
  CycleKind tok;
  CycleKind blk;
  int32_t flags;
  CycleWords* words;
  unsigned long long* wmask;  // per block: (generation << 32) | steps whose scatter writes it
  unsigned long long* pmask;  // per block: (generation << 32) | steps that evict it
  int64_t* status;
};

// ORs `bit` into a per-block word of generation `gen` (a word of another
// generation counts as empty).  A word changes at most 33 times per
// generation (its generation once, then one bit at a time), so the loop ends
// within 34 tries.
__device__ void cycle_mark(unsigned long long* word, unsigned gen, unsigned bit) {
  unsigned long long old = __ldcg(word);
  for (int tries = 0; tries < 40; ++tries) {
    const unsigned long long want = static_cast<unsigned>(old >> 32) == gen
                                        ? (old | bit)
                                        : ((static_cast<unsigned long long>(gen) << 32) | bit);
    if (want == old) return;
    const unsigned long long seen = atomicCAS(word, old, want);
    if (seen == old) return;
    old = seen;
  }
}

__device__ __forceinline__ unsigned cycle_bits(const unsigned long long* word, unsigned gen) {
  const unsigned long long v = __ldcg(word);
  return static_cast<unsigned>(v >> 32) == gen ? static_cast<unsigned>(v) : 0u;
}

// Waits until *counter reaches target (bounded; false when it gave up or the
// grid failed).
__device__ bool cycle_wait_count(const unsigned* counter, unsigned target, const int* failed) {
  uint32_t spins = 0;
  while (ld_acquire_u32(counter) < target) {
    if (++spins > kGridSpinLimit || *reinterpret_cast<const volatile int*>(failed) != 0) return false;
    __nanosleep(64);
  }
  return true;
}

// One warp item, decoded (the same on every lane of the warp).
struct CycleItem {
  int64_t row;      // victim entry (gather: its spill row) or token row q * num_seqs + s (scatter)
  int64_t tab_off;  // cache side of the item's rows: block * block_stride (+ position * token_stride)
  uint64_t aff;     // spill or token side of the item's first row
  int64_t aff_stride;
  uint32_t vecs;    // vectors per row of this kind
  FastDiv div;
  uint32_t c0;      // first vector of each row
  uint32_t nvec;    // vectors per row in this item
  int pl0;
  int nrows;
  int q;
  bool gather;
  bool bulk;        // moved by bulk copies (see CycleKind)
  bool live;        // the item's block id is inside the cache
  bool fence;       // scatter: a later step gathers the block, so its rows must be visible before the signal
  unsigned dep;     // steps whose counters this item waits for
  int64_t blk;      // block id (-1: outside the cache)
  int64_t pos;      // scatter: token position in the block
};

// Decodes item `t` of step layout first_s / gitems_s; lane 0 reads the item's
// block id and that block's marks, and every lane gets them by shuffle.  An
// item of the same sequence or victim as `prev` (the warp's previous item:
// consecutive items mostly are) takes them from `prev` instead, which saves
// two dependent reads.
__device__ __forceinline__ CycleItem cycle_decode(const CycleParams& p, unsigned t, const unsigned* first_s,
                                                  const unsigned* gitems_s, const int64_t* offs_s, unsigned gen,
                                                  const CycleItem* prev, int lane) {
  CycleItem it;
  int q = 0;
  while (t >= first_s[q + 1]) ++q;
  const unsigned local = t - first_s[q];
  it.q = q;
  it.gather = local < gitems_s[q];
  const CycleKind& kind = it.gather ? p.blk : p.tok;
  const unsigned lu = it.gather ? local : local - gitems_s[q];
  const unsigned unit = lu / kind.per_unit;
  const unsigned rem = lu - unit * kind.per_unit;
  const unsigned grp = rem / static_cast<unsigned>(kind.segs);
  const unsigned seg = rem - grp * static_cast<unsigned>(kind.segs);
  it.pl0 = static_cast<int>(grp) * kind.group;
  it.nrows = min(kind.group, p.num_planes - it.pl0);
  it.vecs = kind.vecs;
  it.div = kind.div;
  it.bulk = kind.bulk;
  it.c0 = seg * kCycleItemVecs;
  it.nvec = kind.segs > 1 ? min(kCycleItemVecs, kind.vecs - it.c0) : kind.vecs;
  it.row = it.gather ? offs_s[q] + unit : static_cast<int64_t>(q) * p.num_seqs + unit;
  int64_t blk = -1, pos = 0;
  unsigned dep = 0, fence = 0;
  if (prev != nullptr && prev->gather == it.gather && prev->row == it.row) {
    blk = prev->live ? prev->blk : -1;
    pos = prev->pos;
    dep = prev->dep;
    fence = prev->fence ? 1u : 0u;
  } else if (lane == 0) {
    if (it.gather) {
      const int64_t v = p.victims[it.row];
      if (v >= 0 && v < p.num_blocks) {
        blk = v;
        dep = cycle_bits(&p.wmask[v], gen) & ((1u << q) - 1u);
      }
    } else {
      const int64_t slot = p.slot_mapping[it.row];
      if (slot >= 0 && slot / p.tokens_per_block < p.num_blocks) {
        blk = slot / p.tokens_per_block;
        pos = slot - blk * p.tokens_per_block;
        const unsigned bits = cycle_bits(&p.pmask[blk], gen);
        dep = bits & ((2u << q) - 1u);
        fence = q < 31 ? bits >> (q + 1) : 0u;
      }
    }
  }
  blk = __shfl_sync(0xffffffffu, blk, 0);
  pos = __shfl_sync(0xffffffffu, pos, 0);
  it.dep = __shfl_sync(0xffffffffu, dep, 0);
  it.fence = __shfl_sync(0xffffffffu, fence, 0) != 0u;
  it.live = blk >= 0;
  it.blk = blk;
  it.pos = pos;
  if (it.gather) {
    it.tab_off = blk * p.block_stride;
    it.aff = p.spill.base + static_cast<uint64_t>(chunk_row_offset(p.spill, it.row)) +
             static_cast<uint64_t>(it.pl0) * p.spill.plane_stride;
    it.aff_stride = p.spill.plane_stride;
  } else {
    it.tab_off = blk * p.block_stride + pos * p.token_stride;
    it.aff = p.src.base + static_cast<uint64_t>(chunk_row_offset(p.src, it.row)) +
             static_cast<uint64_t>(it.pl0) * p.src.plane_stride;
    it.aff_stride = p.src.plane_stride;
  }
  return it;
}

// Row r of an item: its cache side and its spill / token side.
__device__ __forceinline__ uint64_t cycle_cache_row(const CycleItem& it, const uint64_t* planes_s, uint32_t r) {
  return planes_s[it.pl0 + static_cast<int>(r)] + static_cast<uint64_t>(it.tab_off);
}
__device__ __forceinline__ uint64_t cycle_other_row(const CycleItem& it, uint32_t r) {
  return it.aff + static_cast<uint64_t>(r) * static_cast<uint64_t>(it.aff_stride);
}

// Loads the item into `buf`.  Bulk items: lane 0 waits until the bulk
// stores that last read this buffer are done reading it (`reads_left` of its
// newer store groups may still be reading), arms the buffer's mbarrier with
// the item's bytes and issues one bulk copy per row.  Other items: every lane
// issues 16-byte cp.async loads for its vectors (through L2, so a gather sees
// the scatters it waited for).  Every lane then commits a cp.async group
// (empty for bulk items and for an item whose block is outside the cache),
// so that waiting for "all but the newest group" means the same either way.
__device__ __forceinline__ void cycle_issue(const CycleItem& it, const uint64_t* planes_s, uint4* buf,
                                            uint64_t* bar, int reads_left, int lane) {
  if (it.live && it.bulk) {
    if (lane == 0) {
      bulk_wait_read(reads_left);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      const uint32_t row_bytes = it.nvec * 16u;
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                   "r"(row_bytes * static_cast<uint32_t>(it.nrows))
                   : "memory");
      for (int r = 0; r < it.nrows; ++r) {
        const uint64_t row = it.gather ? cycle_cache_row(it, planes_s, r) : cycle_other_row(it, r);
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(buf) + static_cast<uint32_t>(r) * row_bytes),
            "l"(row + static_cast<uint64_t>(it.c0) * 16u), "r"(row_bytes), "r"(smem_u32(bar))
            : "memory");
      }
    }
  } else if (it.live) {
    if (lane == 0) bulk_wait_read(reads_left);
    __syncwarp();
    const uint32_t total = static_cast<uint32_t>(it.nrows) * it.nvec;  // <= kCycleItemVecs
    const uint32_t sbuf = static_cast<uint32_t>(__cvta_generic_to_shared(buf));
    for (uint32_t e = static_cast<uint32_t>(lane); e < total; e += 32u) {
      const uint32_t r = it.nrows == 1 ? 0u : fast_div(e, it.div);
      const uint32_t c = it.c0 + e - r * it.vecs;
      const uint64_t row = it.gather ? cycle_cache_row(it, planes_s, r) : cycle_other_row(it, r);
      cp_async16(sbuf + e * 16u, row + static_cast<uint64_t>(c) * 16u);
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Stores the item's vectors from `buf` (its loads have landed): bulk items
// by lane 0, one bulk copy per row committed as one bulk group; the others by
// every lane.
__device__ __forceinline__ void cycle_store(const CycleItem& it, const uint64_t* planes_s, const uint4* buf,
                                            int lane) {
  if (!it.live) return;
  if (it.bulk) {
    if (lane == 0) {
      const uint32_t row_bytes = it.nvec * 16u;
      for (int r = 0; r < it.nrows; ++r) {
        const uint64_t row = it.gather ? cycle_other_row(it, r) : cycle_cache_row(it, planes_s, r);
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                         row + static_cast<uint64_t>(it.c0) * 16u),
                     "r"(smem_u32(buf) + static_cast<uint32_t>(r) * row_bytes), "r"(row_bytes)
                     : "memory");
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
    return;
  }
  const uint32_t total = static_cast<uint32_t>(it.nrows) * it.nvec;
  for (uint32_t e = static_cast<uint32_t>(lane); e < total; e += 32u) {
    const uint32_t r = it.nrows == 1 ? 0u : fast_div(e, it.div);
    const uint32_t c = it.c0 + e - r * it.vecs;
    const uint64_t row = it.gather ? cycle_other_row(it, r) : cycle_cache_row(it, planes_s, r);
    st_stream(reinterpret_cast<uint4*>(row) + c, buf[e]);
  }
}

// Lane 0 waits for the step counters an item depends on; false (grid marked
// failed, timeout reported) when a wait gave up.  Uniform across the warp.
__device__ __forceinline__ bool cycle_wait_deps(const CycleItem& it, CycleWords* w, unsigned s_items,
                                                const unsigned* gitems_s, int64_t* status, int lane) {
  int ok = 1;
  if (lane == 0 && it.dep != 0u) {
    unsigned dep = it.dep;
    while (dep != 0u && ok) {
      const int j = 31 - __clz(dep);  // latest step first
      dep &= ~(1u << j);
      ok = it.gather ? cycle_wait_count(&w->s_done[j], s_items, &w->failed)
                     : cycle_wait_count(&w->g_done[j], gitems_s[j], &w->failed);
    }
    if (!ok && atomicExch(&w->failed, 1) == 0) report(status, KVCA_ERR_DEVICE_TIMEOUT, blockIdx.x);
    // the rows it waited for may have been written by bulk copies
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ void cycle_leave(CycleWords* w) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&w->exits, 1u) == gridDim.x - 1u) {
      w->bar_count = 0u;
      w->failed = 0;
      w->ticket = 0u;
      for (int q = 0; q < kCycleMaxSteps; ++q) {
        w->g_done[q] = 0u;
        w->s_done[q] = 0u;
      }
      w->gen = w->gen + 1u;
      __threadfence();
      w->exits = 0u;
    }
  }
}

// Item numbers a warp works through: kCycleItemsPerTicket consecutive items
// per ticket, the next ticket taken one ticket ahead.
struct CycleTickets {
  unsigned item;
  unsigned end;
  unsigned next_ticket;  // lane 0's prefetched ticket
};

__device__ __forceinline__ unsigned cycle_next_item(CycleTickets& tk, CycleWords* w, unsigned total, int lane) {
  if (tk.item < tk.end) return tk.item++;
  const unsigned t = __shfl_sync(0xffffffffu, tk.next_ticket, 0);
  int stop = 0;
  if (lane == 0) {
    tk.next_ticket = atomicAdd(&w->ticket, 1u);
    stop = *reinterpret_cast<const volatile int*>(&w->failed);
  }
  if (__shfl_sync(0xffffffffu, stop, 0) != 0) return total;
  const unsigned first = t * kCycleItemsPerTicket;
  if (first >= total) return total;
  tk.item = first + 1u;
  tk.end = min(first + kCycleItemsPerTicket, total);
  return first;
}

__global__ void __launch_bounds__(kCycleThreads, 2) move_cycle_kernel(const __grid_constant__ CycleParams p) {
  extern __shared__ __align__(128) uint4 cycle_buf[];
  __shared__ uint64_t planes_s[KVCA_MAX_PLANES];
  __shared__ int64_t offs_s[kCycleMaxSteps + 1];
  __shared__ unsigned first_s[kCycleMaxSteps + 1];  // first item of step q; [num_steps] = all items
  __shared__ unsigned gitems_s[kCycleMaxSteps];     // gather items of step q
  __shared__ unsigned gen_s;
  __shared__ int bad_s;
  __shared__ __align__(8) uint64_t cycle_bars[2 * kCycleWarps];  // one mbarrier per buffer half
  CycleWords* w = p.words;
  const int tid = static_cast<int>(threadIdx.x);
  const int S = p.num_steps;
  const int P = p.num_planes;
  const int64_t N = p.num_seqs;
  for (int i = tid; i < P; i += blockDim.x) planes_s[i] = p.planes[i];
  if (tid <= S) offs_s[tid] = p.offsets[tid];
  if (tid == 0) gen_s = __ldcg(&w->gen);
  if (tid < 2 * kCycleWarps) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&cycle_bars[tid])));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  __syncthreads();
  const unsigned s_items = static_cast<unsigned>(N) * p.tok.per_unit;
  if (tid == 0) {
    int bad = offs_s[0] != 0 || offs_s[S] > p.spill_rows;
    unsigned first = 0;
    for (int q = 0; q < S; ++q) {
      const int64_t nv = offs_s[q + 1] - offs_s[q];
      if (nv < 0) bad = 1;
      first_s[q] = first;
      gitems_s[q] = bad ? 0u : static_cast<unsigned>(nv) * p.blk.per_unit;
      first += gitems_s[q] + s_items;
    }
    first_s[S] = first;
    bad_s = bad;
    if (bad && blockIdx.x == 0) report(p.status, KVCA_ERR_BAD_ARGUMENT, offs_s[S]);
  }
  __syncthreads();
  const unsigned gen = gen_s;
  const bool skip_neg = (p.flags & KVCA_FLAG_SKIP_NEGATIVE) != 0;
  if (!bad_s) {  // mark which steps evict and which write each block
    const int64_t gthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + tid;
    for (int64_t e = gt; e < S * N; e += gthreads) {
      const int64_t slot = p.slot_mapping[e];
      if (slot < 0) {
        if (!skip_neg) report(p.status, KVCA_ERR_BAD_INDEX, slot);
        continue;
      }
      const int64_t blk = slot / p.tokens_per_block;
      if (blk >= p.num_blocks) {
        report(p.status, KVCA_ERR_BAD_INDEX, slot);
        continue;
      }
      cycle_mark(&p.wmask[blk], gen, 1u << static_cast<unsigned>(e / N));
    }
    for (int64_t e = gt; e < offs_s[S]; e += gthreads) {
      const int64_t v = p.victims[e];
      if (v < 0 || v >= p.num_blocks) {
        if (v >= 0 || !skip_neg) report(p.status, KVCA_ERR_BAD_INDEX, v);
        continue;
      }
      int q = 0;
      while (offs_s[q + 1] <= e) ++q;
      cycle_mark(&p.pmask[v], gen, 1u << q);
    }
  }
  if (!grid_barrier_words(&w->bar_count, &w->failed, p.status)) {
    cycle_leave(w);
    return;
  }
  if (!bad_s) {
    // Two items in flight per warp, one in each half of the warp's buffer:
    // the next item's loads are issued before the current item is stored
    // when the next item waits for nothing.  An item is signalled before the
    // warp waits for anything else, so the smallest unsignalled item number
    // never waits for an unsignalled one.
    const int lane = tid & 31;
    const int warp = tid >> 5;
    uint4* bufs = cycle_buf + static_cast<size_t>(warp) * 2 * kCycleItemVecs;
    uint64_t* bars = cycle_bars + 2 * warp;
    uint32_t parity = 0u;  // bit h: phase of half h's mbarrier to wait for next
    uint32_t armed = 0u;   // bit h: bulk loads issued into half h and not yet waited for
    const unsigned total = first_s[S];
    CycleTickets tk;
    tk.item = tk.end = 0u;
    tk.next_ticket = lane == 0 ? atomicAdd(&w->ticket, 1u) : 0u;
    unsigned i0 = cycle_next_item(tk, w, total, lane);
    CycleItem cur;
    bool have = false;
    int half = 0;
    if (i0 < total) {
      cur = cycle_decode(p, i0, first_s, gitems_s, offs_s, gen, nullptr, lane);
      have = cycle_wait_deps(cur, w, s_items, gitems_s, p.status, lane);
      if (have) {
        cycle_issue(cur, planes_s, bufs, &bars[0], 0, lane);
        if (cur.live && cur.bulk) armed |= 1u;
      }
    }
    while (have) {
      const unsigned i1 = cycle_next_item(tk, w, total, lane);
      const bool have_next = i1 < total;
      CycleItem nx;
      bool early = false;
      if (have_next) {
        nx = cycle_decode(p, i1, first_s, gitems_s, offs_s, gen, &cur, lane);
        early = nx.dep == 0u;
        if (early) {
          // the other half was last read by the newest bulk store group
          cycle_issue(nx, planes_s, bufs + (half ^ 1) * kCycleItemVecs, &bars[half ^ 1], 0, lane);
          if (nx.live && nx.bulk) armed |= 1u << (half ^ 1);
        }
      }
      // the current item's loads
      int ok = 1;
      if (cur.live && cur.bulk) {
        if (lane == 0) {
          ok = mbar_wait(&bars[half], (parity >> half) & 1u) ? 1 : 0;
          if (!ok && atomicExch(&w->failed, 1) == 0) report(p.status, KVCA_ERR_DEVICE_TIMEOUT, blockIdx.x);
        }
        parity ^= 1u << half;
        armed &= ~(1u << half);
        ok = __shfl_sync(0xffffffffu, ok, 0);
      } else if (early) {
        cp_async_wait<1>();  // all but the next item's group
      } else {
        cp_async_wait<0>();
      }
      __syncwarp();
      if (!ok) break;  // the loads still in flight are waited for below
      if (cur.gather && lane == 0)  // its reads are done: the block may be overwritten
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&w->g_done[cur.q]) : "memory");
      cycle_store(cur, planes_s, bufs + half * kCycleItemVecs, lane);
      __syncwarp();
      if (!cur.gather && lane == 0) {
        if (cur.fence) {  // a later gather of this block reads these rows
          if (cur.bulk) {
            asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
            asm volatile("fence.proxy.async.global;" ::: "memory");
          }
          __threadfence();
        }
        atomicAdd(&w->s_done[cur.q], 1u);
      }
      if (!have_next) break;
      if (!early) {
        if (!cycle_wait_deps(nx, w, s_items, gitems_s, p.status, lane)) break;
        // the other half was last read by the store group before the newest
        cycle_issue(nx, planes_s, bufs + (half ^ 1) * kCycleItemVecs, &bars[half ^ 1], 1, lane);
        if (nx.live && nx.bulk) armed |= 1u << (half ^ 1);
      }
      cur = nx;
      half ^= 1;
    }
    cp_async_wait<0>();
    if (lane == 0) {
      // bulk loads still in flight land before shared memory is released
      for (int h = 0; h < 2; ++h)
        if (armed & (1u << h)) mbar_wait(&bars[h], (parity >> h) & 1u);
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
    __syncwarp();
  }
  cycle_leave(w);
}

CycleKind make_cycle_kind(int64_t row_bytes, int64_t planes) {
  CycleKind k;
  k.vecs = static_cast<uint32_t>(row_bytes / 16);
  k.div = make_fast_div(k.vecs);
  k.group = static_cast<int>(move_cycle_group(row_bytes, planes));
  k.segs = static_cast<int>(move_cycle_segments(row_bytes));
  k.per_unit = static_cast<unsigned>(((planes + k.group - 1) / k.group) * k.segs);
  k.bulk = row_bytes >= kCycleBulkMinRowBytes;
  return k;
}

}  // namespace

size_t move_cycle_scratch_bytes(int64_t num_blocks) {
  return kCycleHeaderBytes + 2 * static_cast<size_t>(num_blocks) * sizeof(unsigned long long);
}

cudaError_t launch_move_cycle(const CycleArgs& a, cudaStream_t stream) {
  CycleParams p;
  memset(&p, 0, sizeof(p));
  for (int64_t i = 0; i < a.num_planes; ++i) p.planes[i] = a.cache->planes[i];
  p.num_blocks = a.cache->num_blocks;
  p.block_stride = a.cache->block_stride;
  p.tokens_per_block = a.cache->block_size;
  p.token_stride = a.cache->row_stride;
  p.slot_mapping = a.cache->index;
  p.victims = a.victims;
  p.offsets = a.offsets;
  p.src = *a.src;
  p.spill = *a.spill;
  p.num_seqs = a.num_seqs;
  p.spill_rows = a.spill_rows < a.num_victims ? a.spill_rows : a.num_victims;
  p.num_planes = static_cast<int>(a.num_planes);
  p.num_steps = static_cast<int>(a.num_steps);
  p.tok = make_cycle_kind(a.token_row_bytes, a.num_planes);
  p.blk = make_cycle_kind(a.block_row_bytes, a.num_planes);
  p.flags = a.flags;
  p.words = reinterpret_cast<CycleWords*>(a.scratch);
  p.wmask = reinterpret_cast<unsigned long long*>(a.scratch + kCycleHeaderBytes);
  p.pmask = p.wmask + a.cache->num_blocks;
  p.status = a.status;
  static DeviceFlags configured;
  int dev = -1;
  if (needs_setup(configured, &dev)) {
    cudaError_t e = cudaFuncSetAttribute(move_cycle_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kCycleSmemBytes));
    if (e != cudaSuccess) return e;
    // the largest shared-memory carve-out, so that an SM running this CTA
    // still has room for the bookkeeping kernel's CTA
    e = cudaFuncSetAttribute(move_cycle_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    int b = 0;
    const cudaError_t e2 =
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, move_cycle_kernel, kCycleThreads, kCycleSmemBytes);
    if (e2 != cudaSuccess) return e2;
    if (b < 1) return cudaErrorInvalidConfiguration;
    mark_setup(configured, dev);
  }
  int sms = device_sm_count();
  if (sms < 1) sms = 1;
  void* args[] = {&p};
  // one CTA per SM, leaving registers and shared memory beside it for a
  // bookkeeping kernel on another stream
  return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(move_cycle_kernel), dim3(static_cast<unsigned>(sms)),
                                     dim3(kCycleThreads), args, kCycleSmemBytes, stream);
}

cudaError_t launch_exchange(const ExchangeArgs& a, cudaStream_t stream) {
  ExchangeParams p;
  memset(&p, 0, sizeof(p));
  p.a = *a.slots;
  p.store = *a.store;
  p.fill_from = a.fill_from;
  p.gate = a.gate;
  p.num_rows = a.num_rows;
  p.row_vecs = a.row_bytes / a.vec_bytes;
  p.seg_vecs = kMoverSegmentBytes / a.vec_bytes;
  if (p.seg_vecs < 1) p.seg_vecs = 1;
  if (p.seg_vecs >= p.row_vecs) p.seg_vecs = p.row_vecs;
  p.segs_per_row = (p.row_vecs + p.seg_vecs - 1) / p.seg_vecs;
  int64_t lanes = p.seg_vecs / 4;
  if (lanes > 32) lanes = 32;
  p.tpr_log2 = 0;
  while ((int64_t{2} << p.tpr_log2) <= lanes) ++p.tpr_log2;
  p.flags = a.flags;
  p.status = a.status;
  switch (a.vec_bytes) {
    case 16: return launch_exchange_typed<uint4>(p, stream);
    case 8: return launch_exchange_typed<uint2>(p, stream);
    case 4: return launch_exchange_typed<unsigned int>(p, stream);
    case 2: return launch_exchange_typed<unsigned short>(p, stream);
    default: return launch_exchange_typed<unsigned char>(p, stream);
  }
}

#define KVCA_META_DISPATCH(bits, ...)           \
  do {                                          \
    if ((bits) == 16) {                         \
      using MetaT = uint16_t;                   \
      __VA_ARGS__;                              \
    } else {                                    \
      using MetaT = uint8_t;                    \
      __VA_ARGS__;                              \
    }                                           \
  } while (0)

cudaError_t launch_inspect_load(int meta_bits, const int64_t* l2p, int64_t num_logical,
                                const void* meta, int64_t num_slots, const int64_t* ids,
                                int64_t count, int64_t* cur_out, uint8_t* resident_out,
                                int64_t* pin_out, void* usage_out, int64_t* status,
                                cudaStream_t stream) {
  const int threads = 256;
  KVCA_META_DISPATCH(meta_bits, inspect_load_kernel<MetaT><<<grid_for(count, threads), threads, 0, stream>>>(
                                    l2p, num_logical, static_cast<const MetaT*>(meta), num_slots,
                                    ids, count, cur_out, resident_out, pin_out,
                                    static_cast<MetaT*>(usage_out), status));
  return cudaGetLastError();
}

cudaError_t launch_inspect_save(int meta_bits, const int64_t* l2p, int64_t num_logical,
                                const void* meta, int64_t num_slots, const int64_t* ids,
                                int64_t count, int64_t* cur_out, uint8_t* existing_out,
                                void* usage_out, int64_t* status, cudaStream_t stream) {
  const int threads = 256;
  KVCA_META_DISPATCH(meta_bits, inspect_save_kernel<MetaT><<<grid_for(count, threads), threads, 0, stream>>>(
                                    l2p, num_logical, static_cast<const MetaT*>(meta), num_slots,
                                    ids, count, cur_out, existing_out,
                                    static_cast<MetaT*>(usage_out), status));
  return cudaGetLastError();
}

namespace {

// ---------------------------------------------------------------------------
// Clock sweep over a large table on the whole GPU
// ---------------------------------------------------------------------------
//
// pop_kernel runs on one CTA, which holds the bandwidth of one SM: fine when
// the victims are found near the scan start, slow when the pop must rank
// whole usage classes and age every slot (a 1,048,576-slot table then takes
// hundreds of microseconds).  pop_grid_kernel splits the scan order (from
// search_start, wrapping) into one contiguous range per CTA of a cooperative
// grid.  Every CTA marks the blocked slots of its range in shared memory
// (each reads the whole blocked list) and counts its available slots by usage
// class.  CTA 0, whose range starts the scan order, also ranks its usage-0
// slots, the first victims of either order: if they are enough it writes
// them and search_start and tells the grid to stop (no grid barrier at all).
// Otherwise every CTA publishes its counts, meets the others at one bounded
// grid barrier, derives T, the class bases and its own offsets, writes its
// victims and ages its own slots; the CTA holding the last victim writes
// search_start.  search_start is written only when no CTA will read it
// again.  The vector that holds the scan start is split between the first
// range (slots >= start) and the last (slots < start): the first range's
// owner ages all of it, and the last range's owner classifies its part from
// a copy taken before the barrier.  The grid words are zero on entry and the
// last CTA to leave zeroes them again.  Results equal pop_kernel's bit for
// bit.

constexpr int kGridPopThreads = 512;
constexpr int kGridPopWarps = kGridPopThreads / 32;
constexpr int kGridPopMaxCtas = 160;
constexpr int64_t kGridPopMinSlots = 65536;
constexpr int64_t kGridPopMaxSlots = int64_t{1} << 24;  // blocked bits of a range fit in 16 KiB
constexpr size_t kGridPopHeader = 256;
// grid words + per-CTA class counts (sized for 16-bit words: 256 classes)
constexpr size_t kGridPopAreaBytes = kGridPopHeader + size_t{kGridPopMaxCtas} * 256 * sizeof(int);

constexpr int kGridUndecided = 0;
constexpr int kGridDone = 1;  // CTA 0 wrote every victim: the others leave
constexpr int kGridGo = 2;    // the counts of every range decide

struct PopGridWords {
  unsigned int bar_count;  // grid-barrier arrivals
  int failed;              // a barrier wait gave up
  int state;               // kGridUndecided, kGridDone or kGridGo (CTA 0's verdict)
  unsigned int exits;      // CTAs that have left
};

template <typename MetaT>
struct GridPopShared {
  int hist[Meta<MetaT>::kUsageMax + 1];
  long long before[Meta<MetaT>::kUsageMax + 1];  // class members in earlier ranges
  long long cls_base[Meta<MetaT>::kUsageMax + 1];
  long long limit[Meta<MetaT>::kUsageMax + 1];
  long long run[Meta<MetaT>::kUsageMax + 1];
  int scan[33];
  long long start;
  long long need;
  long long before_le;  // prefix order: slots of usage <= T in earlier ranges
  long long last0;      // CTA 0: slot of usage-0 rank count - 1
  long long found0;     // CTA 0: usage-0 slots in its range
  int threshold;
  int bad;
  int state;
  MetaVec<MetaT> split;  // the split start vector, as read before the barrier
};

// Vector and segment bounds of scan-order piece vv.
__device__ __forceinline__ int64_t piece_vector(int64_t vv, int64_t p0, int64_t n, int64_t v0b,
                                                int64_t V0, int64_t* lo, int64_t* hi) {
  if (vv < V0) {
    *lo = p0;
    *hi = n;
    return v0b + vv;
  }
  *lo = 0;
  *hi = p0;
  return vv - V0;
}

// Adds this thread's available slots of one vector to the CTA's class counts.
// 8-bit words: the 16 class counts of a warp travel as 16-bit fields of four
// words through one warp sum each; 16-bit words (256 classes): one shared
// atomic per class and group of equal lanes.
template <typename MetaT>
__device__ __forceinline__ void count_classes(const MetaVec<MetaT>& m, unsigned avail, int* hist) {
  using M = Meta<MetaT>;
  constexpr int kSpv = M::kSlotsPerVec;
  if constexpr (sizeof(MetaT) == 1) {
    unsigned long long f0 = 0ull, f1 = 0ull, f2 = 0ull, f3 = 0ull;  // classes 4q .. 4q + 3
#pragma unroll
    for (int j = 0; j < kSpv; ++j) {
      const unsigned u = M::usage(m.s[j]);
      const unsigned long long one = ((avail >> j) & 1ull) << (16u * (u & 3u));
      f0 += (u >> 2) == 0u ? one : 0ull;
      f1 += (u >> 2) == 1u ? one : 0ull;
      f2 += (u >> 2) == 2u ? one : 0ull;
      f3 += (u >> 2) == 3u ? one : 0ull;
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      f0 += __shfl_xor_sync(0xffffffffu, f0, d);
      f1 += __shfl_xor_sync(0xffffffffu, f1, d);
      f2 += __shfl_xor_sync(0xffffffffu, f2, d);
      f3 += __shfl_xor_sync(0xffffffffu, f3, d);
    }
    const int c = threadIdx.x & 31;
    if (c < 16) {
      const unsigned long long word = c < 4 ? f0 : c < 8 ? f1 : c < 12 ? f2 : f3;
      const int v = static_cast<int>((word >> (16u * (c & 3))) & 0xffffull);
      if (v) atomicAdd(hist + c, v);
    }
  } else {
#pragma unroll
    for (int j = 0; j < kSpv; ++j) {
      const int key = ((avail >> j) & 1u) ? static_cast<int>(M::usage(m.s[j])) : -1;
      const unsigned peers = __match_any_sync(0xffffffffu, key);
      if (key >= 0 && (threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(hist + key, __popc(peers));
    }
  }
}

// The last CTA to leave zeroes the grid words for the next launch.
__device__ __forceinline__ void grid_pop_leave(PopGridWords* gw) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&gw->exits, 1u) == gridDim.x - 1u) {
      gw->bar_count = 0u;
      gw->failed = 0;
      gw->state = kGridUndecided;
      __threadfence();
      gw->exits = 0u;
    }
  }
}

template <typename MetaT>
__global__ void __launch_bounds__(kGridPopThreads)
    pop_grid_kernel(MetaT* meta, int64_t n, int64_t* search_start, const int64_t* blocked,
                    int64_t num_blocked, int64_t count, int64_t* out, unsigned char* area, int order,
                    bool aligned, int64_t* status) {
  using M = Meta<MetaT>;
  constexpr int kSpv = M::kSlotsPerVec;
  constexpr int U = M::kUsageMax + 1;
  extern __shared__ uint32_t blk[];  // blocked bits of this CTA's range, by position in it
  __shared__ GridPopShared<MetaT> sh;
  PopGridWords* gw = reinterpret_cast<PopGridWords*>(area);
  int* ghist = reinterpret_cast<int*>(area + kGridPopHeader);
  const int64_t G = gridDim.x;
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;

  // search_start is rewritten only by CTA 0 when it alone finishes (the others
  // then leave without using what they read) or after the barrier
  if (tid == 0) {
    long long s = static_cast<long long>(__ldcg(search_start) % n);
    if (s < 0) s += n;
    sh.start = s;
    sh.bad = 0;
    sh.found0 = 0;
    sh.last0 = -1;
  }
  __syncthreads();
  const int64_t p0 = sh.start;
  const int64_t v0b = p0 / kSpv;
  const int64_t nvec = (n + kSpv - 1) / kSpv;
  const int64_t V0 = nvec - v0b;
  const int64_t V = V0 + (p0 + kSpv - 1) / kSpv;
  const bool split = (p0 % kSpv) != 0;  // vector v0b is pieces 0 and V - 1
  const int64_t cb = V * b / G;
  const int64_t ce = V * (b + 1) / G;
  const int64_t words = ((ce - cb) * kSpv + 31) / 32;

  // ---- 1. blocked bits of the range, class counts, CTA 0's usage-0 ranks ---
  for (int64_t i = tid; i < words; i += blockDim.x) blk[i] = 0u;
  for (int c = tid; c < U; c += blockDim.x) sh.hist[c] = 0;
  __syncthreads();
  for (int64_t i = tid; i < num_blocked; i += blockDim.x) {
    const int64_t x = blocked[i];
    if (x < 0 || x >= n) {
      sh.bad = 1;
      if (b == 0) report(status, KVCA_ERR_BAD_INDEX, x);
      continue;
    }
    const int64_t vv = x >= p0 ? x / kSpv - v0b : V0 + x / kSpv;
    if (vv >= cb && vv < ce) {
      const int64_t bit = (vv - cb) * kSpv + x % kSpv;
      atomicOr(blk + (bit >> 5), 1u << (bit & 31));
    }
  }
  __syncthreads();
  if (sh.bad) {  // every CTA saw the same list: none goes further
    grid_pop_leave(gw);
    return;
  }

  for (int64_t tile = cb; tile < ce; tile += blockDim.x) {
    const int64_t vv = tile + tid;
    int64_t v = 0;
    MetaVec<MetaT> m;
    m.raw = make_uint4(0u, 0u, 0u, 0u);
    unsigned avail = 0u;
    if (vv < ce) {
      int64_t lo, hi;
      v = piece_vector(vv, p0, n, v0b, V0, &lo, &hi);
      load_meta_vec(meta, n, v, aligned, m);
      if (split && vv == V - 1) sh.split = m;
      const int64_t bit0 = (vv - cb) * kSpv;
#pragma unroll
      for (int j = 0; j < kSpv; ++j) {
        const int64_t slot = v * kSpv + j;
        const int64_t bit = bit0 + j;
        const bool blocked_here = (blk[bit >> 5] >> (bit & 31)) & 1u;
        if (slot >= lo && slot < hi && M::pin(m.s[j]) == 0u && !blocked_here) avail |= 1u << j;
      }
    }
    count_classes<MetaT>(m, avail, sh.hist);
    if (b == 0) {  // uniform per CTA: ranks of usage-0 slots from the scan start
      unsigned zero_mask = 0u;
#pragma unroll
      for (int j = 0; j < kSpv; ++j)
        if (((avail >> j) & 1u) && M::usage(m.s[j]) == 0u) zero_mask |= 1u << j;
      int total;
      const int base = block_excl_scan(__popc(zero_mask), &total, sh.scan);
      int64_t rank = sh.found0 + base;
      while (zero_mask != 0u) {
        const int j = __ffs(zero_mask) - 1;
        zero_mask &= zero_mask - 1u;
        if (rank < count) out[rank] = v * kSpv + j;
        if (rank == count - 1) sh.last0 = v * kSpv + j;
        ++rank;
      }
      __syncthreads();
      if (tid == 0) sh.found0 += total;
      __syncthreads();
    }
  }
  __syncthreads();

  // ---- 2. CTA 0's verdict -------------------------------------------------
  if (b == 0) {
    const bool done = sh.found0 >= count;
    if (!done)
      for (int c = tid; c < U; c += blockDim.x) __stcg(ghist + c, sh.hist[c]);
    __syncthreads();
    if (tid == 0) {
      if (done) *search_start = (sh.last0 + 1) % n;
      __threadfence();
      asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(&gw->state), "r"(done ? kGridDone : kGridGo)
                   : "memory");
    }
    if (done) {
      grid_pop_leave(gw);
      return;
    }
  } else {
    for (int c = tid; c < U; c += blockDim.x) __stcg(ghist + b * U + c, sh.hist[c]);
    if (tid == 0) {
      int state = kGridUndecided;
      if (bounded_wait_change(reinterpret_cast<const unsigned*>(&gw->state), kGridUndecided, &gw->failed))
        state = static_cast<int>(ld_acquire_u32(reinterpret_cast<const unsigned*>(&gw->state)));
      else
        report(status, KVCA_ERR_DEVICE_TIMEOUT, b);
      sh.state = state;
    }
    __syncthreads();
    if (sh.state != kGridGo) {
      grid_pop_leave(gw);
      return;
    }
  }
  if (!grid_barrier_words(&gw->bar_count, &gw->failed, status)) {
    grid_pop_leave(gw);
    return;
  }

  // ---- 3. threshold, class bases and this range's offsets -----------------
  for (int c = warp; c < U; c += kGridPopWarps) {  // one warp per class
    long long tot = 0, bef = 0;
    for (int64_t g = lane; g < G; g += 32) {
      const int h = __ldcg(ghist + g * U + c);
      tot += h;
      if (g < b) bef += h;
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      tot += __shfl_xor_sync(0xffffffffu, tot, d);
      bef += __shfl_xor_sync(0xffffffffu, bef, d);
    }
    if (lane == 0) {
      sh.before[c] = bef;
      sh.limit[c] = tot;  // the class total for now
      sh.run[c] = 0;
    }
  }
  __syncthreads();
  if (tid == 0) {
    long long cum = 0, before_le = 0;
    int t_found = -1;
    for (int c = 0; c < U; ++c) {
      sh.cls_base[c] = cum;
      before_le += sh.before[c];
      cum += sh.limit[c];
      if (cum >= count) {
        t_found = c;
        break;
      }
    }
    sh.threshold = t_found;
    if (t_found >= 0) {
      sh.need = count - sh.cls_base[t_found];
      sh.limit[t_found] = sh.need;
      sh.before_le = before_le;
    }
  }
  __syncthreads();
  const int threshold = sh.threshold;
  if (threshold < 0) {
    if (b == 0 && tid == 0) report(status, KVCA_ERR_INSUFFICIENT_CAPACITY, count);
    grid_pop_leave(gw);
    return;
  }

  // ---- 4. victims and aging of this range ---------------------------------
  int64_t run_prefix = 0;
  for (int64_t tile = cb; tile < ce; tile += blockDim.x) {
    const int64_t vv = tile + tid;
    const bool active = vv < ce;
    MetaVec<MetaT> m;
    unsigned avail = 0u;
    int64_t v = 0;
    if (active) {
      int64_t lo, hi;
      v = piece_vector(vv, p0, n, v0b, V0, &lo, &hi);
      const bool last_piece = split && vv == V - 1;
      if (last_piece) m = sh.split;
      else load_meta_vec(meta, n, v, aligned, m);
      const int64_t bit0 = (vv - cb) * kSpv;
      MetaVec<MetaT> aged;
#pragma unroll
      for (int j = 0; j < kSpv; ++j) {
        const int64_t slot = v * kSpv + j;
        const unsigned w = m.s[j];
        const int64_t bit = bit0 + j;
        const bool blocked_here = (blk[bit >> 5] >> (bit & 31)) & 1u;
        if (slot >= lo && slot < hi && M::pin(w) == 0u && !blocked_here) avail |= 1u << j;
        const unsigned u = M::usage(w);
        aged.s[j] = M::pack(M::pin(w), u > static_cast<unsigned>(threshold) ? u - threshold : 0u);
      }
      // the first piece's owner ages the whole start vector; the last piece never writes
      if (threshold > 0 && !last_piece) store_meta_vec(meta, n, v, aligned, aged);
    }
    if (order == KVCA_POP_ORDER_GROUPED) {
      for (int c = 0; c <= threshold; ++c) {
        if (sh.hist[c] == 0) continue;  // uniform: this range has no member of class c
        unsigned mask = 0u;
        if (active) {
#pragma unroll
          for (int j = 0; j < kSpv; ++j)
            if (((avail >> j) & 1u) && M::usage(m.s[j]) == static_cast<unsigned>(c)) mask |= 1u << j;
        }
        int total;
        const int base = block_excl_scan(__popc(mask), &total, sh.scan);
        int64_t rank = sh.before[c] + sh.run[c] + base;
        while (mask != 0u) {
          const int j = __ffs(mask) - 1;
          mask &= mask - 1u;
          if (rank < sh.limit[c]) {
            out[sh.cls_base[c] + rank] = v * kSpv + j;
            if (c == threshold && rank == sh.need - 1) *search_start = (v * kSpv + j + 1) % n;
          }
          ++rank;
        }
        __syncthreads();
        if (tid == 0) sh.run[c] += total;
        __syncthreads();
      }
    } else {
      unsigned mask = 0u;
      if (active) {
#pragma unroll
        for (int j = 0; j < kSpv; ++j)
          if (((avail >> j) & 1u) && M::usage(m.s[j]) <= static_cast<unsigned>(threshold)) mask |= 1u << j;
      }
      int total;
      const int base = block_excl_scan(__popc(mask), &total, sh.scan);
      int64_t rank = sh.before_le + run_prefix + base;
      while (mask != 0u) {
        const int j = __ffs(mask) - 1;
        mask &= mask - 1u;
        if (rank < count) {
          out[rank] = v * kSpv + j;
          if (rank == count - 1) *search_start = (v * kSpv + j + 1) % n;
        }
        ++rank;
      }
      run_prefix += total;
    }
  }
  grid_pop_leave(gw);
}

size_t grid_pop_area_offset(int64_t num_slots) {
  const size_t bitmap = static_cast<size_t>((num_slots + 31) / 32) * sizeof(uint32_t);
  return (bitmap + 255) / 256 * 256;
}

template <typename MetaT>
cudaError_t launch_pop_grid(MetaT* meta, int64_t n, int64_t* search_start, const int64_t* blocked,
                            int64_t num_blocked, int64_t count, int64_t* out, unsigned char* area,
                            int order, bool aligned, int64_t* status, cudaStream_t stream) {
  constexpr int kSpv = Meta<MetaT>::kSlotsPerVec;
  const int64_t V = (n + kSpv - 1) / kSpv + 1;
  int sms = device_sm_count();
  if (sms < 1) sms = 1;
  int64_t grid = V / 64;
  if (grid > sms) grid = sms;
  if (grid > kGridPopMaxCtas) grid = kGridPopMaxCtas;
  if (grid < 1) grid = 1;
  const int64_t per = (V + grid - 1) / grid;
  const size_t smem = static_cast<size_t>((per * kSpv + 31) / 32) * sizeof(uint32_t);
  void* args[] = {&meta, &n, &search_start, &blocked, &num_blocked, &count, &out, &area, &order,
                  &aligned, &status};
  return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(pop_grid_kernel<MetaT>),
                                     dim3(static_cast<unsigned>(grid)), dim3(kGridPopThreads), args, smem,
                                     stream);
}

}  // namespace

size_t pop_scratch_bytes(int64_t num_slots) {
  if (num_slots <= 0) return 0;
  const size_t bitmap = static_cast<size_t>((num_slots + 31) / 32) * sizeof(uint32_t);
  if (num_slots < kGridPopMinSlots || num_slots > kGridPopMaxSlots) return bitmap;
  return grid_pop_area_offset(num_slots) + kGridPopAreaBytes;
}

int pop_threads_for(int meta_bits, int64_t num_slots) {
  const int64_t spv = meta_bits == 16 ? 8 : 16;
  const int64_t vecs = (num_slots + spv - 1) / spv;
  int64_t threads = ((vecs + 31) / 32) * 32;
  if (threads < 32) threads = 32;
  if (threads > 1024) threads = 1024;
  return static_cast<int>(threads);
}

cudaError_t launch_pop(int meta_bits, int order, void* meta, int64_t num_slots,
                       int64_t* search_start, const int64_t* blocked, int64_t num_blocked,
                       int64_t count, int64_t* out, uint32_t* bitmap, int64_t* status,
                       cudaStream_t stream) {
  const bool aligned = (reinterpret_cast<uintptr_t>(meta) & 15u) == 0u;
  if (num_slots >= kGridPopMinSlots && num_slots <= kGridPopMaxSlots) {  // the whole GPU
    unsigned char* area = reinterpret_cast<unsigned char*>(bitmap) + grid_pop_area_offset(num_slots);
    cudaError_t e = cudaSuccess;
    KVCA_META_DISPATCH(meta_bits, e = launch_pop_grid<MetaT>(static_cast<MetaT*>(meta), num_slots, search_start,
                                                             blocked, num_blocked, count, out, area, order,
                                                             aligned, status, stream));
    return e;
  }
  const int threads = pop_threads_for(meta_bits, num_slots);
  KVCA_META_DISPATCH(meta_bits, pop_kernel<MetaT><<<1, threads, 0, stream>>>(
                                    static_cast<MetaT*>(meta), num_slots, search_start, blocked,
                                    num_blocked, count, out, bitmap, order, aligned, status));
  return cudaGetLastError();
}

cudaError_t launch_commit_load(int meta_bits, int64_t* l2p, int64_t num_logical, int64_t* p2l,
                               void* meta, int64_t num_slots, const int64_t* evicted,
                               int64_t num_evicted, const int64_t* miss_ids,
                               const int64_t* miss_slots, int64_t num_miss,
                               const int64_t* hit_slots, const int64_t* hit_pins,
                               const void* hit_usage, int64_t num_hit, const void* miss_usage,
                               int64_t* status, cudaStream_t stream) {
  int64_t longest = num_evicted > num_miss ? num_evicted : num_miss;
  if (num_hit > longest) longest = num_hit;
  int threads = static_cast<int>(((longest + 31) / 32) * 32);
  if (threads < 32) threads = 32;
  if (threads > 1024) threads = 1024;
  KVCA_META_DISPATCH(meta_bits, commit_load_kernel<MetaT><<<1, threads, 0, stream>>>(
                                    l2p, num_logical, p2l, static_cast<MetaT*>(meta), num_slots,
                                    evicted, num_evicted, miss_ids, miss_slots, num_miss,
                                    hit_slots, hit_pins, static_cast<const MetaT*>(hit_usage),
                                    num_hit, static_cast<const MetaT*>(miss_usage), status));
  return cudaGetLastError();
}

cudaError_t launch_commit_save(int meta_bits, int64_t* l2p, int64_t num_logical, int64_t* p2l,
                               void* meta, int64_t num_slots, const int64_t* evicted,
                               int64_t num_evicted, const int64_t* ids, const int64_t* slots,
                               const void* final_pins, const void* final_usage, int64_t count,
                               int64_t* status, cudaStream_t stream) {
  const int64_t longest = num_evicted > count ? num_evicted : count;
  int threads = static_cast<int>(((longest + 31) / 32) * 32);
  if (threads < 32) threads = 32;
  if (threads > 1024) threads = 1024;
  KVCA_META_DISPATCH(meta_bits, commit_save_kernel<MetaT><<<1, threads, 0, stream>>>(
                                    l2p, num_logical, p2l, static_cast<MetaT*>(meta), num_slots,
                                    evicted, num_evicted, ids, slots,
                                    static_cast<const MetaT*>(final_pins),
                                    static_cast<const MetaT*>(final_usage), count, status));
  return cudaGetLastError();
}

cudaError_t launch_plan_load(int meta_bits, int order, const int64_t* l2p, int64_t num_logical,
                             const int64_t* p2l, void* meta, int64_t num_slots,
                             int64_t* search_start, const int64_t* ids, int64_t count,
                             uint32_t* bitmap, int64_t* result, int64_t* hit_slots,
                             int64_t* hit_pins, void* hit_usage, int64_t* miss_ids, int64_t* victims,
                             int64_t* evict_ids, int64_t* evict_slots, int64_t* counts,
                             int64_t* status, cudaStream_t stream) {
  const bool aligned = (reinterpret_cast<uintptr_t>(meta) & 15u) == 0u;
  KVCA_META_DISPATCH(meta_bits, plan_load_kernel<MetaT><<<1, kPlanThreads, 0, stream>>>(
                                    l2p, num_logical, p2l, static_cast<MetaT*>(meta), num_slots,
                                    search_start, ids, count, bitmap, order, aligned, result,
                                    hit_slots, hit_pins, static_cast<MetaT*>(hit_usage), miss_ids,
                                    victims, evict_ids, evict_slots, counts, status));
  return cudaGetLastError();
}

cudaError_t launch_plan_save(int meta_bits, int order, const int64_t* l2p, int64_t num_logical,
                             const int64_t* p2l, void* meta, int64_t num_slots,
                             int64_t* search_start, const int64_t* ids, int64_t count,
                             uint32_t* bitmap, int64_t* selected, int64_t* move_slots,
                             void* final_pins, void* final_usage, int64_t* allocated,
                             int64_t* evict_ids, int64_t* evict_slots, int64_t* counts,
                             int64_t* status, cudaStream_t stream) {
  const bool aligned = (reinterpret_cast<uintptr_t>(meta) & 15u) == 0u;
  KVCA_META_DISPATCH(meta_bits, plan_save_kernel<MetaT><<<1, kPlanThreads, 0, stream>>>(
                                    l2p, num_logical, p2l, static_cast<MetaT*>(meta), num_slots,
                                    search_start, ids, count, bitmap, order, aligned, selected,
                                    move_slots, static_cast<MetaT*>(final_pins),
                                    static_cast<MetaT*>(final_usage),
                                    allocated, evict_ids, evict_slots, counts, status));
  return cudaGetLastError();
}

cudaError_t launch_append_step(int meta_bits, int order, void* meta, int64_t num_slots,
                               int64_t* search_start, int64_t* l2p, int64_t num_logical,
                               int64_t* p2l, const int64_t* need, int64_t num_need,
                               int64_t* cur_block, int64_t* cur_logical, int64_t* pos,
                               int64_t num_seqs, int64_t block_size, int64_t* next_logical,
                               uint32_t* bitmap, int64_t* victims, int64_t* slot_mapping,
                               int64_t* status, cudaStream_t stream) {
  const bool aligned = (reinterpret_cast<uintptr_t>(meta) & 15u) == 0u;
  (void)bitmap;  // the step blocks no slot
  KVCA_META_DISPATCH(meta_bits, append_step_kernel<MetaT><<<1, kAppendThreads, 0, stream>>>(
                                    static_cast<MetaT*>(meta), num_slots, search_start, l2p,
                                    num_logical, p2l, need, num_need, cur_block, cur_logical, pos,
                                    num_seqs, block_size, next_logical, order, aligned,
                                    victims, slot_mapping, status));
  return cudaGetLastError();
}

cudaError_t launch_append_steps(int meta_bits, int order, void* meta, int64_t num_slots,
                                int64_t* search_start, int64_t* l2p, int64_t num_logical,
                                int64_t* p2l, const int64_t* need, const int64_t* need_offsets,
                                int64_t num_need, int64_t num_steps, int64_t* cur_block,
                                int64_t* cur_logical, int64_t* pos, int64_t num_seqs,
                                int64_t block_size, int64_t* next_logical, int64_t* victims,
                                int64_t* slot_mapping, int64_t* status, cudaStream_t stream) {
  const bool aligned = (reinterpret_cast<uintptr_t>(meta) & 15u) == 0u;
  static DeviceFlags configured;
  int dev = -1;
  if (needs_setup(configured, &dev)) {
    cudaError_t e = cudaFuncSetAttribute(append_steps_kernel<uint8_t>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kAppendDynMax));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(append_steps_kernel<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kAppendDynMax));
    if (e != cudaSuccess) return e;
    mark_setup(configured, dev);
  }
  static_assert(kAppendSmemBytes <= kAppendDynMax, "the staged state always fits");
  const bool staged = num_seqs <= kAppendSmemSeqs;
  const size_t staged_bytes = staged ? static_cast<size_t>(3 * num_seqs + kAppendSmemNeed) * sizeof(int64_t) : 0;
  const size_t mirror_at = (staged_bytes + 15) / 16 * 16;
  const size_t meta_bytes = meta_bits == 16 ? sizeof(uint16_t) : sizeof(uint8_t);
  const size_t mirror_bytes = (static_cast<size_t>(num_slots) * meta_bytes + 15) / 16 * 16;
  const bool mirrored = kAppendMirror && num_slots > 0 && mirror_at + mirror_bytes <= kAppendDynMax;
  const size_t smem = mirrored ? mirror_at + mirror_bytes : staged_bytes;
  const int64_t mirror_off = mirrored ? static_cast<int64_t>(mirror_at) : -1;
  // launches of at most kAppendMaxSteps steps, in stream order
  for (int64_t s0 = 0; s0 < num_steps; s0 += kAppendMaxSteps) {
    const int64_t k = num_steps - s0 < kAppendMaxSteps ? num_steps - s0 : kAppendMaxSteps;
    KVCA_META_DISPATCH(meta_bits, append_steps_kernel<MetaT><<<1, kAppendThreads, smem, stream>>>(
                                      static_cast<MetaT*>(meta), num_slots, search_start, l2p,
                                      num_logical, p2l, need, need_offsets + s0, num_need, k,
                                      cur_block, cur_logical, pos, num_seqs, block_size,
                                      next_logical, order, aligned, victims,
                                      slot_mapping + s0 * num_seqs, status, staged, mirror_off));
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_store_load_meta(int meta_bits, int order, int64_t* l2p, int64_t num_logical,
                                   int64_t* p2l, void* meta, int64_t num_slots,
                                   int64_t* search_start, const int64_t* ids, int64_t count,
                                   uint32_t* bitmap, int32_t* scratch, uint8_t* present,
                                   int64_t* work, void* work_meta, int64_t* result,
                                   int64_t* counts, int64_t* status, cudaStream_t stream) {
  const int64_t k = count;
  int64_t* hit_slots = work;
  int64_t* hit_pins = work + k;
  int64_t* miss_ids = work + 2 * k;
  int64_t* victims = work + 3 * k;
  int64_t* evict_ids = work + 4 * k;
  int64_t* evict_slots = work + 5 * k;
  int64_t* xslot = work + 6 * k;
  int64_t* spill_to = work + 7 * k;
  int64_t* fill_from = work + 8 * k;
  // xslot, spill_to and fill_from index the exchange: -1 (skipped, no error)
  // wherever the finish kernel writes nothing; the gate starts closed
  cudaError_t e = cudaMemsetAsync(xslot, 0xFF, 3 * k * sizeof(int64_t), stream);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(counts + 7, 0, sizeof(int64_t), stream);
  if (e != cudaSuccess) return e;
  e = launch_plan_load(meta_bits, order, l2p, num_logical, p2l, meta, num_slots, search_start, ids,
                       count, bitmap, result, hit_slots, hit_pins, work_meta, miss_ids, victims,
                       evict_ids, evict_slots, counts, status, stream);
  if (e != cudaSuccess) return e;
  KVCA_META_DISPATCH(meta_bits, store_load_finish_kernel<MetaT><<<1, 1024, 0, stream>>>(
                                    l2p, num_logical, p2l, static_cast<MetaT*>(meta), num_slots,
                                    counts, hit_slots, hit_pins,
                                    static_cast<const MetaT*>(work_meta), miss_ids, victims,
                                    evict_ids, scratch, present, xslot, spill_to, fill_from,
                                    status));
  return cudaGetLastError();
}

cudaError_t launch_store_save_meta(int meta_bits, int order, int64_t* l2p, int64_t num_logical,
                                   int64_t* p2l, void* meta, int64_t num_slots,
                                   int64_t* search_start, const int64_t* ids, int64_t count,
                                   uint32_t* bitmap, int32_t* scratch, uint8_t* present,
                                   int64_t* work, void* work_meta, int64_t* counts,
                                   int64_t* status, cudaStream_t stream) {
  const int64_t k = count;
  int64_t* selected = work;
  int64_t* allocated = work + k;
  int64_t* evict_ids = work + 2 * k;
  int64_t* evict_slots = work + 3 * k;
  int64_t* move_slots = work + 4 * k;
  const size_t wsz = meta_bits == 8 ? 1 : 2;
  void* final_pins = work_meta;
  void* final_usage = static_cast<char*>(work_meta) + k * wsz;
  // evict_ids, evict_slots and move_slots index the copies: -1 where unwritten
  cudaError_t e = cudaMemsetAsync(evict_ids, 0xFF, 3 * k * sizeof(int64_t), stream);
  if (e != cudaSuccess) return e;
  e = launch_plan_save(meta_bits, order, l2p, num_logical, p2l, meta, num_slots, search_start, ids,
                       count, bitmap, selected, move_slots, final_pins, final_usage, allocated,
                       evict_ids, evict_slots, counts, status, stream);
  if (e != cudaSuccess) return e;
  KVCA_META_DISPATCH(meta_bits, store_save_finish_kernel<MetaT><<<1, 1024, 0, stream>>>(
                                    l2p, num_logical, p2l, static_cast<MetaT*>(meta), num_slots,
                                    counts, ids, count, selected,
                                    static_cast<const MetaT*>(final_pins),
                                    static_cast<const MetaT*>(final_usage), evict_ids,
                                    evict_slots, scratch, present, status));
  return cudaGetLastError();
}

// Threads of a small store call's CTA: its phases are chains of short
// dependent steps joined by block barriers, and barriers of 8 warps are
// cheaper than of 32; larger requests keep 1,024 threads for their scans.
unsigned small_store_threads(int64_t count) { return count <= 256 ? 256u : 1024u; }

cudaError_t launch_store_load_small(int meta_bits, int order, int64_t* l2p, int64_t num_logical, int64_t* p2l,
                                    void* meta, int64_t num_slots, int64_t* search_start, const int64_t* ids,
                                    int64_t count, uint32_t* bitmap, int32_t* scratch, uint8_t* present,
                                    int64_t* work, void* work_meta, int64_t* result, int64_t* counts,
                                    int64_t* status, const StoreRowArgs& r, cudaStream_t stream,
                                    int64_t* host_counts, int64_t seq) {
  const bool aligned = (reinterpret_cast<uintptr_t>(meta) & 15u) == 0u;
  const StoreRows rows{r.actual, r.actual_stride, r.storage, r.storage_stride, r.data, r.row_bytes, r.vec};
  KVCA_META_DISPATCH(meta_bits, store_load_small_kernel<MetaT><<<1, small_store_threads(count), 0, stream>>>(
                                    l2p, num_logical, p2l, static_cast<MetaT*>(meta), num_slots, search_start, ids,
                                    count, bitmap, order, aligned, scratch, present, work,
                                    static_cast<MetaT*>(work_meta), result, counts, status, rows, host_counts,
                                    seq));
  return cudaGetLastError();
}

cudaError_t launch_store_save_small(int meta_bits, int order, int64_t* l2p, int64_t num_logical, int64_t* p2l,
                                    void* meta, int64_t num_slots, int64_t* search_start, const int64_t* ids,
                                    int64_t count, uint32_t* bitmap, int32_t* scratch, uint8_t* present,
                                    int64_t* work, void* work_meta, int64_t* counts, int64_t* status,
                                    const StoreRowArgs& r, cudaStream_t stream, int64_t* host_counts,
                                    int64_t seq) {
  const bool aligned = (reinterpret_cast<uintptr_t>(meta) & 15u) == 0u;
  const StoreRows rows{r.actual, r.actual_stride, r.storage, r.storage_stride, r.data, r.row_bytes, r.vec};
  KVCA_META_DISPATCH(meta_bits, store_save_small_kernel<MetaT><<<1, small_store_threads(count), 0, stream>>>(
                                    l2p, num_logical, p2l, static_cast<MetaT*>(meta), num_slots, search_start, ids,
                                    count, bitmap, order, aligned, scratch, present, work,
                                    static_cast<MetaT*>(work_meta), counts, status, rows, host_counts, seq));
  return cudaGetLastError();
}

cudaError_t launch_release(int meta_bits, const int64_t* l2p, int64_t num_logical, void* meta,
                           int64_t num_slots, const int64_t* ids, int64_t count, int64_t* status,
                           cudaStream_t stream) {
  int threads = static_cast<int>(((count + 31) / 32) * 32);
  if (threads < 32) threads = 32;
  if (threads > 1024) threads = 1024;
  KVCA_META_DISPATCH(meta_bits, release_kernel<MetaT><<<1, threads, 0, stream>>>(
                                    l2p, num_logical, static_cast<MetaT*>(meta), num_slots, ids,
                                    count, status));
  return cudaGetLastError();
}

cudaError_t launch_clock_stream(int meta_bits, int order, void* meta, int64_t num_slots,
                                int64_t* search_start, int64_t num_steps, int64_t alloc_per_step,
                                const int64_t* reaccess, int64_t reaccess_per_step,
                                int64_t* victims, int64_t* steps_done, int64_t* status,
                                cudaStream_t stream) {
  int threads = pop_threads_for(meta_bits, num_slots);
  const int64_t bump_threads =
      ((reaccess_per_step + kStreamMaxReaccessPerThread - 1) / kStreamMaxReaccessPerThread + 31) /
      32 * 32;
  if (bump_threads > threads) threads = static_cast<int>(bump_threads > 1024 ? 1024 : bump_threads);
  const bool aligned = (reinterpret_cast<uintptr_t>(meta) & 15u) == 0u;
  KVCA_META_DISPATCH(meta_bits, clock_stream_kernel<MetaT><<<1, threads, 0, stream>>>(
                                    static_cast<MetaT*>(meta), num_slots, search_start, num_steps,
                                    alloc_per_step, reaccess, reaccess_per_step, victims,
                                    steps_done, order, aligned, status));
  return cudaGetLastError();
}

// The grid barrier's bounded wait on a word nothing may change: reports
// KVCA_ERR_DEVICE_TIMEOUT (value -1) when *flag stays `from`.
__global__ void wait_selftest_kernel(const unsigned* flag, unsigned from, int64_t* status) {
  if (threadIdx.x == 0 && !bounded_wait_change(flag, from, nullptr))
    report(status, KVCA_ERR_DEVICE_TIMEOUT, -1);
}

template <typename MetaT>
cudaError_t launch_stream_grid(int grid, MetaT* meta, int64_t num_slots, int64_t* search_start,
                               int64_t num_steps, int64_t alloc_per_step, const int64_t* reaccess,
                               int64_t reaccess_per_step, int64_t* victims, int64_t* steps_done,
                               int order, bool aligned, unsigned char* scratch, int64_t* status,
                               cudaStream_t stream) {
  if (grid == 1) {
    clock_stream_batched_kernel<MetaT><<<1, kStreamThreads, 0, stream>>>(
        meta, num_slots, search_start, num_steps, alloc_per_step, reaccess, reaccess_per_step,
        victims, steps_done, order, aligned, scratch, status);
    return cudaGetLastError();
  }
  void* args[] = {&meta,     &num_slots,  &search_start, &num_steps, &alloc_per_step,
                  &reaccess, &reaccess_per_step, &victims, &steps_done, &order,
                  &aligned,  &scratch,    &status};
  return cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(clock_stream_batched_kernel<MetaT>),
                                     dim3(grid), dim3(kStreamThreads), args, 0, stream);
}

template <typename MetaT>
int stream_grid_size(int ctas) {
  if (ctas > 0) return ctas < kStreamMaxCtas ? ctas : kStreamMaxCtas;
  // one CTA per SM (a cooperative grid must be resident all at once)
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, clock_stream_batched_kernel<MetaT>,
                                                    kStreamThreads, 0) != cudaSuccess ||
      per_sm < 1)
    return 1;
  const int sms = device_sm_count();
  return sms < 1 ? 1 : (sms < kStreamMaxCtas ? sms : kStreamMaxCtas);
}

cudaError_t launch_wait_selftest(const uint32_t* flag, uint32_t from, int64_t* status,
                                 cudaStream_t stream) {
  wait_selftest_kernel<<<1, 32, 0, stream>>>(flag, from, status);
  return cudaGetLastError();
}

cudaError_t launch_clock_stream_batched(int meta_bits, int order, void* meta, int64_t num_slots,
                                        int64_t* search_start, int64_t num_steps,
                                        int64_t alloc_per_step, const int64_t* reaccess,
                                        int64_t reaccess_per_step, int64_t* victims,
                                        int64_t* steps_done, unsigned char* scratch, int ctas,
                                        int64_t* status, cudaStream_t stream) {
  bool aligned = (reinterpret_cast<uintptr_t>(meta) & 15u) == 0u;
  cudaError_t e = cudaMemsetAsync(scratch + 32 * num_slots, 0, sizeof(StreamGrid), stream);
  if (e != cudaSuccess) return e;
  KVCA_META_DISPATCH(meta_bits,
                     e = launch_stream_grid<MetaT>(stream_grid_size<MetaT>(ctas),
                                                   static_cast<MetaT*>(meta), num_slots,
                                                   search_start, num_steps, alloc_per_step,
                                                   reaccess, reaccess_per_step, victims,
                                                   steps_done, order, aligned, scratch, status,
                                                   stream));
  return e;
}

}  // namespace kvca

// ---------------------------------------------------------------------------
// Clock sweep for callers that cannot allocate device memory
// ---------------------------------------------------------------------------
//
// kvca_pop_reusable_slots needs a blocked-slot bitmap from its caller.  Some
// callers cannot provide one: a serving loop whose device memory is reserved
// up front and must not touch the allocator again, a host language runtime
// that owns no device allocator, or an embedding whose memory budget is fixed
// at start-up.  For them the bitmap lives in a
// file-scope device array instead, sized for at most KVCA_NOALLOC_MAX_SLOTS
// slots (128 KiB), which every GPU that loads this library holds until the
// process exits.

#include <mutex>

namespace kvca {
namespace {

constexpr int64_t kNoAllocWords = KVCA_NOALLOC_MAX_SLOTS / 32;
constexpr int kMaxDevices = 64;

// Shared by every call on a device; it keeps whatever the last call left.
static __device__ __align__(256) uint32_t g_pop_scratch_bitmap[kNoAllocWords];

std::mutex g_scratch_mutex;
uint32_t* g_scratch_address[kMaxDevices] = {};

// Device address of g_pop_scratch_bitmap on the current device, looked up
// once per device (host code only holds a stand-in for the symbol).  The
// cached address belongs to the context that was current at the lookup; a
// cudaDeviceReset destroys that context, so a process that resets a device
// must not call the no-alloc entry point on it again.
cudaError_t scratch_bitmap_address(uint32_t** address) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_address[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_pop_scratch_bitmap);
    if (e != cudaSuccess) return e;
    g_scratch_address[dev] = static_cast<uint32_t*>(p);
  }
  *address = g_scratch_address[dev];
  return cudaSuccess;
}

// pop_kernel with the bitmap in the shared device array: the words this call
// reads are zeroed first, since the previous call's contents are not trusted.
template <typename MetaT>
__global__ void __launch_bounds__(1024)
    pop_noalloc_kernel(MetaT* meta, int64_t num_slots, int64_t* search_start,
                       const int64_t* blocked, int64_t num_blocked, int64_t count, int64_t* out,
                       uint32_t* bitmap, int order, bool aligned, int64_t* status) {
  __shared__ PopShared<MetaT> sh;
  __shared__ int bad_blocked;
  const int64_t words = (num_slots + 31) / 32;
  for (int64_t i = threadIdx.x; i < words; i += blockDim.x) bitmap[i] = 0u;
  if (threadIdx.x == 0) bad_blocked = 0;
  __syncthreads();
  for (int64_t i = threadIdx.x; i < num_blocked; i += blockDim.x) {
    const int64_t b = blocked[i];
    if (b < 0 || b >= num_slots) {
      bad_blocked = 1;
      report(status, KVCA_ERR_BAD_INDEX, b);
    } else {
      atomicOr(bitmap + (b >> 5), 1u << (b & 31));
    }
  }
  __syncthreads();
  if (bad_blocked == 0) {
    const int rc = pop_cta<MetaT>(meta, num_slots, search_start, bitmap, count, out, order,
                                  aligned, sh);
    if (rc != KVCA_OK && threadIdx.x == 0) report(status, rc, count);
  }
}

}  // namespace
}  // namespace kvca

extern "C" int kvca_pop_reusable_slots_noalloc(int meta_bits, int order, void* d_slot_meta,
                                               int64_t num_slots, int64_t* d_search_start,
                                               const int64_t* d_blocked, int64_t num_blocked,
                                               int64_t count, int64_t* d_out, int64_t* d_status,
                                               kvca_stream_t stream) {
  if (meta_bits != 8 && meta_bits != 16) return KVCA_ERR_BAD_ARGUMENT;
  if (order != KVCA_POP_ORDER_GROUPED && order != KVCA_POP_ORDER_PREFIX)
    return KVCA_ERR_BAD_ARGUMENT;
  if (num_slots <= 0 || count < 0 || num_blocked < 0) return KVCA_ERR_BAD_ARGUMENT;
  if (num_slots > KVCA_NOALLOC_MAX_SLOTS) return KVCA_ERR_SIZE_LIMIT;
  if (count == 0) return KVCA_OK;
  // d_status is required: a bad blocked id or too few reusable slots is only
  // found on the device, and without the status pair it would go unreported.
  if (!d_slot_meta || !d_search_start || !d_out || !d_status) return KVCA_ERR_BAD_ARGUMENT;
  if (num_blocked > 0 && !d_blocked) return KVCA_ERR_BAD_ARGUMENT;
  uint32_t* bitmap = nullptr;
  if (kvca::scratch_bitmap_address(&bitmap) != cudaSuccess) return KVCA_ERR_CUDA;
  const int threads = kvca::pop_threads_for(meta_bits, num_slots);
  const bool aligned = (reinterpret_cast<uintptr_t>(d_slot_meta) & 15u) == 0u;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (meta_bits == 16) {
    kvca::pop_noalloc_kernel<uint16_t><<<1, threads, 0, s>>>(
        static_cast<uint16_t*>(d_slot_meta), num_slots, d_search_start, d_blocked, num_blocked,
        count, d_out, bitmap, order, aligned, d_status);
  } else {
    kvca::pop_noalloc_kernel<uint8_t><<<1, threads, 0, s>>>(
        static_cast<uint8_t*>(d_slot_meta), num_slots, d_search_start, d_blocked, num_blocked,
        count, d_out, bitmap, order, aligned, d_status);
  }
  return cudaGetLastError() == cudaSuccess ? KVCA_OK : KVCA_ERR_CUDA;
}
