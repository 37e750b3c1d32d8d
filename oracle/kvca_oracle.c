/*
 * kvca_oracle.c - TEST INFRASTRUCTURE ONLY.
 *
 * A sequential CPU restatement of the reference's strict (pure PyTorch) slot
 * metadata path and clock sweep, used as the checker for the CUDA kernels.
 * Only the test suite, the smoke check and the CPU-baseline leg of the
 * benchmark load it; the product never does.
 *
 * Every function follows one reference function, cited by file:line of the
 * reference project (adapter.py unless noted).  It is pinned by the
 * reference's own known-answer tests (test_adapter_npu_kernels.py:42-194)
 * and by fixtures generated from the reference itself (tests/golden/).
 *
 * Slot metadata word: pin count in the low half, usage count in the high
 * half; meta_bits 8 -> 4+4 bits in uint8, 16 -> 8+8 bits in uint16
 * (adapter.py:17-36).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OK 0
#define INSUFFICIENT 1
#define BAD_INDEX 2
#define BAD_ARGUMENT 3

typedef struct {
  int bits;        /* field width: 4 or 8 */
  uint32_t mask;   /* (1 << bits) - 1 */
  int wide;        /* 0: uint8 words, 1: uint16 words */
} codec;

static int make_codec(int meta_bits, codec* c) {
  if (meta_bits == 8) {
    c->bits = 4;
    c->wide = 0;
  } else if (meta_bits == 16) {
    c->bits = 8;
    c->wide = 1;
  } else {
    return BAD_ARGUMENT;
  }
  c->mask = (1u << c->bits) - 1u;
  return OK;
}

static uint32_t get_word(const codec* c, const void* meta, int64_t i) {
  return c->wide ? ((const uint16_t*)meta)[i] : ((const uint8_t*)meta)[i];
}

static void set_word(const codec* c, void* meta, int64_t i, uint32_t w) {
  if (c->wide) ((uint16_t*)meta)[i] = (uint16_t)w;
  else ((uint8_t*)meta)[i] = (uint8_t)w;
}

/* _slot_meta_pin_counts, adapter.py:1419-1420 */
static uint32_t pin_of(const codec* c, uint32_t w) { return w & c->mask; }
/* _slot_meta_usage_counts, adapter.py:1423-1424 */
static uint32_t usage_of(const codec* c, uint32_t w) { return (w >> c->bits) & c->mask; }
/* _pack_slot_meta, adapter.py:1427-1432 (int32 arithmetic, both fields masked) */
static uint32_t pack(const codec* c, int64_t pin, int64_t usage) {
  return ((uint32_t)((int32_t)pin) & c->mask) | (((uint32_t)((int32_t)usage) & c->mask) << c->bits);
}
/* _saturating_increment_usage, adapter.py:1414-1416 */
static uint32_t sat_inc(const codec* c, uint32_t usage) {
  return usage + 1u > c->mask ? c->mask : usage + 1u;
}

static int64_t floor_mod(int64_t a, int64_t n) {
  int64_t r = a % n;
  return r < 0 ? r + n : r;
}

/* KVCacheAdapter._inspect_load_requests strict branch, adapter.py:417-431 */
int oracle_inspect_load(int meta_bits, const int64_t* l2p, int64_t num_logical, const void* meta,
                        int64_t num_slots, const int64_t* ids, int64_t count, int64_t* cur_out,
                        uint8_t* resident_out, int64_t* pin_out, void* usage_out) {
  codec c;
  if (make_codec(meta_bits, &c)) return BAD_ARGUMENT;
  for (int64_t i = 0; i < count; ++i)
    if (ids[i] < 0 || ids[i] >= num_logical) return BAD_INDEX;
  for (int64_t i = 0; i < count; ++i) {
    const int64_t cur = l2p[ids[i]];
    if (cur >= num_slots) return BAD_INDEX;
    cur_out[i] = cur;
    resident_out[i] = cur >= 0;
    pin_out[i] = 0;
    set_word(&c, usage_out, i, 0);
    if (cur >= 0) {
      const uint32_t w = get_word(&c, meta, cur);
      pin_out[i] = (int64_t)pin_of(&c, w) + 1;
      set_word(&c, usage_out, i, sat_inc(&c, usage_of(&c, w)));
    }
  }
  return OK;
}

/* KVCacheAdapter._inspect_save_requests strict branch, adapter.py:456-470 */
int oracle_inspect_save(int meta_bits, const int64_t* l2p, int64_t num_logical, const void* meta,
                        int64_t num_slots, const int64_t* ids, int64_t count, int64_t* cur_out,
                        uint8_t* existing_out, void* usage_out) {
  codec c;
  if (make_codec(meta_bits, &c)) return BAD_ARGUMENT;
  for (int64_t i = 0; i < count; ++i)
    if (ids[i] < 0 || ids[i] >= num_logical) return BAD_INDEX;
  for (int64_t i = 0; i < count; ++i) {
    const int64_t cur = l2p[ids[i]];
    if (cur >= num_slots) return BAD_INDEX;
    cur_out[i] = cur;
    existing_out[i] = cur >= 0;
    set_word(&c, usage_out, i,
             cur >= 0 ? sat_inc(&c, usage_of(&c, get_word(&c, meta, cur))) : 1u);
  }
  return OK;
}

/*
 * KVCacheAdapter._pop_reusable_slots strict branch, adapter.py:493-525
 * (order 0, "grouped"), and the reference CUDA kernel's selection rule,
 * csrc/kv_adapter_cuda.cu:101-236 (order 1, "prefix"), over packed metadata.
 */
static int cmp_i64(const void* a, const void* b) {
  const int64_t x = *(const int64_t*)a, y = *(const int64_t*)b;
  return x < y ? -1 : x > y;
}

/* available_mask = reusable (pin == 0) minus blocked, adapter.py:493-495;
 * blocked ids are kept sorted and looked up by binary search. */
static int is_available(const codec* c, const void* meta, int64_t slot, const int64_t* blocked_sorted,
                        int64_t num_blocked) {
  if (pin_of(c, get_word(c, meta, slot)) != 0) return 0;
  return num_blocked == 0 ||
         bsearch(&slot, blocked_sorted, (size_t)num_blocked, sizeof(int64_t), cmp_i64) == NULL;
}

/* threshold_out (optional): the usage class T of the pop, -1 when nothing
 * was selected (count 0 or an error). */
static int pop_impl(int meta_bits, int order, void* meta, int64_t num_slots, int64_t* search_start,
                    const int64_t* blocked, int64_t num_blocked, int64_t count, int64_t* out,
                    int64_t* threshold_out) {
  codec c;
  if (threshold_out) *threshold_out = -1;
  if (make_codec(meta_bits, &c)) return BAD_ARGUMENT;
  if (num_slots <= 0 || count < 0) return BAD_ARGUMENT;
  if (count == 0) return OK; /* adapter.py:473-474 */
  for (int64_t b = 0; b < num_blocked; ++b)
    if (blocked[b] < 0 || blocked[b] >= num_slots) return BAD_INDEX; /* index_fill_ raises */

  int64_t* bl = NULL;
  if (num_blocked > 0) {
    bl = (int64_t*)malloc(sizeof(int64_t) * (size_t)num_blocked);
    if (!bl) return BAD_ARGUMENT;
    memcpy(bl, blocked, sizeof(int64_t) * (size_t)num_blocked);
    qsort(bl, (size_t)num_blocked, sizeof(int64_t), cmp_i64);
  }
  const int64_t start = search_start[0];
  const int64_t usage_max = (int64_t)c.mask;
  int64_t selected = 0;
  int64_t threshold = -1;

  if (order == 0) {
    /* thresholds in order; within one, scan order from search_start;
     * take until count (adapter.py:496-515) */
    for (int64_t t = 0; t <= usage_max && threshold < 0; ++t) {
      for (int64_t j = 0; j < num_slots; ++j) {
        const int64_t slot = floor_mod(start + j, num_slots);
        if (usage_of(&c, get_word(&c, meta, slot)) != (uint32_t)t) continue;
        if (!is_available(&c, meta, slot, bl, num_blocked)) continue;
        out[selected++] = slot;
        if (selected == count) {
          threshold = t;
          break;
        }
      }
    }
  } else {
    /* smallest T with #available(usage <= T) >= count, then the first
     * count available slots in scan order with usage <= T */
    int64_t eligible = 0;
    for (int64_t t = 0; t <= usage_max && threshold < 0; ++t) {
      for (int64_t i = 0; i < num_slots; ++i)
        if (usage_of(&c, get_word(&c, meta, i)) == (uint32_t)t &&
            is_available(&c, meta, i, bl, num_blocked))
          ++eligible;
      if (eligible >= count) threshold = t;
    }
    if (threshold >= 0) {
      for (int64_t j = 0; j < num_slots && selected < count; ++j) {
        const int64_t slot = floor_mod(start + j, num_slots);
        if (usage_of(&c, get_word(&c, meta, slot)) <= (uint32_t)threshold &&
            is_available(&c, meta, slot, bl, num_blocked))
          out[selected++] = slot;
      }
    }
  }
  free(bl);
  if (threshold < 0) return INSUFFICIENT; /* adapter.py:525: nothing mutated */

  if (threshold > 0) { /* global aging, adapter.py:517-522 */
    for (int64_t i = 0; i < num_slots; ++i) {
      const uint32_t w = get_word(&c, meta, i);
      const int64_t u = (int64_t)usage_of(&c, w) - threshold;
      set_word(&c, meta, i, pack(&c, pin_of(&c, w), u < 0 ? 0 : u));
    }
  }
  search_start[0] = (out[count - 1] + 1) % num_slots; /* adapter.py:523 */
  if (threshold_out) *threshold_out = threshold;
  return OK;
}

int oracle_pop(int meta_bits, int order, void* meta, int64_t num_slots, int64_t* search_start,
               const int64_t* blocked, int64_t num_blocked, int64_t count, int64_t* out) {
  return pop_impl(meta_bits, order, meta, num_slots, search_start, blocked, num_blocked, count, out,
                  NULL);
}

/* KVCacheAdapter._commit_load_metadata strict branch, adapter.py:595-604 */
int oracle_commit_load(int meta_bits, int64_t* l2p, int64_t num_logical, int64_t* p2l, void* meta,
                       int64_t num_slots, const int64_t* evicted, int64_t num_evicted,
                       const int64_t* miss_ids, const int64_t* miss_slots, int64_t num_miss,
                       const int64_t* hit_slots, const int64_t* hit_pins, const void* hit_usage,
                       int64_t num_hit, const void* miss_usage) {
  codec c;
  if (make_codec(meta_bits, &c)) return BAD_ARGUMENT;
  for (int64_t i = 0; i < num_evicted; ++i)
    if (evicted[i] < 0 || evicted[i] >= num_logical) return BAD_INDEX;
  for (int64_t i = 0; i < num_miss; ++i)
    if (miss_ids[i] < 0 || miss_ids[i] >= num_logical || miss_slots[i] < 0 ||
        miss_slots[i] >= num_slots)
      return BAD_INDEX;
  for (int64_t i = 0; i < num_hit; ++i)
    if (hit_slots[i] < 0 || hit_slots[i] >= num_slots) return BAD_INDEX;
  for (int64_t i = 0; i < num_evicted; ++i) l2p[evicted[i]] = -1;
  for (int64_t i = 0; i < num_miss; ++i) l2p[miss_ids[i]] = miss_slots[i];
  for (int64_t i = 0; i < num_miss; ++i) p2l[miss_slots[i]] = miss_ids[i];
  for (int64_t i = 0; i < num_hit; ++i)
    set_word(&c, meta, hit_slots[i], pack(&c, hit_pins[i], get_word(&c, hit_usage, i)));
  for (int64_t i = 0; i < num_miss; ++i)
    set_word(&c, meta, miss_slots[i], pack(&c, 1, get_word(&c, miss_usage, i)));
  return OK;
}

/* KVCacheAdapter._commit_save_metadata strict branch, adapter.py:647-651 */
int oracle_commit_save(int meta_bits, int64_t* l2p, int64_t num_logical, int64_t* p2l, void* meta,
                       int64_t num_slots, const int64_t* evicted, int64_t num_evicted,
                       const int64_t* ids, const int64_t* slots, const void* final_pins,
                       const void* final_usage, int64_t count) {
  codec c;
  if (make_codec(meta_bits, &c)) return BAD_ARGUMENT;
  for (int64_t i = 0; i < num_evicted; ++i)
    if (evicted[i] < 0 || evicted[i] >= num_logical) return BAD_INDEX;
  for (int64_t i = 0; i < count; ++i)
    if (ids[i] < 0 || ids[i] >= num_logical || slots[i] < 0 || slots[i] >= num_slots)
      return BAD_INDEX;
  for (int64_t i = 0; i < num_evicted; ++i) l2p[evicted[i]] = -1;
  for (int64_t i = 0; i < count; ++i) l2p[ids[i]] = slots[i];
  for (int64_t i = 0; i < count; ++i) p2l[slots[i]] = ids[i];
  for (int64_t i = 0; i < count; ++i)
    set_word(&c, meta, slots[i],
             pack(&c, get_word(&c, final_pins, i), get_word(&c, final_usage, i)));
  return OK;
}

/* KVCacheAdapter.release strict branch, adapter.py:332-336: new values are
 * computed from one snapshot, then written (index_select, then index_put_). */
int oracle_release(int meta_bits, const int64_t* l2p, int64_t num_logical, void* meta,
                   int64_t num_slots, const int64_t* ids, int64_t count) {
  codec c;
  if (make_codec(meta_bits, &c)) return BAD_ARGUMENT;
  for (int64_t i = 0; i < count; ++i) {
    if (ids[i] < 0 || ids[i] >= num_logical) return BAD_INDEX;
    if (l2p[ids[i]] < 0 || l2p[ids[i]] >= num_slots) return BAD_INDEX;
  }
  uint32_t* next = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(count > 0 ? count : 1));
  if (!next) return BAD_ARGUMENT;
  for (int64_t i = 0; i < count; ++i) {
    const uint32_t w = get_word(&c, meta, l2p[ids[i]]);
    /* uint pin - 1 wraps, then the pack masks it to the field width */
    next[i] = pack(&c, (int64_t)pin_of(&c, w) - 1, usage_of(&c, w));
  }
  for (int64_t i = 0; i < count; ++i) set_word(&c, meta, l2p[ids[i]], next[i]);
  free(next);
  return OK;
}

/*
 * Clock stream: steps of pop (no blocked slots) -> refill the victims with
 * usage 1 keeping their pin (the save-miss commit, adapter.py:233-242 and
 * :647-651) -> usage bump of re-accessed slots from one snapshot
 * (adapter.py:1414-1416 applied through index_put_).  Returns the status of
 * the first failing step; *steps_done counts completed steps.
 */
/* step_threshold (optional, num_steps entries): each completed step's usage
 * class T (T > 0: that pop aged every slot), for the workload's algorithmic
 * byte count. */
int oracle_clock_stream_traced(int meta_bits, int order, void* meta, int64_t num_slots,
                               int64_t* search_start, int64_t num_steps, int64_t alloc_per_step,
                               const int64_t* reaccess, int64_t reaccess_per_step,
                               int64_t* victims, int64_t* steps_done, int8_t* step_threshold) {
  codec c;
  if (make_codec(meta_bits, &c)) return BAD_ARGUMENT;
  uint32_t* next = (uint32_t*)malloc(sizeof(uint32_t) *
                                     (size_t)(reaccess_per_step > 0 ? reaccess_per_step : 1));
  if (!next) return BAD_ARGUMENT;
  int rc = OK;
  int64_t step = 0;
  for (; step < num_steps; ++step) {
    int64_t* out = victims + step * alloc_per_step;
    int64_t t = -1;
    rc = pop_impl(meta_bits, order, meta, num_slots, search_start, NULL, 0, alloc_per_step, out, &t);
    if (rc != OK) break;
    if (step_threshold) step_threshold[step] = (int8_t)(t > 127 ? 127 : t);
    for (int64_t i = 0; i < alloc_per_step; ++i)
      set_word(&c, meta, out[i], pack(&c, pin_of(&c, get_word(&c, meta, out[i])), 1));
    const int64_t* ids = reaccess + step * reaccess_per_step;
    for (int64_t i = 0; i < reaccess_per_step; ++i) {
      if (ids[i] < 0 || ids[i] >= num_slots) {
        rc = BAD_INDEX;
        break;
      }
      const uint32_t w = get_word(&c, meta, ids[i]);
      next[i] = pack(&c, pin_of(&c, w), sat_inc(&c, usage_of(&c, w)));
    }
    if (rc != OK) break;
    for (int64_t i = 0; i < reaccess_per_step; ++i) set_word(&c, meta, ids[i], next[i]);
  }
  free(next);
  *steps_done = step;
  return rc;
}

int oracle_clock_stream(int meta_bits, int order, void* meta, int64_t num_slots,
                        int64_t* search_start, int64_t num_steps, int64_t alloc_per_step,
                        const int64_t* reaccess, int64_t reaccess_per_step, int64_t* victims,
                        int64_t* steps_done) {
  return oracle_clock_stream_traced(meta_bits, order, meta, num_slots, search_start, num_steps,
                                    alloc_per_step, reaccess, reaccess_per_step, victims,
                                    steps_done, NULL);
}
