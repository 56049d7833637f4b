// Host-side bookkeeping of the steady-state caches, kept by the library next to the device pools it indexes.
//
// The reference keeps this in Python (engine/runtime/dit_fast.py:58-97 SlotPool / FastCache, :480-490 the order and
// trim after a solve).  Here it is native: a request's caches are a handle into a registry, pool slots come from a
// bitmap allocator, and a steady-state call builds its key lists from the records and updates them after enqueueing
// the solve, so the host does no per-key work in Python.
//
// What must stay as the reference has it (the interface of the drop-in): a cache keeps, per CFG row, its key slots in
// the reference's tensor order (each kept window's keys in front of the older ones: the reference concatenates
// [new, cache]), and after a kept window the order is cut to its first `keep` entries plus its last 100
// (token2wav_batch.py:33-39); `length` and `keep` are what the engine reads and sets.  Slot ids themselves are
// arbitrary: attention sees the set of keys, so allocation order never changes a result.
#pragma once

#include <stdint.h>

#include <vector>

namespace t2w {

constexpr int kTrimSuffix = 100;  // keys kept after the first `keep` (the reference's TRIM_SUFFIX)

// Pool slot ids 0 .. n-1 as a bitmap (bit set = in use), searched from a rotating word cursor so consecutive
// allocations walk the pool instead of rescanning its used head.  ids below `reserved` are never handed out.
class SlotBitmap {
 public:
  void init(int n, int reserved) {
    n_ = n;
    words_.assign((size_t)(n + 63) / 64, 0ull);
    for (int i = n; i < (int)words_.size() * 64; ++i) words_[i >> 6] |= 1ull << (i & 63);  // bits past the end
    for (int i = 0; i < reserved && i < n; ++i) words_[i >> 6] |= 1ull << (i & 63);
    reserved_ = reserved < n ? reserved : n;
    used_ = reserved_;
    cursor_ = 0;
  }
  int size() const { return n_; }
  int used() const { return used_ - reserved_; }  // handed out (reserved ids not counted)
  int available() const { return n_ - used_; }
  // k ids into out[0 .. k), all or nothing.
  bool take(int k, int32_t* out) {
    if (k < 0 || k > available()) return false;
    const size_t nw = words_.size();
    int got = 0;
    for (size_t step = 0; got < k && step < nw; ++step) {
      const size_t w = (cursor_ + step) % nw;
      uint64_t freebits = ~words_[w];
      while (freebits && got < k) {
        const int b = __builtin_ctzll(freebits);
        freebits &= freebits - 1;
        words_[w] |= 1ull << b;
        out[got++] = (int32_t)(w * 64 + b);
      }
      if (got == k) cursor_ = w;
    }
    used_ += got;
    return got == k;  // always true given the count check above
  }
  bool owned(int32_t id) const {
    return id >= reserved_ && id < n_ && (words_[id >> 6] >> (id & 63) & 1ull);
  }
  void give(const int32_t* ids, size_t k) {
    for (size_t i = 0; i < k; ++i) {
      const int32_t id = ids[i];
      words_[id >> 6] &= ~(1ull << (id & 63));
    }
    used_ -= (int)k;
  }

 private:
  std::vector<uint64_t> words_;
  int n_ = 0, used_ = 0, reserved_ = 0;
  size_t cursor_ = 0;
};

// One request's caches: for each CFG row (0 conditional, 1 unconditional) its key slots in the reference's order and
// its conv-cache row slot; `keep` is the trim length (the prompt's mel frames).
struct CacheRecord {
  bool live = false;
  uint32_t generation = 0;
  int32_t keep = 0;
  int32_t rowslot[2] = {-1, -1};
  std::vector<int32_t> keys[2];
};

// Handles are (generation << kIndexBits) | index, so a released handle that is used again is recognised as stale.
class CacheRegistry {
 public:
  static constexpr int kIndexBits = 20;
  static constexpr uint32_t kIndexMask = (1u << kIndexBits) - 1;

  void init(int n_slots, int n_rowslots) {
    slots.init(n_slots, 0);
    rows.init(n_rowslots, 1);  // row slot 0: the write target of rows that keep nothing
    recs_.clear();
    vacant_.clear();
  }
  // A new empty record with both row slots taken; -1 when the records or row slots are exhausted.
  int32_t open() {
    int32_t rs[2];
    if (!rows.take(2, rs)) return -1;
    uint32_t idx;
    if (!vacant_.empty()) {
      idx = vacant_.back();
      vacant_.pop_back();
    } else {
      if (recs_.size() > kIndexMask) {
        rows.give(rs, 2);
        return -1;
      }
      idx = (uint32_t)recs_.size();
      recs_.emplace_back();
    }
    CacheRecord& r = recs_[idx];
    r.live = true;
    r.generation = (r.generation + 1) & ((1u << (31 - kIndexBits)) - 1);
    r.keep = 0;
    r.rowslot[0] = rs[0];
    r.rowslot[1] = rs[1];
    r.keys[0].clear();
    r.keys[1].clear();
    return (int32_t)((r.generation << kIndexBits) | idx);
  }
  CacheRecord* find(int32_t handle) {
    if (handle < 0) return nullptr;
    const uint32_t idx = (uint32_t)handle & kIndexMask, gen = (uint32_t)handle >> kIndexBits;
    if (idx >= recs_.size()) return nullptr;
    CacheRecord& r = recs_[idx];
    return (r.live && r.generation == gen) ? &r : nullptr;
  }
  // Return every slot of the record to the pools and retire the handle.
  void close(int32_t handle) {
    CacheRecord* r = find(handle);
    if (!r) return;
    for (int h = 0; h < 2; ++h) {
      slots.give(r->keys[h].data(), r->keys[h].size());
      r->keys[h].clear();
    }
    rows.give(r->rowslot, 2);
    r->rowslot[0] = r->rowslot[1] = -1;
    r->live = false;
    vacant_.push_back((uint32_t)handle & kIndexMask);
  }
  int live() const { return (int)(recs_.size() - vacant_.size()); }

  // After a kept window: the window's new slots go in front of the row's order, then the order is cut to its first
  // `keep` and last kTrimSuffix entries; the cut slots return to the pool.
  void commit_window(CacheRecord& r, int h, const int32_t* fresh, int n_fresh) {
    std::vector<int32_t>& k = r.keys[h];
    k.insert(k.begin(), fresh, fresh + n_fresh);
    const int keep = r.keep < 0 ? 0 : r.keep;
    if ((long long)k.size() > (long long)keep + kTrimSuffix) {
      const size_t cut0 = (size_t)keep, cut1 = k.size() - kTrimSuffix;
      slots.give(k.data() + cut0, cut1 - cut0);
      k.erase(k.begin() + cut0, k.begin() + cut1);
    }
  }

  SlotBitmap slots;  // key slots of the K/V pool
  SlotBitmap rows;   // conv-cache row slots

 private:
  std::vector<CacheRecord> recs_;
  std::vector<uint32_t> vacant_;
};

}  // namespace t2w
