// Host-side bookkeeping of host-streamed experts: which (layer, expert) each
// HBM slot holds, which expert a call evicts (LRU or LFRU), the scratch slots
// that serve experts the cache does not admit, and router-lookahead prefetch.
// It restates ExpertStore's cache (crates/kestrel-memory/src/expert.rs):
//   score / victim / admit / touch   expert.rs:305-356
//   get                              expert.rs:358-424 (one demand use)
//   prefetch (+ speculative pool)    expert.rs:451-521
//   request                          expert.rs:523-537
//   record_lookahead / decay         expert.rs:539-551
// and the order Transformer::moe_ffn visits a call's experts (ready ones
// first, transformer.rs:530-534).
//
// No CUDA here: the caller (api.cu) performs the copies a plan lists, tells
// the cache when a prefetch copy has landed (mark_done), and the policy is
// unit-tested on the CPU.
//
// Differences from the reference, all forced by one GPU launch serving every
// expert of a call at once:
// * the experts of the current call are never victims of its own admissions
//   (the reference may evict a needed expert between two `get`s);
// * when the call's non-admitted experts outnumber the scratch slots, the
//   rest are admitted by force (LRU victim) instead of waiting for a scratch
//   buffer;
// * the speculative pool has its own slots (after the scratch slots), and a
//   slot a demand call read is not reloaded before that call's kernels end.
#pragma once

#include <algorithm>
#include <cstdint>
#include <unordered_map>
#include <vector>

namespace kc {

enum class ExpertPolicy { Lfru = 0, Lru = 1 };  // expert.rs:35-38

// Counters of ExpertMetrics (expert.rs:127-153) that apply here.
struct ExpertCacheStats {
  uint64_t requests = 0, hits = 0, late = 0, misses = 0, scratch_loads = 0, bytes_read = 0;
  uint64_t prefetch_issued = 0, prefetch_used = 0, prefetch_wasted = 0, evictions = 0;
  uint64_t lookahead_predicted = 0, lookahead_correct = 0, reads = 0, forced = 0, spec_pauses = 0;
};

class ExpertCache {
 public:
  struct Load {
    int expert;
    int slot;
  };

  // Slots: cache [0, capacity), scratch [capacity, capacity + scratch),
  // speculative pool [capacity + scratch, + spec). Clears all state.
  void configure(int capacity, int scratch, int spec, ExpertPolicy policy) {
    capacity_ = std::max(0, capacity);
    scratch_ = std::max(0, scratch);
    spec_n_ = std::max(0, spec);
    policy_ = policy;
    slots_.assign(capacity_, Slot{});
    spec_.clear();
    spec_slot_.assign(spec_n_, SpecSlot{});
    spec_issued_ = spec_used_ = spec_paused_ = 0;
    where_.clear();
    heat_.clear();
    last_.clear();
    clock_ = 0;
    call_ = 0;
    n_cached_ = 0;
    stats_ = ExpertCacheStats{};
  }
  int capacity() const { return capacity_; }
  int scratch() const { return scratch_; }
  int spec() const { return spec_n_; }
  int slots() const { return capacity_ + scratch_ + spec_n_; }
  int cached() const { return n_cached_; }
  const ExpertCacheStats& stats() const { return stats_; }
  void add_bytes(uint64_t bytes, uint64_t reads) {
    stats_.bytes_read += bytes;
    stats_.reads += reads;
  }

  // Slot holding (layer, e), or -1.
  int slot_of(int layer, int e) const {
    auto it = where_.find(key(layer, e));
    return it == where_.end() ? -1 : it->second;
  }
  // Whether slot s (cache or speculative) still waits for a prefetch copy.
  bool pending(int s) const {
    if (s >= 0 && s < capacity_) return slots_[s].pending;
    const int i = s - capacity_ - scratch_;
    return i >= 0 && i < spec_n_ && spec_slot_[i].pending;
  }
  // The prefetch copy into slot s has landed (ExpertBuf's ticket done).
  void mark_done(int s) {
    if (s >= 0 && s < capacity_) slots_[s].pending = false;
    const int i = s - capacity_ - scratch_;
    if (i >= 0 && i < spec_n_) spec_slot_[i].pending = false;
  }

  // One MoE call of `layer` over the batch union `experts` (ascending ids,
  // no repeats): ExpertStore::request for all of them, then ExpertStore::get
  // for each in Transformer::moe_ffn's order. slot_out[i] receives the slot
  // of experts[i]; `loads` the copies to issue before the call's kernels run
  // (each expert into its slot); `waits` the cache slots the call reads while
  // their prefetch copy may be in flight. Returns false when the slots cannot
  // hold the call's experts at once (capacity + scratch too small); the
  // experts the call admitted are then dropped again.
  bool demand(int layer, const int* experts, int n, int* slot_out, std::vector<Load>& loads,
              std::vector<int>& waits) {
    loads.clear();
    waits.clear();
    ++call_;
    need_.assign(experts, experts + n);
    cur_layer_ = layer;
    std::vector<char> demanded(n, 0);
    // ExpertStore::request: admit the missing ones (their miss counted now).
    for (int i = 0; i < n; ++i) {
      const uint64_t k = key(layer, experts[i]);
      if (where_.count(k)) continue;
      const int s = admit(k, false, false);
      if (s >= 0) {
        ++stats_.misses;
        demanded[i] = 1;
        loads.push_back({experts[i], s});
      }
    }
    // Transformer::moe_ffn: experts that are ready first, then the others,
    // each in ascending id order (a stable sort on "not ready").
    std::vector<int> order;
    order.reserve(n);
    for (int pass = 0; pass < 2; ++pass)
      for (int i = 0; i < n; ++i) {
        auto it = where_.find(key(layer, experts[i]));
        const bool ready = it != where_.end() && !demanded[i] && !slots_[it->second].pending;
        if (ready == (pass == 0)) order.push_back(i);
      }
    int next_scratch = capacity_;
    for (int i : order) {
      const uint64_t k = key(layer, experts[i]);
      ++stats_.requests;
      touch(k);
      auto it = where_.find(k);
      if (it != where_.end()) {
        Slot& sl = slots_[it->second];
        if (sl.prefetched) {
          sl.prefetched = false;
          ++stats_.prefetch_used;
        }
        if (demanded[i]) {
          // counted as a miss by the request phase
        } else if (!sl.pending) {
          ++stats_.hits;
        } else {
          ++stats_.late;
          waits.push_back(it->second);
        }
        sl.call = call_;
        slot_out[i] = it->second;
        continue;
      }
      // Predicted by lookahead but not cached: served from the speculative
      // pool (expert.rs:377-388); the slot is free again once this call ends.
      const int si = spec_find(k);
      if (si >= 0) {
        const int s = spec_[si].slot;
        spec_[si] = spec_.back();  // Vec::swap_remove
        spec_.pop_back();
        ++spec_used_;
        ++stats_.prefetch_used;
        SpecSlot& ss = spec_slot_[s - capacity_ - scratch_];
        ss.held = false;
        ss.call = call_;
        if (!ss.pending) {
          ++stats_.hits;
        } else {
          ++stats_.late;
          waits.push_back(s);
        }
        slot_out[i] = s;
        continue;
      }
      ++stats_.misses;
      int s = admit(k, false, false);
      if (s < 0) {
        if (next_scratch < capacity_ + scratch_) {
          ++stats_.scratch_loads;
          slot_out[i] = next_scratch;
          loads.push_back({experts[i], next_scratch++});
          continue;
        }
        s = admit(k, false, true);
        if (s < 0) {
          // Nothing is copied for a failed call: the experts it admitted
          // leave the cache again (its victims stay evicted).
          for (const Load& ld : loads)
            if (ld.slot < capacity_) {
              where_.erase(slots_[ld.slot].k);
              slots_[ld.slot] = Slot{};
              --n_cached_;
            }
          loads.clear();
          waits.clear();
          need_.clear();
          cur_layer_ = -1;
          return false;
        }
        ++stats_.forced;
      }
      slots_[s].call = call_;
      slot_out[i] = s;
      loads.push_back({experts[i], s});
    }
    for (int i = 0; i < n; ++i)
      if (slot_out[i] < capacity_) slots_[slot_out[i]].call = call_;
    need_.clear();
    cur_layer_ = -1;
    return true;
  }

  // ExpertStore::prefetch: start loading predicted experts of `layer` that
  // are not cached, if the cache admits them (by their current heat; a guess
  // is not touched). Experts of the latest demand call (its kernels may still
  // run) and slots still being filled are not victims.
  void prefetch(int layer, const int* experts, int n, std::vector<Load>& loads) {
    loads.clear();
    for (int i = 0; i < n; ++i) {
      const uint64_t k = key(layer, experts[i]);
      if (where_.count(k)) continue;
      const int s = admit(k, true, false);
      if (s >= 0) {
        ++stats_.prefetch_issued;
        slots_[s].pending = true;
        loads.push_back({experts[i], s});
        continue;
      }
      // Not admissible: load into the speculative pool instead, never
      // displacing a cached expert, while the pool pays off.
      if (spec_paused_ > 0) {
        if (--spec_paused_ == 0) spec_issued_ = spec_used_ = 0;  // re-probe
        continue;
      }
      if (spec_n_ == 0 || spec_find(k) >= 0) continue;
      if (spec_issued_ >= 128) {
        const double acc = (double)spec_used_ / (double)spec_issued_;
        spec_issued_ = spec_used_ = 0;
        if (acc < kSpecMinAccuracy) {
          ++stats_.spec_pauses;
          spec_paused_ = 4096;
          continue;
        }
      }
      int slot = -1;
      if ((int)spec_.size() < spec_n_) {
        // A pool slot no prediction holds and no call in flight reads.
        for (int j = 0; j < spec_n_ && slot < 0; ++j)
          if (!spec_slot_[j].held && spec_slot_[j].call != call_) slot = capacity_ + scratch_ + j;
      } else {
        // Replace the oldest speculative load whose copy has landed (a stale
        // prediction).
        for (size_t j = 0; j < spec_.size(); ++j)
          if (!spec_slot_[spec_[j].slot - capacity_ - scratch_].pending) {
            ++stats_.prefetch_wasted;
            slot = spec_[j].slot;
            spec_.erase(spec_.begin() + j);  // Vec::remove
            break;
          }
      }
      if (slot < 0) continue;
      SpecSlot& ss = spec_slot_[slot - capacity_ - scratch_];
      ss.held = true;
      ss.pending = true;
      spec_.push_back({k, slot});
      ++spec_issued_;
      ++stats_.prefetch_issued;
      loads.push_back({experts[i], slot});
    }
  }

  void record_lookahead(uint64_t predicted, uint64_t correct) {
    stats_.lookahead_predicted += predicted;
    stats_.lookahead_correct += correct;
  }

  // Halve all heat so placement follows the workload (expert.rs:545-551).
  void decay() {
    for (auto it = heat_.begin(); it != heat_.end();) {
      it->second >>= 1;
      if (it->second == 0)
        it = heat_.erase(it);
      else
        ++it;
    }
  }

  // Heat and last use of (layer, e), for tests.
  uint32_t heat(int layer, int e) const {
    auto it = heat_.find(key(layer, e));
    return it == heat_.end() ? 0 : it->second;
  }
  uint64_t last(int layer, int e) const {
    auto it = last_.find(key(layer, e));
    return it == last_.end() ? 0 : it->second;
  }

 private:
  struct Slot {
    bool used = false;        // holds an expert
    uint64_t k = 0;           // which (layer << 32 | e)
    bool prefetched = false;  // loaded by prefetch and not yet used
    bool pending = false;     // prefetch copy possibly still in flight
    uint64_t call = 0;        // latest demand call that reads it
  };

  struct Spec {
    uint64_t k;
    int slot;
  };
  struct SpecSlot {
    bool held = false;     // holds a prediction listed in spec_
    bool pending = false;  // its copy possibly still in flight
    uint64_t call = 0;     // latest demand call that read it
  };
  static constexpr double kSpecMinAccuracy = 0.5;  // ExpertStore::spec_min_accuracy's default

  static uint64_t key(int layer, int e) { return ((uint64_t)(uint32_t)layer << 32) | (uint32_t)e; }

  int spec_find(uint64_t k) const {
    for (size_t j = 0; j < spec_.size(); ++j)
      if (spec_[j].k == k) return (int)j;
    return -1;
  }

  uint64_t score(uint64_t k) const {
    auto li = last_.find(k);
    const uint64_t last = li == last_.end() ? 0 : li->second;
    if (policy_ == ExpertPolicy::Lru) return last;
    auto hi = heat_.find(k);
    const uint64_t heat = hi == heat_.end() ? 0 : hi->second;
    const uint64_t age = clock_ - last;
    return (heat << 8) | (age >= 255 ? 0 : 255 - age);
  }

  void touch(uint64_t k) {
    ++clock_;
    uint32_t& h = heat_[k];
    if (h != UINT32_MAX) ++h;
    last_[k] = clock_;
  }

  // Victim slot for admitting k, or -1 (expert.rs:321-331). Evictable: a
  // cached expert whose copy has landed, not needed by the current demand
  // call, and (for a prefetch) not read by the latest demand call.
  int victim(uint64_t k, bool prefetch, bool force) const {
    int best = -1;
    uint64_t best_score = 0;
    for (int s = 0; s < capacity_; ++s) {
      const Slot& sl = slots_[s];
      if (!sl.used || sl.pending) continue;
      if (prefetch && sl.call == call_) continue;
      if (!prefetch && is_needed(sl.k)) continue;
      const uint64_t sc = score(sl.k);
      if (best < 0 || sc < best_score) {
        best = s;
        best_score = sc;
      }
    }
    if (best < 0) return -1;
    if (force || policy_ == ExpertPolicy::Lru) return best;
    const uint64_t hs = score(k);
    return hs > best_score + (best_score >> 2) + (4u << 8) ? best : -1;
  }

  // Whether k is one of the current demand call's experts (need_ ascending).
  bool is_needed(uint64_t k) const {
    return (int)(k >> 32) == cur_layer_ && std::binary_search(need_.begin(), need_.end(), (int)(uint32_t)k);
  }

  // Insert k into a free or evicted cache slot; returns it or -1
  // (expert.rs:333-356).
  int admit(uint64_t k, bool prefetch, bool force) {
    int s = -1;
    if (n_cached_ < capacity_) {
      for (int i = 0; i < capacity_; ++i)
        if (!slots_[i].used) {
          s = i;
          break;
        }
      ++n_cached_;
    } else {
      s = victim(k, prefetch, force);
      if (s < 0) return -1;
      Slot& old = slots_[s];
      where_.erase(old.k);
      ++stats_.evictions;
      if (old.prefetched) ++stats_.prefetch_wasted;
    }
    Slot& sl = slots_[s];
    sl = Slot{};
    sl.used = true;
    sl.k = k;
    sl.prefetched = prefetch;
    where_[k] = s;
    return s;
  }

  int capacity_ = 0, scratch_ = 0, spec_n_ = 0;
  std::vector<Spec> spec_;           // speculative loads, oldest first
  std::vector<SpecSlot> spec_slot_;  // [spec_n_]
  uint64_t spec_issued_ = 0, spec_used_ = 0, spec_paused_ = 0;  // the pool's accuracy window
  ExpertPolicy policy_ = ExpertPolicy::Lfru;
  std::vector<Slot> slots_;
  std::unordered_map<uint64_t, int> where_;
  std::unordered_map<uint64_t, uint32_t> heat_;
  std::unordered_map<uint64_t, uint64_t> last_;
  uint64_t clock_ = 0, call_ = 0;
  int n_cached_ = 0;
  std::vector<int> need_;  // experts of the current demand call (of cur_layer_)
  int cur_layer_ = -1;
  ExpertCacheStats stats_;
};

}  // namespace kc
