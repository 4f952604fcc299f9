// Residency decisions of an over-budget expert slot cache, host only.
//
// num_slots device slots hold (layer, expert) weights; hn_slots_admit makes
// one call's experts resident and says which slots to load, evicting among
// the slots the call does not need: the least frequently used (a use count
// per (layer, expert) that halves every decay_every uses, ties to the least
// recently used), or the least recently used.  The reference keeps this
// bookkeeping in Python per layer (cache/expert_cache.py); here it is one
// table for all layers, behind the C ABI.
#include <algorithm>
#include <mutex>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "common.cuh"

struct hn_slots {
  int S;
  int policy;  // HN_SLOTS_LFU / HN_SLOTS_LRU
  int64_t decay_every;
  int64_t clock = 0;
  std::vector<int64_t> owner;     // key per slot, -1 free
  std::vector<int64_t> last_use;  // clock of the last use per slot
  std::unordered_map<int64_t, int> where;
  std::unordered_map<int64_t, double> freq;
  int64_t hits = 0, misses = 0, evictions = 0;
  std::mutex mu;
};

namespace {
int64_t key_of(int layer, int expert) { return ((int64_t)layer << 32) | (uint32_t)expert; }
}  // namespace

extern "C" {

hn_slots* hn_slots_create(int num_slots, int policy, int64_t decay_every) {
  if (num_slots < 1 || (policy != HN_SLOTS_LFU && policy != HN_SLOTS_LRU) || decay_every < 1) return nullptr;
  hn_slots* s = new hn_slots();
  s->S = num_slots;
  s->policy = policy;
  s->decay_every = decay_every;
  s->owner.assign(num_slots, -1);
  s->last_use.assign(num_slots, 0);
  return s;
}

void hn_slots_destroy(hn_slots* s) { delete s; }

int hn_slots_admit(hn_slots* s, int layer, const int32_t* experts, int n, int32_t* loads, int32_t* evicted,
                   int* n_evicted) {
  if (!s || n < 0 || (n > 0 && !experts) || !loads || !evicted || !n_evicted) return -HN_ERR_INVALID;
  std::lock_guard<std::mutex> lock(s->mu);
  std::vector<int> es;
  for (int i = 0; i < n; ++i)
    if (experts[i] >= 0) es.push_back(experts[i]);
  std::sort(es.begin(), es.end());
  es.erase(std::unique(es.begin(), es.end()), es.end());
  if ((int)es.size() > s->S) return -HN_ERR_WORKSPACE;  // nothing changes
  std::unordered_set<int64_t> keep;
  for (int e : es) keep.insert(key_of(layer, e));
  int nl = 0, ne = 0;
  for (int e : es) {
    const int64_t key = key_of(layer, e);
    s->clock += 1;
    s->freq[key] += 1.0;
    if (s->clock % s->decay_every == 0) {
      for (auto it = s->freq.begin(); it != s->freq.end();) {
        if (it->second < 1.0 / 64) {
          it = s->freq.erase(it);
        } else {
          it->second *= 0.5;
          ++it;
        }
      }
    }
    const auto hit = s->where.find(key);
    if (hit != s->where.end()) {
      s->hits += 1;
      s->last_use[hit->second] = s->clock;
      continue;
    }
    s->misses += 1;
    int victim = -1;
    for (int q = 0; q < s->S && victim < 0; ++q)
      if (s->owner[q] < 0) victim = q;
    if (victim < 0) {
      double best_f = 0.0;
      int64_t best_t = 0;
      for (int q = 0; q < s->S; ++q) {
        if (keep.count(s->owner[q])) continue;
        const auto fi = s->freq.find(s->owner[q]);
        const double f = s->policy == HN_SLOTS_LFU ? (fi == s->freq.end() ? 0.0 : fi->second) : 0.0;
        const int64_t t = s->last_use[q];
        if (victim < 0 || f < best_f || (f == best_f && t < best_t)) {
          victim = q;
          best_f = f;
          best_t = t;
        }
      }
    }
    // a victim exists: the call needs at most S experts and keeps only its own
    const int64_t old = s->owner[victim];
    if (old >= 0) {
      s->evictions += 1;
      s->where.erase(old);
      evicted[2 * ne] = (int32_t)(old >> 32);
      evicted[2 * ne + 1] = (int32_t)(old & 0xffffffff);
      ++ne;
    }
    s->owner[victim] = key;
    s->where[key] = victim;
    s->last_use[victim] = s->clock;
    loads[2 * nl] = victim;
    loads[2 * nl + 1] = e;
    ++nl;
  }
  *n_evicted = ne;
  return nl;
}

int hn_slots_lookup(hn_slots* s, int layer, int expert) {
  if (!s) return -1;
  std::lock_guard<std::mutex> lock(s->mu);
  const auto it = s->where.find(key_of(layer, expert));
  return it == s->where.end() ? -1 : it->second;
}

int hn_slots_stats(hn_slots* s, int64_t* out3) {
  if (!s || !out3) return HN_ERR_INVALID;
  std::lock_guard<std::mutex> lock(s->mu);
  out3[0] = s->hits;
  out3[1] = s->misses;
  out3[2] = s->evictions;
  return HN_OK;
}

}  // extern "C"
