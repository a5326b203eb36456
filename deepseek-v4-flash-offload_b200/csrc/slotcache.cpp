// LRU slot cache of the expert bank (host bookkeeping only).
//
// The reference keeps its packed-expert cache in a Python OrderedDict that
// ExpertBank.get_packed walks once per expert per layer (offload.py:103-129):
// a hit moves the key to the most-recently-used end, a miss inserts it and
// evicts from the least-recently-used end while over capacity.  Here the
// cache maps (layer, expert) to a slot of the device arena and serves a whole
// layer's batch of experts in one call: the keys of one batch must be
// resident together, so a miss never evicts another key of the same batch.
// The caller copies the weights of each missed key into its slot (one
// cudaMemcpyAsync of the packed slot, on its copy stream, after the kernels
// that last read the slot).
#include <stdint.h>

#include <list>
#include <new>
#include <unordered_map>
#include <unordered_set>
#include <utility>
#include <vector>

#include "capi_internal.h"

namespace {

struct Key {
  int64_t layer, expert;
  bool operator==(const Key& o) const { return layer == o.layer && expert == o.expert; }
};
struct KeyHash {
  size_t operator()(const Key& k) const {
    return std::hash<int64_t>()(k.layer * 1000003 + k.expert);
  }
};

}  // namespace

struct dsv4_slotcache {
  int64_t capacity = 0;
  std::list<std::pair<Key, int32_t>> order;   // least recently used first
  std::unordered_map<Key, std::list<std::pair<Key, int32_t>>::iterator, KeyHash> where;
  std::vector<int32_t> free_slots;             // taken from the back: slot 0 first
  int64_t hits = 0, misses = 0, evictions = 0;

  void reset_free() {
    free_slots.clear();
    for (int64_t s = capacity - 1; s >= 0; --s) free_slots.push_back((int32_t)s);
  }
};

extern "C" int dsv4_slotcache_create(dsv4_slotcache** out, int64_t n_slots) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(out, "null pointer");
  DSV4_CHECK_ARG(n_slots >= 0 && n_slots <= INT32_MAX, "n_slots must be in [0, 2^31)");
  dsv4_slotcache* c = new (std::nothrow) dsv4_slotcache();
  if (!c) return ::dsv4::fail(DSV4_ENOMEM, "dsv4_slotcache_create: out of host memory");
  c->capacity = n_slots;
  c->reset_free();
  *out = c;
  DSV4_API_END
}

extern "C" int dsv4_slotcache_destroy(dsv4_slotcache* c) {
  delete c;
  return DSV4_OK;
}

extern "C" int dsv4_slotcache_lookup(dsv4_slotcache* c, const int64_t* layer, const int64_t* expert, int64_t n,
                                     int32_t* slot_out, uint8_t* miss_out) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(c, "null cache");
  DSV4_CHECK_ARG(n >= 0, "n must be >= 0");
  DSV4_CHECK_ARG(n == 0 || (layer && expert && slot_out && miss_out), "null pointer");
  std::unordered_set<Key, KeyHash> batch;
  batch.reserve((size_t)n * 2 + 1);
  for (int64_t i = 0; i < n; ++i) batch.insert(Key{layer[i], expert[i]});
  if ((int64_t)batch.size() > c->capacity)
    return ::dsv4::fail(DSV4_ENOMEM, std::to_string(batch.size()) + " experts needed at once but only " +
                                         std::to_string(c->capacity) + " slots");
  for (int64_t i = 0; i < n; ++i) {
    const Key k{layer[i], expert[i]};
    auto it = c->where.find(k);
    if (it != c->where.end()) {
      ++c->hits;
      c->order.splice(c->order.end(), c->order, it->second);   // to the MRU end
      slot_out[i] = it->second->second;
      miss_out[i] = 0;
      continue;
    }
    ++c->misses;
    int32_t s;
    if (!c->free_slots.empty()) {
      s = c->free_slots.back();
      c->free_slots.pop_back();
    } else {
      // the least recently used key outside this batch; one exists because
      // the batch has at most `capacity` distinct keys and this one is new
      auto v = c->order.begin();
      while (batch.count(v->first)) ++v;
      s = v->second;
      c->where.erase(v->first);
      c->order.erase(v);
      ++c->evictions;
    }
    c->order.emplace_back(k, s);
    c->where[k] = std::prev(c->order.end());
    slot_out[i] = s;
    miss_out[i] = 1;
  }
  DSV4_API_END
}

extern "C" int32_t dsv4_slotcache_slot_of(const dsv4_slotcache* c, int64_t layer, int64_t expert) {
  if (!c) return -1;
  auto it = c->where.find(Key{layer, expert});
  return it == c->where.end() ? -1 : it->second->second;
}

extern "C" int dsv4_slotcache_stats(const dsv4_slotcache* c, int64_t* out4) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(c && out4, "null pointer");
  out4[0] = c->hits;
  out4[1] = c->misses;
  out4[2] = c->evictions;
  out4[3] = (int64_t)c->where.size();
  DSV4_API_END
}

extern "C" int dsv4_slotcache_snapshot(const dsv4_slotcache* c, int64_t* layer_out, int64_t* expert_out,
                                       int32_t* slot_out, int64_t cap, int64_t* n_out) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(c && n_out, "null pointer");
  DSV4_CHECK_ARG(cap >= 0 && (cap == 0 || (layer_out && expert_out && slot_out)), "bad output buffers");
  int64_t i = 0;
  for (const auto& e : c->order) {
    if (i >= cap) break;
    layer_out[i] = e.first.layer;
    expert_out[i] = e.first.expert;
    slot_out[i] = e.second;
    ++i;
  }
  *n_out = (int64_t)c->where.size();
  DSV4_API_END
}

extern "C" int dsv4_slotcache_clear(dsv4_slotcache* c) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(c, "null cache");
  c->order.clear();
  c->where.clear();
  c->reset_free();
  DSV4_API_END
}
