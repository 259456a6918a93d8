// Prefix-cache index in C++ (host code): the chained exact-content block keys
// and the key -> cached-blocks map behind BlockManager's prefix cache
// (src/nanovllm_ascend/npu/block_manager.py:57-65 key = (parent key, block's
// token ids); :136-152 longest-prefix lookup returning each key's first
// cached block; :154-179 hashing the full prompt blocks after prefill;
// :76-81, :89 a reused physical block forgets its key; :187-192 clear).
//
// Keys are interned (parent key, tokens) pairs with reference counts: a key
// lives while a block carries it or an interned child names it as parent,
// so two chains get the same key exactly when their whole token content is
// equal, and hashing a block costs O(block_size) whatever its depth.
#include <cstring>
#include <new>
#include <unordered_map>
#include <vector>

#include "host_common.h"

struct nvk_prefix_index {
  struct Spec {
    int64_t parent;  // -1: no parent
    std::vector<int64_t> tokens;
    bool operator==(const Spec& o) const { return parent == o.parent && tokens == o.tokens; }
  };
  struct SpecHash {
    size_t operator()(const Spec& s) const {
      uint64_t h = 0x9E3779B97F4A7C15ull ^ static_cast<uint64_t>(s.parent + 1);
      for (int64_t t : s.tokens) {  // splitmix-style mixing of every token id
        uint64_t z = h + 0x9E3779B97F4A7C15ull + static_cast<uint64_t>(t);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        h = z ^ (z >> 31);
      }
      return static_cast<size_t>(h ^ s.tokens.size());
    }
  };
  struct Entry {
    Spec spec;
    int64_t refs = 0;
    std::vector<int32_t> holders;  // blocks cached under this key, in caching order
  };

  int num_blocks = 0, block_size = 0;
  int64_t next_key = 0;
  std::unordered_map<Spec, int64_t, SpecHash> ids;
  std::unordered_map<int64_t, Entry> entries;
  std::vector<int64_t> block_key;  // per physical block, -1 = not cached
  int64_t cached_keys = 0;         // keys with at least one holder

  Spec spec_of(int64_t parent, const int64_t* tokens, int64_t num_tokens, int block_idx) const {
    Spec s;
    s.parent = parent;
    const int64_t start = static_cast<int64_t>(block_idx) * block_size;
    const int64_t end = start + block_size < num_tokens ? start + block_size : num_tokens;
    if (end > start) s.tokens.assign(tokens + start, tokens + end);
    return s;
  }

  int64_t acquire(Spec&& s) {
    auto it = ids.find(s);
    int64_t key;
    if (it == ids.end()) {
      key = next_key++;
      const int64_t parent = s.parent;
      Entry e;
      e.spec = s;
      ids.emplace(std::move(s), key);
      entries.emplace(key, std::move(e));
      if (parent >= 0) entries[parent].refs += 1;
    } else {
      key = it->second;
    }
    entries[key].refs += 1;
    return key;
  }

  void release(int64_t key) {
    while (key >= 0) {
      auto it = entries.find(key);
      if (it == entries.end()) return;
      if (--it->second.refs > 0) return;
      const int64_t parent = it->second.spec.parent;
      ids.erase(it->second.spec);
      entries.erase(it);
      key = parent;
    }
  }

  void forget(int32_t block) {
    const int64_t key = block_key[block];
    if (key < 0) return;
    auto& holders = entries[key].holders;
    for (size_t i = 0; i < holders.size(); ++i)
      if (holders[i] == block) {
        holders.erase(holders.begin() + static_cast<long>(i));
        break;
      }
    if (holders.empty()) --cached_keys;
    release(key);
    block_key[block] = -1;
  }
};

namespace {
int check_index(const nvk_prefix_index* idx, const char* who) {
  if (!idx) return nvk::fail(NVK_ERR_INVALID_ARGUMENT, "%s: null index", who);
  return NVK_OK;
}
}  // namespace

extern "C" int nvk_prefix_create(int num_blocks, int block_size, nvk_prefix_index** out) {
  if (!out || num_blocks <= 0 || block_size <= 0)
    return nvk::fail(NVK_ERR_INVALID_ARGUMENT, "prefix_create: bad arguments (blocks=%d block_size=%d)", num_blocks,
                     block_size);
  auto* idx = new (std::nothrow) nvk_prefix_index();
  if (!idx) return nvk::fail(NVK_ERR_INVALID_ARGUMENT, "prefix_create: out of host memory");
  idx->num_blocks = num_blocks;
  idx->block_size = block_size;
  idx->block_key.assign(static_cast<size_t>(num_blocks), -1);
  *out = idx;
  return NVK_OK;
}

extern "C" void nvk_prefix_destroy(nvk_prefix_index* idx) { delete idx; }

extern "C" int nvk_prefix_find_longest(nvk_prefix_index* idx, const int64_t* token_ids, int64_t num_tokens,
                                       int max_blocks, int32_t* block_ids, int* count) {
  int rc = check_index(idx, "prefix_find_longest");
  if (rc != NVK_OK) return rc;
  if (!count || (max_blocks > 0 && (!token_ids || !block_ids)) || num_tokens < 0)
    return nvk::fail(NVK_ERR_INVALID_ARGUMENT, "prefix_find_longest: null pointer or negative length");
  int found = 0;
  int64_t parent = -1;
  for (int b = 0; b < max_blocks; ++b) {
    auto it = idx->ids.find(idx->spec_of(parent, token_ids, num_tokens, b));
    if (it == idx->ids.end()) break;
    const auto& holders = idx->entries[it->second].holders;
    if (holders.empty()) break;
    block_ids[found++] = holders.front();
    parent = it->second;
  }
  *count = found;
  return NVK_OK;
}

extern "C" int nvk_prefix_cache_blocks(nvk_prefix_index* idx, const int32_t* table, int table_len,
                                       int num_cached_blocks, int num_full_blocks, const int64_t* token_ids,
                                       int64_t num_tokens) {
  int rc = check_index(idx, "prefix_cache_blocks");
  if (rc != NVK_OK) return rc;
  if (num_cached_blocks < 0 || num_full_blocks > table_len || (num_full_blocks > 0 && (!table || !token_ids)))
    return nvk::fail(NVK_ERR_INVALID_ARGUMENT, "prefix_cache_blocks: bad arguments (cached=%d full=%d table=%d)",
                     num_cached_blocks, num_full_blocks, table_len);
  for (int i = 0; i < num_full_blocks; ++i)
    if (table[i] < 0 || table[i] >= idx->num_blocks)
      return nvk::fail(NVK_ERR_INVALID_ARGUMENT, "prefix_cache_blocks: block id %d out of range", table[i]);
  int64_t parent = num_cached_blocks > 0 && num_cached_blocks <= table_len ? idx->block_key[table[num_cached_blocks - 1]] : -1;
  for (int b = num_cached_blocks; b < num_full_blocks; ++b) {
    const int32_t block = table[b];
    if (idx->block_key[block] >= 0) {  // already cached (e.g. a shared prefix block)
      parent = idx->block_key[block];
      continue;
    }
    const int64_t key = idx->acquire(idx->spec_of(parent, token_ids, num_tokens, b));
    idx->block_key[block] = key;
    auto& holders = idx->entries[key].holders;
    if (holders.empty()) ++idx->cached_keys;
    holders.push_back(block);
    parent = key;
  }
  return NVK_OK;
}

extern "C" int nvk_prefix_forget_block(nvk_prefix_index* idx, int block_id) {
  int rc = check_index(idx, "prefix_forget_block");
  if (rc != NVK_OK) return rc;
  if (block_id < 0 || block_id >= idx->num_blocks)
    return nvk::fail(NVK_ERR_INVALID_ARGUMENT, "prefix_forget_block: block id %d out of range", block_id);
  idx->forget(block_id);
  return NVK_OK;
}

extern "C" int64_t nvk_prefix_block_key(const nvk_prefix_index* idx, int block_id) {
  if (!idx || block_id < 0 || block_id >= idx->num_blocks) return -1;
  return idx->block_key[block_id];
}

extern "C" int nvk_prefix_clear(nvk_prefix_index* idx) {
  int rc = check_index(idx, "prefix_clear");
  if (rc != NVK_OK) return rc;
  idx->ids.clear();
  idx->entries.clear();
  idx->block_key.assign(idx->block_key.size(), -1);
  idx->cached_keys = 0;
  return NVK_OK;
}

extern "C" int64_t nvk_prefix_num_cached_keys(const nvk_prefix_index* idx) { return idx ? idx->cached_keys : 0; }

extern "C" int64_t nvk_prefix_num_keys(const nvk_prefix_index* idx) {
  return idx ? static_cast<int64_t>(idx->entries.size()) : 0;
}
