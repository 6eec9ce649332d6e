// Host-side paged KV-cache page tables with the reference's semantics.
//
// Mirrors cudaforge::memory::PagedKVCache (csrc/include/cudaforge/memory/
// paged_kv_cache.h:97-178, csrc/src/memory/paged_kv_cache.cpp): LIFO free
// stack initialised N-1..0 (:44-53), prefix-hash tree with reference counts
// and LRU eviction of cached prefix blocks (:80-165), register / append /
// unregister / fork (:167-316), batch flattening with -1 padding and context
// length = (blocks-1)*block_size + last.filled (:318-396), and pool
// addressing id*bytes_per_block + layer*layer_block_bytes (:409-421).  The
// allocation order (and therefore every page table) is identical to the
// reference for the same sequence of calls; the block hash is the
// reference's formula so prefix-cache hits agree as well.
//
// Device memory is not owned here: the K/V pools are caller-provided device
// pointers (the Python layer allocates them with torch).  The batch metadata
// is flattened into caller buffers; the caller copies it to the device on its
// stream.
#include <cstdint>
#include <cstring>
#include <list>
#include <memory>
#include <mutex>
#include <new>
#include <unordered_map>
#include <vector>

#include "cf_api.h"

namespace {

struct Block {
  uint32_t refs = 0;
  uint32_t filled = 0;
  uint64_t hash = 0;
  bool cached = false;
  std::list<int32_t>::iterator lru;
};

struct Node {
  int32_t block = -1;
  std::unordered_map<uint64_t, std::shared_ptr<Node>> kids;
};

struct Cache {
  cf_kv_config cfg;
  void *kpool = nullptr, *vpool = nullptr;
  size_t layer_block_bytes = 0, bytes_per_block = 0;
  std::mutex mu;
  std::vector<Block> blocks;
  std::vector<int32_t> free_stack;
  std::list<int32_t> lru;  // front = most recently released
  std::shared_ptr<Node> root = std::make_shared<Node>();
  std::unordered_map<uint64_t, std::shared_ptr<Node>> by_hash;
  std::unordered_map<uint64_t, std::vector<int32_t>> tables;
  uint64_t hits = 0, misses = 0, evictions = 0;

  static uint64_t block_hash(const int32_t *t, uint32_t n, uint64_t parent) {
    uint64_t h = parent ^ 0x9e3779b97f4a7c15ULL;
    for (uint32_t i = 0; i < n; ++i) {
      const uint64_t v = static_cast<uint64_t>(static_cast<int64_t>(t[i]));  // std::hash<int32_t>
      h ^= v + 0x9e3779b9u + (h << 6) + (h >> 2);
    }
    return h;
  }

  bool evict_one() {
    for (auto it = lru.rbegin(); it != lru.rend(); ++it) {
      const int32_t id = *it;
      Block &b = blocks[id];
      if (b.refs != 0) continue;
      by_hash.erase(b.hash);  // the tree edge is kept, exactly as the reference does
      lru.erase(std::next(it).base());
      b.cached = false;
      b.hash = 0;
      b.filled = 0;
      b.lru = lru.end();
      free_stack.push_back(id);
      ++evictions;
      return true;
    }
    return false;
  }

  // -1 when the pool is exhausted
  int32_t take_block() {
    if (free_stack.empty() && !evict_one()) return -1;
    const int32_t id = free_stack.back();
    free_stack.pop_back();
    Block &b = blocks[id];
    b.refs = 1;
    b.filled = 0;
    b.cached = false;
    return id;
  }

  void release_block(int32_t id) {
    if (id < 0 || static_cast<uint64_t>(id) >= cfg.total_gpu_blocks) return;
    Block &b = blocks[id];
    if (b.refs == 0) return;
    if (--b.refs == 0) {
      if (cfg.enable_prefix_caching && b.hash != 0) {
        b.cached = true;
        lru.push_front(id);
        b.lru = lru.begin();
      } else {
        b.filled = 0;
        free_stack.push_back(id);
      }
    }
  }
};

}  // namespace

struct cf_kvcache {
  Cache c;
};

extern "C" cf_kvcache *cf_kvcache_create(const cf_kv_config *cfg, void *key_pool, void *val_pool) {
  if (!cfg || cfg->block_size == 0 || cfg->total_gpu_blocks == 0 || cfg->total_gpu_blocks > INT32_MAX) return nullptr;
  cf_kvcache *h = new (std::nothrow) cf_kvcache();
  if (!h) return nullptr;
  Cache &c = h->c;
  c.cfg = *cfg;
  c.kpool = key_pool;
  c.vpool = val_pool;
  c.layer_block_bytes = (size_t)cfg->num_kv_heads * cfg->block_size * cfg->head_dim * cfg->element_size_bytes;
  c.bytes_per_block = (size_t)cfg->num_layers * c.layer_block_bytes;
  c.blocks.resize(cfg->total_gpu_blocks);
  c.free_stack.reserve(cfg->total_gpu_blocks);
  for (int64_t i = (int64_t)cfg->total_gpu_blocks - 1; i >= 0; --i) {
    c.blocks[i].lru = c.lru.end();
    c.free_stack.push_back((int32_t)i);
  }
  return h;
}

extern "C" void cf_kvcache_destroy(cf_kvcache *h) { delete h; }

extern "C" int cf_kvcache_register_sequence(cf_kvcache *h, uint64_t seq, const int32_t *tokens, uint32_t n,
                                            uint32_t *matched_out) {
  if (!h || (n && !tokens)) return CF_EINVAL;
  Cache &c = h->c;
  std::lock_guard<std::mutex> g(c.mu);
  if (matched_out) *matched_out = 0;
  if (c.tables.count(seq)) return CF_OK;  // already registered: no-op, 0 matched
  const uint32_t bs = c.cfg.block_size;
  const uint32_t full = n / bs;
  std::vector<int32_t> table;
  uint32_t matched = 0;
  uint64_t parent = 0;
  std::shared_ptr<Node> node = c.root;
  if (c.cfg.enable_prefix_caching) {
    for (uint32_t b = 0; b < full; ++b) {
      const uint64_t hv = Cache::block_hash(tokens + (size_t)b * bs, bs, parent);
      auto it = node->kids.find(hv);
      if (it == node->kids.end()) break;
      Block &blk = c.blocks[it->second->block];
      ++blk.refs;
      if (blk.cached) {
        blk.cached = false;
        if (blk.lru != c.lru.end()) {
          c.lru.erase(blk.lru);
          blk.lru = c.lru.end();
        }
      }
      table.push_back(it->second->block);
      matched += bs;
      ++c.hits;
      parent = hv;
      node = it->second;
    }
  }
  const uint32_t rest = n - matched;
  const uint32_t start = matched / bs;
  for (uint32_t b = 0; b < rest / bs; ++b) {
    const uint64_t hv = Cache::block_hash(tokens + (size_t)(start + b) * bs, bs, parent);
    const int32_t id = c.take_block();
    if (id < 0) return CF_ENOMEM;  // the reference throws here, keeping what it took
    c.blocks[id].filled = bs;
    c.blocks[id].hash = hv;
    auto nn = std::make_shared<Node>();
    nn->block = id;
    node->kids[hv] = nn;
    c.by_hash[hv] = nn;
    table.push_back(id);
    ++c.misses;
    parent = hv;
    node = nn;
  }
  if (rest % bs != 0 || table.empty()) {
    const int32_t id = c.take_block();
    if (id < 0) return CF_ENOMEM;  // the reference throws here, keeping what it took
    c.blocks[id].filled = rest % bs;
    table.push_back(id);
  }
  c.tables[seq] = std::move(table);
  if (matched_out) *matched_out = matched;
  return CF_OK;
}

extern "C" int cf_kvcache_append_tokens(cf_kvcache *h, uint64_t seq, uint32_t n) {
  if (!h) return CF_EINVAL;
  Cache &c = h->c;
  std::lock_guard<std::mutex> g(c.mu);
  auto it = c.tables.find(seq);
  if (it == c.tables.end()) return CF_ERANGE;
  std::vector<int32_t> &t = it->second;
  const uint32_t bs = c.cfg.block_size;
  Block &last = c.blocks[t.back()];
  const uint32_t room = bs - last.filled;
  if (n <= room) {
    last.filled += n;
    return CF_OK;
  }
  uint32_t rem = n - room;
  last.filled = bs;
  const uint32_t extra = (rem + bs - 1) / bs;
  for (uint32_t i = 0; i < extra; ++i) {
    const int32_t id = c.take_block();
    if (id < 0) return CF_ENOMEM;  // as the reference: blocks taken so far stay appended
    const uint32_t add = rem < bs ? rem : bs;
    c.blocks[id].filled = add;
    rem -= add;
    t.push_back(id);
  }
  return CF_OK;
}

extern "C" int cf_kvcache_append_batch(cf_kvcache *h, const uint64_t *seqs, const int32_t *n, uint32_t batch) {
  if (!h || (batch && (!seqs || !n))) return CF_EINVAL;
  for (uint32_t i = 0; i < batch; ++i) {  // batch order == the reference's per-call order
    if (n[i] <= 0) continue;
    const int rc = cf_kvcache_append_tokens(h, seqs[i], (uint32_t)n[i]);
    if (rc != CF_OK) return rc;
  }
  return CF_OK;
}

extern "C" int cf_kvcache_unregister_sequence(cf_kvcache *h, uint64_t seq) {
  if (!h) return CF_EINVAL;
  Cache &c = h->c;
  std::lock_guard<std::mutex> g(c.mu);
  auto it = c.tables.find(seq);
  if (it == c.tables.end()) return CF_OK;
  for (int32_t id : it->second) c.release_block(id);
  c.tables.erase(it);
  return CF_OK;
}

extern "C" int cf_kvcache_fork_sequence(cf_kvcache *h, uint64_t parent, uint64_t child) {
  if (!h) return CF_EINVAL;
  Cache &c = h->c;
  std::lock_guard<std::mutex> g(c.mu);
  auto it = c.tables.find(parent);
  if (it == c.tables.end()) return CF_ERANGE;
  for (int32_t id : it->second) ++c.blocks[id].refs;
  c.tables[child] = it->second;
  return CF_OK;
}

extern "C" int cf_kvcache_get_block_table(cf_kvcache *h, uint64_t seq, int32_t *out, uint32_t cap, uint32_t *len) {
  if (!h || !len) return CF_EINVAL;
  Cache &c = h->c;
  std::lock_guard<std::mutex> g(c.mu);
  auto it = c.tables.find(seq);
  if (it == c.tables.end()) return CF_ERANGE;
  *len = (uint32_t)it->second.size();
  if (out) {
    const uint32_t n = *len < cap ? *len : cap;
    std::memcpy(out, it->second.data(), n * sizeof(int32_t));
  }
  return CF_OK;
}

extern "C" int cf_kvcache_prepare_batch(cf_kvcache *h, const uint64_t *seqs, uint32_t batch, int32_t *tables,
                                        uint32_t table_cap, int32_t *context_lens, uint32_t *max_blocks_out) {
  if (!h || (batch && (!seqs || !context_lens)) || !max_blocks_out) return CF_EINVAL;
  Cache &c = h->c;
  std::lock_guard<std::mutex> g(c.mu);
  if (batch > c.cfg.max_supported_batch_size) return CF_ERANGE;
  size_t mb = 0;
  for (uint32_t i = 0; i < batch; ++i) {
    auto it = c.tables.find(seqs[i]);
    if (it == c.tables.end()) return CF_ERANGE;
    mb = it->second.size() > mb ? it->second.size() : mb;
  }
  if (mb > c.cfg.max_blocks_per_sequence) return CF_ERANGE;
  *max_blocks_out = (uint32_t)mb;
  if (tables && (uint64_t)batch * mb > table_cap) return CF_EINVAL;
  for (uint32_t i = 0; i < batch; ++i) {
    const std::vector<int32_t> &t = c.tables[seqs[i]];
    if (tables) {
      for (size_t j = 0; j < mb; ++j) tables[i * mb + j] = j < t.size() ? t[j] : -1;
    }
    context_lens[i] = (int32_t)((t.size() - 1) * c.cfg.block_size + c.blocks[t.back()].filled);
  }
  return CF_OK;
}

extern "C" int cf_kvcache_export_free_stack(cf_kvcache *h, int32_t *out, uint32_t cap, uint32_t *n) {
  if (!h || !n) return CF_EINVAL;
  Cache &c = h->c;
  std::lock_guard<std::mutex> g(c.mu);
  *n = (uint32_t)c.free_stack.size();
  if (out) std::memcpy(out, c.free_stack.data(), (c.free_stack.size() < cap ? c.free_stack.size() : cap) * 4);
  return CF_OK;
}

extern "C" int cf_kvcache_get_stats(cf_kvcache *h, cf_kv_stats *s) {
  if (!h || !s) return CF_EINVAL;
  Cache &c = h->c;
  std::lock_guard<std::mutex> g(c.mu);
  s->total_blocks = c.cfg.total_gpu_blocks;
  s->free_blocks = c.free_stack.size();
  s->cached_prefix_blocks = c.lru.size();
  s->allocated_blocks = s->total_blocks - s->free_blocks - s->cached_prefix_blocks;
  s->total_memory_bytes = s->total_blocks * c.bytes_per_block * 2;
  s->used_memory_bytes = (s->allocated_blocks + s->cached_prefix_blocks) * c.bytes_per_block * 2;
  s->pool_utilization_ratio = (double)(s->total_blocks - s->free_blocks) / (double)s->total_blocks;
  s->active_sequences_count = (uint32_t)c.tables.size();
  s->prefix_cache_hits = c.hits;
  s->prefix_cache_misses = c.misses;
  s->lru_evictions_count = c.evictions;
  return CF_OK;
}

extern "C" void *cf_kvcache_key_block_ptr(cf_kvcache *h, int32_t block, uint32_t layer) {
  if (!h) return nullptr;
  return static_cast<uint8_t *>(h->c.kpool) + (size_t)block * h->c.bytes_per_block + layer * h->c.layer_block_bytes;
}

extern "C" void *cf_kvcache_value_block_ptr(cf_kvcache *h, int32_t block, uint32_t layer) {
  if (!h) return nullptr;
  return static_cast<uint8_t *>(h->c.vpool) + (size_t)block * h->c.bytes_per_block + layer * h->c.layer_block_bytes;
}
