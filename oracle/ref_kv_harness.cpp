// TEST INFRASTRUCTURE ONLY -- C entry points around the UNMODIFIED reference
// PagedKVCache / BlockAllocator (csrc/src/memory/*.cpp), built by
// oracle/Makefile into oracle/_ref/libkv_ref.so against fake_cudart.cpp.
#include "cudaforge/memory/paged_kv_cache.h"

#include <cstdint>
#include <cstring>
#include <vector>

using namespace cudaforge::memory;

struct RefKV {
  BlockAllocator alloc;
  PagedKVCache cache;
  RefKV(const KVCacheConfig &c) : alloc(0.05), cache(c, alloc) {}
};

extern "C" {
void *refkv_create(uint32_t layers, uint32_t heads, uint32_t dim, uint32_t bs, uint64_t total, int prefix,
                   uint64_t max_batch, uint64_t max_blocks) {
  KVCacheConfig c;
  c.num_layers = layers;
  c.num_kv_heads = heads;
  c.head_dim = dim;
  c.block_size = bs;
  c.element_size_bytes = 2;
  c.total_gpu_blocks = total;
  c.enable_prefix_caching = prefix != 0;
  c.max_supported_batch_size = max_batch;
  c.max_blocks_per_sequence = max_blocks;
  return new RefKV(c);
}
void refkv_destroy(void *h) { delete static_cast<RefKV *>(h); }
// 0 ok, -5 out of pages, -2 other error
int refkv_register(void *h, uint64_t seq, const int32_t *tok, uint32_t n, uint32_t *matched) {
  try {
    *matched = static_cast<RefKV *>(h)->cache.register_sequence_with_prefix(seq, std::span<const int32_t>(tok, n));
  } catch (const OutOfPagesException &) {
    return -5;
  } catch (...) {
    return -2;
  }
  return 0;
}
int refkv_append(void *h, uint64_t seq, uint32_t n) {
  try {
    static_cast<RefKV *>(h)->cache.append_tokens(seq, n);
  } catch (const OutOfPagesException &) {
    return -5;
  } catch (...) {
    return -2;
  }
  return 0;
}
int refkv_unregister(void *h, uint64_t seq) {
  static_cast<RefKV *>(h)->cache.unregister_sequence(seq);
  return 0;
}
int refkv_fork(void *h, uint64_t p, uint64_t c) {
  try {
    static_cast<RefKV *>(h)->cache.fork_sequence(p, c);
  } catch (...) {
    return -2;
  }
  return 0;
}
int refkv_table(void *h, uint64_t seq, int32_t *out, uint32_t cap, uint32_t *len) {
  try {
    const auto &t = static_cast<RefKV *>(h)->cache.get_block_table(seq);
    *len = (uint32_t)t.size();
    for (uint32_t i = 0; i < *len && i < cap; ++i) out[i] = t[i];
  } catch (...) {
    return -2;
  }
  return 0;
}
// Runs prepare_batch_metadata; with the fake runtime the "device" buffers are
// host memory and are read back directly.
int refkv_prepare(void *h, const uint64_t *seqs, uint32_t b, int32_t *tables, uint32_t cap, int32_t *ctx,
                  uint32_t *max_blocks) {
  try {
    std::vector<uint64_t> ids(seqs, seqs + b);
    KVCacheBatchDescriptor d = static_cast<RefKV *>(h)->cache.prepare_batch_metadata(ids, nullptr);
    *max_blocks = (uint32_t)d.max_blocks_per_seq;
    if ((uint64_t)b * d.max_blocks_per_seq > cap) return -1;
    std::memcpy(tables, d.block_tables, sizeof(int32_t) * b * d.max_blocks_per_seq);
    std::memcpy(ctx, d.context_lens, sizeof(int32_t) * b);
  } catch (...) {
    return -2;
  }
  return 0;
}
void refkv_stats(void *h, uint64_t *out) {
  KVCacheStats s = static_cast<RefKV *>(h)->cache.get_stats();
  out[0] = s.total_blocks; out[1] = s.free_blocks; out[2] = s.allocated_blocks; out[3] = s.cached_prefix_blocks;
  out[4] = s.active_sequences_count; out[5] = s.prefix_cache_hits; out[6] = s.prefix_cache_misses;
  out[7] = s.lru_evictions_count;
}
}
