// Device-resident page-table growth: PagedKVCache::append_tokens
// (csrc/src/memory/paged_kv_cache.cpp:255-286) for a whole batch, on the GPU,
// so that a speculative step needs no host round trip between acceptance and
// the KV commit.
//
// Semantics are the host cache's (cudaforge_b200/csrc/paged_kv_cache.cpp,
// page tables bit-identical to the reference's): sequences grow in batch
// order; a sequence whose last block has room for its n new tokens only
// fills it; otherwise it takes ceil((n - room) / block_size) blocks, each
// popped from the top of the LIFO free stack.  Pops in batch order make
// sequence b's i-th new block stack[top - 1 - E_b - i], E_b the blocks taken
// by the sequences before it (an exclusive prefix sum), so one CTA computes
// every table at once.  No eviction: when the stack runs short (or a table
// would exceed max_blocks) nothing changes and the status word records
// CF_ENOMEM / CF_ERANGE -- the host path, which can evict cached prefix
// blocks, handles those batches.
#include "common.cuh"

namespace {

constexpr int kThreads = 1024;

__device__ __forceinline__ int blocks_needed(const cf_kv_append_args &a, int b, int &len) {
  const int bs = a.block_size;
  const int n = max(a.n_append[b], 0) + a.n_add;
  len = a.table_len[b];
  const int room = len * bs - a.context_lens[b];  // free slots of the last block
  return n <= room ? 0 : (n - room + bs - 1) / bs;
}

// Inclusive block-wide prefix sum (Hillis-Steele; every thread calls it).
__device__ __forceinline__ int block_inclusive_sum(int v, int32_t *s) {
  const int tid = threadIdx.x;
  s[tid] = v;
  __syncthreads();
  for (int o = 1; o < kThreads; o <<= 1) {
    const int w = tid >= o ? s[tid - o] : 0;
    __syncthreads();
    s[tid] += w;
    __syncthreads();
  }
  const int r = s[tid];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kThreads) kv_append_kernel(const cf_kv_append_args a) {
  __shared__ int32_t s_scan[kThreads];
  __shared__ int32_t s_tot, s_fail;
  const int tid = threadIdx.x;
  if (tid == 0) { s_tot = 0; s_fail = 0; }
  __syncthreads();
  // pass 1: the blocks every sequence needs, and whether the batch fits (nothing is written yet)
  for (int b0 = 0; b0 < a.batch; b0 += kThreads) {
    const int b = b0 + tid;
    int len = 0, extra = 0;
    if (b < a.batch) {
      extra = blocks_needed(a, b, len);
      if (len + extra > a.max_blocks) atomicExch(&s_fail, CF_ERANGE);
    }
    const int incl = block_inclusive_sum(extra, s_scan);
    if (tid == kThreads - 1) s_tot += incl;
    __syncthreads();
  }
  int fail = s_fail;
  if (!fail && s_tot > *a.free_top) fail = CF_ENOMEM;  // the same inputs in every thread: a uniform decision
  if (fail) {
    if (tid == 0 && a.status) atomicExch(a.status, fail);
    return;
  }
  // pass 2: sequence b's i-th new block is stack[top - 1 - E_b - i]
  const int top = *a.free_top;
  int base = 0;
  for (int b0 = 0; b0 < a.batch; b0 += kThreads) {
    const int b = b0 + tid;
    int len = 0, extra = 0;
    if (b < a.batch) extra = blocks_needed(a, b, len);
    const int incl = block_inclusive_sum(extra, s_scan);
    const int excl = base + incl - extra;
    if (b < a.batch) {
      int32_t *row = a.tables + (int64_t)b * a.max_blocks;
      for (int i = 0; i < extra; ++i) row[len + i] = a.free_stack[top - 1 - excl - i];
      a.table_len[b] = len + extra;
    }
    if (tid == kThreads - 1) s_tot = incl;  // reuse: this chunk's total
    __syncthreads();
    base += s_tot;
    __syncthreads();
  }
  if (tid == 0) *a.free_top = top - base;
}

}  // namespace

extern "C" int cf_kv_append_device(const cf_kv_append_args *args, void *stream) {
  if (!args) return CF_EINVAL;
  const cf_kv_append_args &a = *args;
  if (a.batch < 0 || a.block_size <= 0 || a.max_blocks <= 0 || a.n_add < 0) return CF_EINVAL;
  if (a.batch == 0) return CF_OK;
  if (!a.n_append || !a.free_stack || !a.free_top || !a.tables || !a.table_len || !a.context_lens) return CF_EINVAL;
  kv_append_kernel<<<1, kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return cf_launch_status();
}
