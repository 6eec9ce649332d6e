// Accepted-KV commit: scratch rows of the verify step -> paged pool slots.
//
// Grid (B, layer_count); each CTA streams the n_b committed tokens x Hkv heads
// x head_dim of one layer of one sequence with 16-byte vector copies.  Pure
// data movement: HBM roofline with algorithmic bytes 2 (K, V) x 2 (read +
// write) x n x Hkv x D x elem per layer.
#include "common.cuh"

namespace {

__global__ void kv_commit_kernel(const cf_kv_commit_args a) {
  const int b = blockIdx.x;
  const int l = a.layer_begin + blockIdx.y;
  const int Hkv = a.kv.num_kv_heads, D = a.kv.head_dim, bs = a.kv.block_size;
  const int n = min(a.rows, a.n_commit[b] + a.n_commit_add);
  if (n <= 0) return;
  const int vec = D / 8;  // 16-B vectors per head row (16-bit elements)
  const int64_t layer_block = (int64_t)Hkv * bs * D;  // elements
  const int64_t block_elems = (int64_t)a.kv.num_layers * layer_block;
  const int start = a.start_pos[b];
  const int total = n * Hkv * vec;
  const uint16_t *kn = reinterpret_cast<const uint16_t *>(a.k_new);
  const uint16_t *vn = reinterpret_cast<const uint16_t *>(a.v_new);
  uint16_t *kp = reinterpret_cast<uint16_t *>(a.kv.key_pool);
  uint16_t *vp = reinterpret_cast<uint16_t *>(a.kv.val_pool);
  for (int idx = threadIdx.x; idx < total; idx += blockDim.x) {
    const int v = idx % vec;
    const int h = (idx / vec) % Hkv;
    const int j = idx / (vec * Hkv);
    const int src_row = a.row_index ? a.row_index[(int64_t)b * a.rows + j] : j;
    const int pos = start + j;
    const int page = pos / bs, slot = pos % bs;
    const int blk = (pos >= 0 && page < a.max_blocks) ? a.block_tables[(int64_t)b * a.max_blocks + page] : -1;
    if (blk < 0 || blk >= a.kv.total_blocks || src_row < 0 || src_row >= a.rows) {
      if (a.status) atomicExch(a.status, CF_ERANGE);
      continue;
    }
    const int64_t src = ((((int64_t)l * a.batch + b) * a.rows + src_row) * Hkv + h) * D + v * 8;
    const int64_t dst = blk * block_elems + l * layer_block + ((int64_t)h * bs + slot) * D + v * 8;
    *reinterpret_cast<uint4 *>(kp + dst) = *reinterpret_cast<const uint4 *>(kn + src);
    *reinterpret_cast<uint4 *>(vp + dst) = *reinterpret_cast<const uint4 *>(vn + src);
  }
}

}  // namespace

extern "C" int cf_kv_commit(const cf_kv_commit_args *args, void *stream) {
  if (!args) return CF_EINVAL;
  const cf_kv_commit_args &a = *args;
  if (a.batch < 0 || a.rows <= 0 || a.layer_begin < 0 || a.layer_count < 0 ||
      a.layer_begin + a.layer_count > a.kv.num_layers)
    return CF_EINVAL;
  if (a.batch == 0 || a.layer_count == 0) return CF_OK;
  if (a.kv.head_dim % 8 || (a.kv.dtype != CF_BF16 && a.kv.dtype != CF_F16)) return CF_EINVAL;
  if (!a.k_new || !a.v_new || !a.n_commit || !a.start_pos || !a.block_tables || !a.kv.key_pool || !a.kv.val_pool)
    return CF_EINVAL;
  if ((reinterpret_cast<uintptr_t>(a.k_new) | reinterpret_cast<uintptr_t>(a.v_new) |
       reinterpret_cast<uintptr_t>(a.kv.key_pool) | reinterpret_cast<uintptr_t>(a.kv.val_pool)) & 15)
    return CF_EINVAL;
  dim3 grid(a.batch, a.layer_count);
  kv_commit_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return cf_launch_status();
}
