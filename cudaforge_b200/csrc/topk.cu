// Row-wise top-k (k <= 8) of logits: the draft-tree builder's candidate
// selection (children of a node = the k highest draft logits of its row,
// descending, ties to the lower token id).  No reference counterpart: the
// reference drafts chains only (cudaforge/speculative.py:113-123).
//
// One CTA per row.  Every thread keeps a sorted top-k of the elements it
// strides over (16-byte loads), then k rounds of a block-wide arg-max over
// the threads' current heads select the row's top-k in order.  HBM-bound:
// one read of the row.
#include "common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kMaxK = 8;

// (a, ia) ranks before (b, ib): larger value first, then the lower index; NaN ranks last
__device__ __forceinline__ bool before(float a, int32_t ia, float b, int32_t ib) {
  if (a != a) return false;
  if (b != b) return true;
  return a > b || (a == b && ia < ib);
}

template <typename T, int k>
__global__ void __launch_bounds__(kThreads) topk_rows_kernel(const T *__restrict__ x, int64_t row_stride, int64_t V,
                                                             int32_t *__restrict__ out_idx,
                                                             float *__restrict__ out_val) {
  const int row = blockIdx.x, tid = threadIdx.x;
  const T *xr = x + (int64_t)row * row_stride;
  float tv[k];
  int32_t ti[k];
#pragma unroll
  for (int j = 0; j < k; ++j) { tv[j] = __int_as_float(0x7fc00000); ti[j] = INT32_MAX; }
  // sorted insertion, fully unrolled so the lists stay in registers
  auto push = [&](float v, int32_t i) {
    if (!before(v, i, tv[k - 1], ti[k - 1])) return;
#pragma unroll
    for (int j = k - 1; j > 0; --j) {
      const bool up = before(v, i, tv[j - 1], ti[j - 1]);
      const bool here = !up && before(v, i, tv[j], ti[j]);
      tv[j] = up ? tv[j - 1] : (here ? v : tv[j]);
      ti[j] = up ? ti[j - 1] : (here ? i : ti[j]);
    }
    if (before(v, i, tv[0], ti[0])) { tv[0] = v; ti[0] = i; }
  };
  constexpr int VEC = 16 / sizeof(T);
  const bool vec_ok = (reinterpret_cast<uintptr_t>(xr) & 15) == 0;
  if (vec_ok) {
    const int64_t nvec = V / VEC;
    for (int64_t v = tid; v < nvec; v += kThreads) {
      cf::Vec16<T> q;
      q.raw = reinterpret_cast<const uint4 *>(xr)[v];
#pragma unroll
      for (int j = 0; j < VEC; ++j) push(q.get(j), (int32_t)(v * VEC + j));
    }
    for (int64_t i = nvec * VEC + tid; i < V; i += kThreads) push(cf::to_float(xr[i]), (int32_t)i);
  } else {
    for (int64_t i = tid; i < V; i += kThreads) push(cf::to_float(xr[i]), (int32_t)i);
  }
  __shared__ float sv[kThreads / 32];
  __shared__ int32_t si[kThreads / 32];
  __shared__ int32_t s_win;
  const int w = tid >> 5, l = tid & 31;
  for (int r = 0; r < k; ++r) {
    float bv = tv[0];
    int32_t bi = ti[0];
    // the owner is identified by its index (indices are unique across threads)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
      const int32_t i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      if (before(v2, i2, bv, bi)) { bv = v2; bi = i2; }
    }
    if (l == 0) { sv[w] = bv; si[w] = bi; }
    __syncthreads();
    if (tid == 0) {
      float b = sv[0];
      int32_t i = si[0];
      for (int q = 1; q < kThreads / 32; ++q)
        if (before(sv[q], si[q], b, i)) { b = sv[q]; i = si[q]; }
      s_win = i;
      out_idx[(int64_t)row * k + r] = i == INT32_MAX ? -1 : i;
      if (out_val) out_val[(int64_t)row * k + r] = b;
    }
    __syncthreads();
    if (ti[0] == s_win) {  // pop this thread's head
#pragma unroll
      for (int j = 0; j < k - 1; ++j) { tv[j] = tv[j + 1]; ti[j] = ti[j + 1]; }
      tv[k - 1] = __int_as_float(0x7fc00000);
      ti[k - 1] = INT32_MAX;
    }
    __syncthreads();
  }
}

template <typename T>
int launch(const void *x, int64_t row_stride, int32_t rows, int64_t V, int32_t k, int32_t *idx, float *val,
           cudaStream_t s) {
  const T *p = reinterpret_cast<const T *>(x);
  switch (k) {
#define CF_K(K) case K: topk_rows_kernel<T, K><<<rows, kThreads, 0, s>>>(p, row_stride, V, idx, val); break;
    CF_K(1) CF_K(2) CF_K(3) CF_K(4) CF_K(5) CF_K(6) CF_K(7) CF_K(8)
#undef CF_K
    default: return CF_EINVAL;
  }
  return cf_launch_status();
}

}  // namespace

extern "C" int cf_topk_rows(const void *logits, int64_t row_stride, int32_t rows, int64_t vocab, int32_t dtype,
                            int32_t k, int32_t *out_idx, float *out_val, void *stream) {
  if (rows < 0 || vocab < 1 || vocab > INT32_MAX - 1 || k < 1 || k > kMaxK || row_stride < vocab) return CF_EINVAL;
  if (rows == 0) return CF_OK;
  if (!logits || !out_idx || rows > 2147483647) return CF_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CF_F32: return launch<float>(logits, row_stride, rows, vocab, k, out_idx, out_val, s);
    case CF_BF16: return launch<__nv_bfloat16>(logits, row_stride, rows, vocab, k, out_idx, out_val, s);
    case CF_F16: return launch<__half>(logits, row_stride, rows, vocab, k, out_idx, out_val, s);
    default: return CF_EINVAL;
  }
}
