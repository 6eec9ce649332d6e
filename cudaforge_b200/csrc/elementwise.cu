// Small fused ops of the verify forward: embedding gather, RMSNorm, RoPE on
// the fused QKV rows (with the K/V scatter into this step's scratch), SwiGLU.
// All are HBM-bound single passes with 16-byte vector access where the row
// layout allows it.
#include "common.cuh"

namespace {

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

template <typename T>
__global__ void embedding_kernel(const int32_t *ids, const T *table, int vocab, int dim, T *out) {
  const int m = blockIdx.x;
  const int id = ids[m];
  const bool ok = id >= 0 && id < vocab;
  const uint4 *src = reinterpret_cast<const uint4 *>(table + (int64_t)(ok ? id : 0) * dim);
  uint4 *dst = reinterpret_cast<uint4 *>(out + (int64_t)m * dim);
  for (int v = threadIdx.x; v < dim / 8; v += blockDim.x) dst[v] = ok ? src[v] : make_uint4(0, 0, 0, 0);
}

template <typename T>
__global__ void rmsnorm_kernel(const T *x, int64_t ldx, const T *w, T *out, int64_t ldo, int dim, float eps) {
  const int m = blockIdx.x;
  const T *xr = x + (int64_t)m * ldx;
  float ss = 0.0f;
  for (int v = threadIdx.x; v < dim / 8; v += blockDim.x) {
    cf::Vec16<T> pk;
    pk.raw = reinterpret_cast<const uint4 *>(xr)[v];
#pragma unroll
    for (int j = 0; j < 8; ++j) { const float f = pk.get(j); ss += f * f; }
  }
  ss = cf::warp_sum(ss);
  __shared__ float red[32];
  const int w_ = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w_] = ss;
  __syncthreads();
  if (w_ == 0) {
    ss = l < (int)(blockDim.x >> 5) ? red[l] : 0.0f;
    ss = cf::warp_sum(ss);
    if (l == 0) red[0] = ss;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)dim + eps);
  T *orow = out + (int64_t)m * ldo;
  for (int v = threadIdx.x; v < dim / 8; v += blockDim.x) {
    cf::Vec16<T> pk, pw;
    pk.raw = reinterpret_cast<const uint4 *>(xr)[v];
    pw.raw = reinterpret_cast<const uint4 *>(w)[v];
    uint4 o;
    T *op = reinterpret_cast<T *>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) op[j] = from_f<T>(pk.get(j) * inv * pw.get(j));
    reinterpret_cast<uint4 *>(orow)[v] = o;
  }
}

// One CTA per row m; threads over (head, i < D/2) pairs for the Hq + Hkv
// rotated heads, then the V copy.
template <typename T>
__global__ void rope_qkv_kernel(T *qkv, int64_t ld, int Hq, int Hkv, int D, const int32_t *pos, float log2_base,
                                T *k_new, T *v_new) {
  const int m = blockIdx.x;
  T *row = qkv + (int64_t)m * ld;
  const float p = (float)pos[m];
  const int half = D / 2;
  const int pairs = (Hq + Hkv) * half;
  for (int idx = threadIdx.x; idx < pairs; idx += blockDim.x) {
    const int hh = idx / half, i = idx % half;
    const float inv_freq = exp2f(-((float)(2 * i) / (float)D) * log2_base);
    float s, c;
    sincosf(p * inv_freq, &s, &c);
    const T *src = row + (int64_t)hh * D;
    const float x1 = cf::to_float(src[i]), x2 = cf::to_float(src[i + half]);
    const float o1 = x1 * c - x2 * s, o2 = x1 * s + x2 * c;
    if (hh < Hq) {
      row[(int64_t)hh * D + i] = from_f<T>(o1);
      row[(int64_t)hh * D + i + half] = from_f<T>(o2);
    } else {
      T *dst = k_new + ((int64_t)m * Hkv + (hh - Hq)) * D;
      dst[i] = from_f<T>(o1);
      dst[i + half] = from_f<T>(o2);
    }
  }
  const uint4 *vsrc = reinterpret_cast<const uint4 *>(row + (int64_t)(Hq + Hkv) * D);
  uint4 *vdst = reinterpret_cast<uint4 *>(v_new + (int64_t)m * Hkv * D);
  for (int v = threadIdx.x; v < Hkv * D / 8; v += blockDim.x) vdst[v] = vsrc[v];
}

template <typename T>
__global__ void silu_mul_kernel(const T *gu, int64_t ldg, T *out, int64_t ldo, int ffn) {
  const int m = blockIdx.y;
  const T *g = gu + (int64_t)m * ldg;
  T *o = out + (int64_t)m * ldo;
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < ffn / 8; v += gridDim.x * blockDim.x) {
    cf::Vec16<T> a, u;
    a.raw = reinterpret_cast<const uint4 *>(g)[v];
    u.raw = reinterpret_cast<const uint4 *>(g + ffn)[v];
    uint4 r;
    T *rp = reinterpret_cast<T *>(&r);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float x = a.get(j);
      rp[j] = from_f<T>(x / (1.0f + expf(-x)) * u.get(j));
    }
    reinterpret_cast<uint4 *>(o)[v] = r;
  }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" int cf_embedding(const int32_t *ids, int32_t m, const void *table, int32_t vocab, int32_t dim, void *out,
                            int32_t dtype, void *stream) {
  if (m < 0 || dim <= 0 || dim % 8 || !ids || !table || !out || !aligned16(table) || !aligned16(out)) return CF_EINVAL;
  if (m == 0) return CF_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CF_BF16)
    embedding_kernel<<<m, 128, 0, s>>>(ids, (const __nv_bfloat16 *)table, vocab, dim, (__nv_bfloat16 *)out);
  else if (dtype == CF_F16)
    embedding_kernel<<<m, 128, 0, s>>>(ids, (const __half *)table, vocab, dim, (__half *)out);
  else
    return CF_EINVAL;
  return cf_launch_status();
}

extern "C" int cf_rmsnorm(const void *x, int64_t ldx, const void *w, void *out, int64_t ldo, int32_t m, int32_t dim,
                          float eps, int32_t dtype, void *stream) {
  if (m < 0 || dim <= 0 || dim % 8 || ldx % 8 || ldo % 8 || !x || !w || !out) return CF_EINVAL;
  if (!aligned16(x) || !aligned16(w) || !aligned16(out)) return CF_EINVAL;
  if (m == 0) return CF_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int threads = dim >= 4096 ? 512 : 128;
  if (dtype == CF_BF16)
    rmsnorm_kernel<<<m, threads, 0, s>>>((const __nv_bfloat16 *)x, ldx, (const __nv_bfloat16 *)w,
                                         (__nv_bfloat16 *)out, ldo, dim, eps);
  else if (dtype == CF_F16)
    rmsnorm_kernel<<<m, threads, 0, s>>>((const __half *)x, ldx, (const __half *)w, (__half *)out, ldo, dim, eps);
  else
    return CF_EINVAL;
  return cf_launch_status();
}

extern "C" int cf_rope_qkv(void *qkv, int64_t ld, int32_t m, int32_t num_q_heads, int32_t num_kv_heads,
                           int32_t head_dim, const int32_t *pos, float base, void *k_new, void *v_new, int32_t dtype,
                           void *stream) {
  if (m < 0 || head_dim % 16 || num_q_heads <= 0 || num_kv_heads <= 0 || !qkv || !pos || !k_new || !v_new)
    return CF_EINVAL;
  if (ld % 8 || !aligned16(qkv) || !aligned16(v_new) || !(base > 1.0f)) return CF_EINVAL;
  if (m == 0) return CF_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const float lb = log2f(base);
  if (dtype == CF_BF16)
    rope_qkv_kernel<<<m, 256, 0, s>>>((__nv_bfloat16 *)qkv, ld, num_q_heads, num_kv_heads, head_dim, pos, lb,
                                      (__nv_bfloat16 *)k_new, (__nv_bfloat16 *)v_new);
  else if (dtype == CF_F16)
    rope_qkv_kernel<<<m, 256, 0, s>>>((__half *)qkv, ld, num_q_heads, num_kv_heads, head_dim, pos, lb,
                                      (__half *)k_new, (__half *)v_new);
  else
    return CF_EINVAL;
  return cf_launch_status();
}

extern "C" int cf_silu_mul(const void *gu, int64_t ldg, void *out, int64_t ldo, int32_t m, int32_t ffn, int32_t dtype,
                           void *stream) {
  if (m < 0 || ffn <= 0 || ffn % 8 || ldg % 8 || ldo % 8 || !gu || !out || !aligned16(gu) || !aligned16(out))
    return CF_EINVAL;
  if (m == 0) return CF_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid((ffn / 8 + 255) / 256, m);
  if (dtype == CF_BF16)
    silu_mul_kernel<<<grid, 256, 0, s>>>((const __nv_bfloat16 *)gu, ldg, (__nv_bfloat16 *)out, ldo, ffn);
  else if (dtype == CF_F16)
    silu_mul_kernel<<<grid, 256, 0, s>>>((const __half *)gu, ldg, (__half *)out, ldo, ffn);
  else
    return CF_EINVAL;
  return cf_launch_status();
}
