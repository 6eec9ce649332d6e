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

// RoPE (half split): the row's rotation table, (cos, sin) of p * base^(-2i/D)
// for i < D/2, computed once per row in shared memory (every head of the row
// shares it), with explicitly rounded products (no FMA contraction) so the
// plain and the split-K kernels below compute the same bits.
constexpr int kMaxHalf = 128;  // head_dim <= 256

__device__ __forceinline__ void rope_table(float p, int D, float log2_base, float2 *tab) {
  for (int i = threadIdx.x; i < D / 2; i += blockDim.x) {
    const float inv_freq = exp2f(__fmul_rn(-__fdiv_rn((float)(2 * i), (float)D), log2_base));
    float sn, cs;
    sincosf(__fmul_rn(p, inv_freq), &sn, &cs);
    tab[i] = make_float2(cs, sn);
  }
  __syncthreads();
}

// Four consecutive pairs (x1[j], x2[j]) = (x[i0+j], x[i0+j+D/2]).
__device__ __forceinline__ void rope4(const float2 *tab, int i0, const float (&x1)[4], const float (&x2)[4],
                                      float (&o1)[4], float (&o2)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = tab[i0 + j];
    o1[j] = __fsub_rn(__fmul_rn(x1[j], t.x), __fmul_rn(x2[j], t.y));
    o2[j] = __fadd_rn(__fmul_rn(x1[j], t.y), __fmul_rn(x2[j], t.x));
  }
}

template <typename T>
__device__ __forceinline__ void load4(const T *p, float (&o)[4]) {
  const uint2 r = *reinterpret_cast<const uint2 *>(p);
  const T *t = reinterpret_cast<const T *>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) o[j] = cf::to_float(t[j]);
}

template <typename T>
__device__ __forceinline__ void store4(T *p, const float (&v)[4]) {
  uint2 r;
  T *t = reinterpret_cast<T *>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) t[j] = from_f<T>(v[j]);
  *reinterpret_cast<uint2 *>(p) = r;
}

// Where the rotated pairs of head hh go: q heads back into the qkv row, k heads
// into this step's K scratch [m][Hkv][D].
template <typename T>
__device__ __forceinline__ T *rope_dst(T *row, T *k_new, int m, int hh, int Hq, int Hkv, int D) {
  return hh < Hq ? row + (int64_t)hh * D : k_new + ((int64_t)m * Hkv + (hh - Hq)) * D;
}

// One CTA per row m.  Work items: (head, 4 pairs) for the Hq + Hkv rotated
// heads (8-byte vector accesses), then 16-byte copies of the V heads.
template <typename T>
__global__ void rope_qkv_kernel(T *qkv, int64_t ld, int Hq, int Hkv, int D, const int32_t *pos, float log2_base,
                                T *k_new, T *v_new) {
  const int m = blockIdx.x;
  T *row = qkv + (int64_t)m * ld;
  __shared__ float2 tab[kMaxHalf];
  rope_table((float)pos[m], D, log2_base, tab);
  const int half = D / 2, q4 = half / 4;
  const int items = (Hq + Hkv) * q4;
  for (int idx = threadIdx.x; idx < items; idx += blockDim.x) {
    const int hh = idx / q4, i0 = (idx % q4) * 4;
    float x1[4], x2[4], o1[4], o2[4];
    load4(row + (int64_t)hh * D + i0, x1);
    load4(row + (int64_t)hh * D + i0 + half, x2);
    rope4(tab, i0, x1, x2, o1, o2);
    T *dst = rope_dst(row, k_new, m, hh, Hq, Hkv, D);
    store4(dst + i0, o1);
    store4(dst + i0 + half, o2);
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

// ---------------------------------------------------------------------------
// Split-K consumers: the producing GEMM left `splits` fp32 partials
// [splits][m][n] (cf_w4a16_gemm_partials); each kernel below first forms the
// GEMM output exactly as the split-K reduction would (fixed order s = 0..S-1,
// then + residual, then one rounding to T) and then does its own work on those
// values, so the result is bit-identical to reduce-then-consume.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void reduce8(const float *part, int splits, int64_t plane, int64_t off, const T *res,
                                        float (&o)[8]) {
  float4 a, b;
  cf::Vec16<T> rv;
  if (res) rv.raw = *reinterpret_cast<const uint4 *>(res);  // issued with the partial loads
  if (splits <= 4) {
    // the fused consumers' case (2-4 splits): every load in flight at once, then the sums
    // in the order s = 0..splits-1 (the same result as the loop below)
    float4 pa[4], pb[4];
#pragma unroll
    for (int s = 0; s < 4; ++s)
      if (s < splits) {
        pa[s] = *reinterpret_cast<const float4 *>(part + s * plane + off);
        pb[s] = *reinterpret_cast<const float4 *>(part + s * plane + off + 4);
      }
    a = pa[0];
    b = pb[0];
#pragma unroll
    for (int s = 1; s < 4; ++s)
      if (s < splits) {
        a.x += pa[s].x; a.y += pa[s].y; a.z += pa[s].z; a.w += pa[s].w;
        b.x += pb[s].x; b.y += pb[s].y; b.z += pb[s].z; b.w += pb[s].w;
      }
  } else {
    a = *reinterpret_cast<const float4 *>(part + off);
    b = *reinterpret_cast<const float4 *>(part + off + 4);
    for (int s = 1; s < splits; ++s) {
      const float4 c = *reinterpret_cast<const float4 *>(part + s * plane + off);
      const float4 d = *reinterpret_cast<const float4 *>(part + s * plane + off + 4);
      a.x += c.x; a.y += c.y; a.z += c.z; a.w += c.w;
      b.x += d.x; b.y += d.y; b.z += d.z; b.w += d.w;
    }
  }
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  if (res) {
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] += rv.get(j);
  }
}

// y = T(sum of partials + residual) (written, the residual stream); out = RMSNorm(y) * w.
template <typename T>
__global__ void splitk_rmsnorm_kernel(const float *part, int splits, int64_t plane, int n, const T *res,
                                      int64_t ldr, T *y, int64_t ldy, const T *w, T *out, int64_t ldo, int dim,
                                      float eps) {
  const int m = blockIdx.x;
  T *yr = y + (int64_t)m * ldy;
  float ss = 0.0f;
  constexpr int kKeep = 4;  // vectors of the row kept in registers for the second pass
  uint4 kept[kKeep];
  // the same per-thread order as cf_rmsnorm (vectors v = tid, tid + blockDim, ...): same sums
#pragma unroll
  for (int k = 0; k < kKeep; ++k) {
    const int v = threadIdx.x + k * blockDim.x;
    kept[k] = make_uint4(0, 0, 0, 0);
    if (v >= dim / 8) continue;
    float f8[8];
    reduce8<T>(part, splits, plane, (int64_t)m * n + v * 8, res ? res + (int64_t)m * ldr + v * 8 : nullptr, f8);
    uint4 o;
    T *op = reinterpret_cast<T *>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) op[j] = from_f<T>(f8[j]);
    reinterpret_cast<uint4 *>(yr)[v] = o;
    kept[k] = o;
    cf::Vec16<T> pk;
    pk.raw = o;
#pragma unroll
    for (int j = 0; j < 8; ++j) { const float f = pk.get(j); ss += f * f; }
  }
  for (int v = threadIdx.x + kKeep * blockDim.x; v < dim / 8; v += blockDim.x) {  // very wide rows
    float f8[8];
    reduce8<T>(part, splits, plane, (int64_t)m * n + v * 8, res ? res + (int64_t)m * ldr + v * 8 : nullptr, f8);
    uint4 o;
    T *op = reinterpret_cast<T *>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) op[j] = from_f<T>(f8[j]);
    reinterpret_cast<uint4 *>(yr)[v] = o;
    cf::Vec16<T> pk;
    pk.raw = o;
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
  auto norm_store = [&](int v, const uint4 raw) {
    cf::Vec16<T> pk, pw;
    pk.raw = raw;
    pw.raw = reinterpret_cast<const uint4 *>(w)[v];
    uint4 o;
    T *op = reinterpret_cast<T *>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) op[j] = from_f<T>(pk.get(j) * inv * pw.get(j));
    reinterpret_cast<uint4 *>(orow)[v] = o;
  };
#pragma unroll
  for (int k = 0; k < kKeep; ++k) {
    const int v = threadIdx.x + k * blockDim.x;
    if (v < dim / 8) norm_store(v, kept[k]);
  }
  for (int v = threadIdx.x + kKeep * blockDim.x; v < dim / 8; v += blockDim.x)
    norm_store(v, reinterpret_cast<const uint4 *>(yr)[v]);  // this thread's own values, written above
}

// The RoPE / K-V scatter of rope_qkv_kernel on T(sum of partials); rotated q goes to qkv.
template <typename T>
__global__ void splitk_rope_qkv_kernel(const float *part, int splits, int64_t plane, int n, T *qkv, int64_t ld,
                                       int Hq, int Hkv, int D, const int32_t *pos, float log2_base, T *k_new,
                                       T *v_new) {
  const int m = blockIdx.x;
  T *row = qkv + (int64_t)m * ld;
  const float *prow = part + (int64_t)m * n;
  __shared__ float2 tab[kMaxHalf];
  rope_table((float)pos[m], D, log2_base, tab);
  const int half = D / 2, q4 = half / 4;
  const int items = (Hq + Hkv) * q4;
  // four GEMM outputs at column col, reduced in split order and rounded to T
  auto val4 = [&](int col, float (&o)[4]) {
    float4 a = *reinterpret_cast<const float4 *>(prow + col);
    for (int sp = 1; sp < splits; ++sp) {
      const float4 c = *reinterpret_cast<const float4 *>(prow + sp * plane + col);
      a.x += c.x; a.y += c.y; a.z += c.z; a.w += c.w;
    }
    o[0] = cf::to_float(from_f<T>(a.x)); o[1] = cf::to_float(from_f<T>(a.y));
    o[2] = cf::to_float(from_f<T>(a.z)); o[3] = cf::to_float(from_f<T>(a.w));
  };
  for (int idx = threadIdx.x; idx < items; idx += blockDim.x) {
    const int hh = idx / q4, i0 = (idx % q4) * 4;
    float x1[4], x2[4], o1[4], o2[4];
    val4(hh * D + i0, x1);
    val4(hh * D + i0 + half, x2);
    rope4(tab, i0, x1, x2, o1, o2);
    T *dst = rope_dst(row, k_new, m, hh, Hq, Hkv, D);
    store4(dst + i0, o1);
    store4(dst + i0 + half, o2);
  }
  T *vdst = v_new + (int64_t)m * Hkv * D;
  const int v0 = (Hq + Hkv) * D;
  for (int v = threadIdx.x; v < Hkv * D / 8; v += blockDim.x) {
    float f8[8];
    reduce8<T>(part, splits, plane, (int64_t)m * n + v0 + v * 8, nullptr, f8);
    uint4 o;
    T *op = reinterpret_cast<T *>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) op[j] = from_f<T>(f8[j]);
    reinterpret_cast<uint4 *>(vdst)[v] = o;
  }
}

// SwiGLU on T(sum of partials) of the fused gate|up rows.
template <typename T>
__global__ void splitk_silu_mul_kernel(const float *part, int splits, int64_t plane, int n, T *out, int64_t ldo,
                                       int ffn) {
  const int m = blockIdx.y;
  T *o = out + (int64_t)m * ldo;
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < ffn / 8; v += gridDim.x * blockDim.x) {
    float g8[8], u8[8];
    reduce8<T>(part, splits, plane, (int64_t)m * n + v * 8, nullptr, g8);
    reduce8<T>(part, splits, plane, (int64_t)m * n + ffn + v * 8, nullptr, u8);
    uint4 r;
    T *rp = reinterpret_cast<T *>(&r);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float x = cf::to_float(from_f<T>(g8[j]));
      rp[j] = from_f<T>(x / (1.0f + expf(-x)) * cf::to_float(from_f<T>(u8[j])));
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
  if (m < 0 || head_dim % 16 || head_dim > 2 * kMaxHalf || num_q_heads <= 0 || num_kv_heads <= 0 || !qkv || !pos || !k_new || !v_new)
    return CF_EINVAL;
  if (ld % 8 || !aligned16(qkv) || !aligned16(k_new) || !aligned16(v_new) || !(base > 1.0f)) return CF_EINVAL;
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

extern "C" int cf_splitk_rmsnorm(const float *partials, int32_t splits, int32_t m, int32_t n, const void *residual,
                                 int64_t ldr, void *y, int64_t ldy, const void *w, void *out, int64_t ldo, float eps,
                                 int32_t dtype, void *stream) {
  if (m < 0 || n <= 0 || n % 8 || splits < 1 || ldy % 8 || ldo % 8 || (residual && ldr % 8)) return CF_EINVAL;
  if (!partials || !y || !w || !out || !aligned16(partials) || !aligned16(y) || !aligned16(w) || !aligned16(out) ||
      (residual && !aligned16(residual)))
    return CF_EINVAL;
  if (m == 0) return CF_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int threads = n >= 4096 ? 512 : 128;  // as cf_rmsnorm: the same reduction order
  const int64_t plane = (int64_t)m * n;
  if (dtype == CF_BF16)
    splitk_rmsnorm_kernel<<<m, threads, 0, s>>>(partials, splits, plane, n, (const __nv_bfloat16 *)residual, ldr,
                                                (__nv_bfloat16 *)y, ldy, (const __nv_bfloat16 *)w,
                                                (__nv_bfloat16 *)out, ldo, n, eps);
  else if (dtype == CF_F16)
    splitk_rmsnorm_kernel<<<m, threads, 0, s>>>(partials, splits, plane, n, (const __half *)residual, ldr,
                                                (__half *)y, ldy, (const __half *)w, (__half *)out, ldo, n, eps);
  else
    return CF_EINVAL;
  return cf_launch_status();
}

extern "C" int cf_splitk_rope_qkv(const float *partials, int32_t splits, int32_t m, void *qkv, int64_t ld,
                                  int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, const int32_t *pos,
                                  float base, void *k_new, void *v_new, int32_t dtype, void *stream) {
  if (m < 0 || splits < 1 || head_dim % 16 || head_dim > 2 * kMaxHalf || num_q_heads <= 0 || num_kv_heads <= 0 ||
      !partials || !qkv || !pos || !k_new || !v_new)
    return CF_EINVAL;
  if (ld % 8 || !aligned16(partials) || !aligned16(qkv) || !aligned16(k_new) || !aligned16(v_new) || !(base > 1.0f))
    return CF_EINVAL;
  if (m == 0) return CF_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const float lb = log2f(base);
  const int n = (num_q_heads + 2 * num_kv_heads) * head_dim;
  const int64_t plane = (int64_t)m * n;
  if (dtype == CF_BF16)
    splitk_rope_qkv_kernel<<<m, 256, 0, s>>>(partials, splits, plane, n, (__nv_bfloat16 *)qkv, ld, num_q_heads,
                                             num_kv_heads, head_dim, pos, lb, (__nv_bfloat16 *)k_new,
                                             (__nv_bfloat16 *)v_new);
  else if (dtype == CF_F16)
    splitk_rope_qkv_kernel<<<m, 256, 0, s>>>(partials, splits, plane, n, (__half *)qkv, ld, num_q_heads,
                                             num_kv_heads, head_dim, pos, lb, (__half *)k_new, (__half *)v_new);
  else
    return CF_EINVAL;
  return cf_launch_status();
}

extern "C" int cf_splitk_silu_mul(const float *partials, int32_t splits, int32_t m, int32_t ffn, void *out,
                                  int64_t ldo, int32_t dtype, void *stream) {
  if (m < 0 || splits < 1 || ffn <= 0 || ffn % 8 || ldo % 8 || !partials || !out || !aligned16(partials) ||
      !aligned16(out))
    return CF_EINVAL;
  if (m == 0) return CF_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid((ffn / 8 + 255) / 256, m);
  const int n = 2 * ffn;
  const int64_t plane = (int64_t)m * n;
  if (dtype == CF_BF16)
    splitk_silu_mul_kernel<<<grid, 256, 0, s>>>(partials, splits, plane, n, (__nv_bfloat16 *)out, ldo, ffn);
  else if (dtype == CF_F16)
    splitk_silu_mul_kernel<<<grid, 256, 0, s>>>(partials, splits, plane, n, (__half *)out, ldo, ffn);
  else
    return CF_EINVAL;
  return cf_launch_status();
}
