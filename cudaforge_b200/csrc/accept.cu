// Fused acceptance sampling for speculative decoding (sm_100a).
//
// Replaces the reference's CPU verifier SpeculativeEngine::verify_candidates
// / verify_candidates_greedy (csrc/src/scheduler/speculative.cpp:50-150) and
// the two vocab-wide softmaxes of cudaforge/speculative.py:118, :145.
//
// Two launches on the caller's stream:
//   1. row_stats_kernel  grid (2K+1, B): one CTA streams one logits row with
//      16-byte vector loads and keeps an online (max, sum) of
//      exp2(x * log2(e)/T - max) per thread, merged by a fixed-order block
//      reduction.  This pass reads every logit exactly once and is the
//      HBM-bound part (B*(2K+1)*V*sizeof(logit) bytes).
//   2. decide_kernel     grid (B): one CTA per sequence evaluates the K
//      acceptance tests, then the single draw (residual, target fallback or
//      bonus) with the reference's sequential fp32 inverse CDF, or the greedy
//      argmax chain.
// The probability of element x in a row with stats (mc, s) is, everywhere in
// this file (and in the optional parity export),
//     P(x) = exp2f(fl(x * c) - mc) / s,   c = log2(e) / T,
// computed with explicit round-to-nearest intrinsics (no FMA contraction), so
// the value a decision sees is the value the parity export writes.
#include "common.cuh"

#include <math.h>

namespace {

constexpr int kStatsThreads = 512;
constexpr int kDecideThreads = 256;  // warp 0 runs the serial chain, warps 1-7 produce
constexpr int kChunk = 2048;         // elements per double-buffered chunk

struct RowStat {
  float mc;  // max_i fl(x_i * c)
  float s;   // sum_i exp2f(fl(x_i * c) - mc), fixed reduction order
};

template <typename T>
__device__ __forceinline__ const T *row_ptr(const void *base, int64_t seq_stride,
                                            int64_t row_stride, int b, int r) {
  return reinterpret_cast<const T *>(base) + (int64_t)b * seq_stride + (int64_t)r * row_stride;
}

__device__ __forceinline__ float prob_of(float x, float c, RowStat st) {
  float t = __fsub_rn(__fmul_rn(x, c), st.mc);
  return __fdiv_rn(exp2f(t), st.s);
}

__device__ __forceinline__ void merge_stat(float &m, float &s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) { m = m2; s = s2; return; }
  float mn = fmaxf(m, m2);
  s = __fadd_rn(__fmul_rn(s, exp2f(__fsub_rn(m, mn))), __fmul_rn(s2, exp2f(__fsub_rn(m2, mn))));
  m = mn;
}

// ---------------------------------------------------------------------------
// Pass 1: per-row (max, sum).  Row r < K is draft row r, r >= K target row r-K.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kStatsThreads)
row_stats_kernel(cf_accept_args a, float c, RowStat *stats) {
  const int r = blockIdx.x, b = blockIdx.y;
  const int rows = 2 * a.k + 1;
  if (r < a.k && a.draft_logits == nullptr) {  // greedy without draft logits
    if (threadIdx.x == 0) stats[(int64_t)b * rows + r] = RowStat{-INFINITY, 0.0f};
    return;
  }
  const T *x = (r < a.k) ? row_ptr<T>(a.draft_logits, a.draft_seq_stride, a.draft_row_stride, b, r)
                         : row_ptr<T>(a.target_logits, a.target_seq_stride, a.target_row_stride, b, r - a.k);
  const int64_t V = a.vocab;
  float m = -INFINITY, s = 0.0f;
  constexpr int N = cf::Vec16<T>::N;
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  int64_t head = 0;
  if (vec_ok) {
    const int64_t nvec = V / N;
    const uint4 *xv = reinterpret_cast<const uint4 *>(x);
    for (int64_t v = threadIdx.x; v < nvec; v += kStatsThreads) {
      cf::Vec16<T> pk;
      pk.raw = __ldcs(xv + v);  // streamed once: do not keep in L1/L2
      float t[N];
      float cm = -INFINITY;
#pragma unroll
      for (int j = 0; j < N; ++j) {
        t[j] = __fmul_rn(pk.get(j), c);
        cm = fmaxf(cm, t[j]);
      }
      if (cm > m) {
        if (m != -INFINITY) s = __fmul_rn(s, exp2f(__fsub_rn(m, cm)));
        m = cm;
      }
      if (m != -INFINITY) {
#pragma unroll
        for (int j = 0; j < N; ++j) s = __fadd_rn(s, exp2f(__fsub_rn(t[j], m)));
      }
    }
    head = nvec * N;
  }
  for (int64_t i = head + threadIdx.x; i < V; i += kStatsThreads) {
    float t = __fmul_rn(cf::to_float(x[i]), c);
    if (t > m) {
      if (m != -INFINITY) s = __fmul_rn(s, exp2f(__fsub_rn(m, t)));
      m = t;
    }
    if (m != -INFINITY) s = __fadd_rn(s, exp2f(__fsub_rn(t, m)));
  }
  // fixed-order reduction: warp butterfly, then warp 0 over the warp results
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    merge_stat(m, s, m2, s2);
  }
  __shared__ float sm[kStatsThreads / 32], ss[kStatsThreads / 32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { sm[w] = m; ss[w] = s; }
  __syncthreads();
  if (w == 0) {
    m = (l < kStatsThreads / 32) ? sm[l] : -INFINITY;
    s = (l < kStatsThreads / 32) ? ss[l] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      merge_stat(m, s, m2, s2);
    }
    if (l == 0) stats[(int64_t)b * rows + r] = RowStat{m, s};
  }
}

// ---------------------------------------------------------------------------
// Optional parity export of the probabilities the decisions use.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void export_probs_kernel(cf_accept_args a, float c, const RowStat *stats) {
  const int r = blockIdx.x, b = blockIdx.y;
  const int rows = 2 * a.k + 1;
  const bool draft = r < a.k;
  if (draft ? (a.probs_draft == nullptr || a.draft_logits == nullptr) : a.probs_target == nullptr) return;
  const T *x = draft ? row_ptr<T>(a.draft_logits, a.draft_seq_stride, a.draft_row_stride, b, r)
                     : row_ptr<T>(a.target_logits, a.target_seq_stride, a.target_row_stride, b, r - a.k);
  float *out = draft ? a.probs_draft + ((int64_t)b * a.k + r) * a.vocab
                     : a.probs_target + ((int64_t)b * (a.k + 1) + (r - a.k)) * a.vocab;
  const RowStat st = stats[(int64_t)b * rows + r];
  for (int64_t i = threadIdx.x; i < a.vocab; i += blockDim.x) out[i] = prob_of(cf::to_float(x[i]), c, st);
}

// ---------------------------------------------------------------------------
// Pass 2 helpers: the reference's sequential fp32 chains, run by one thread
// over double-buffered chunks that warps 1-7 fill in parallel.
// ---------------------------------------------------------------------------
struct ChainShared {
  float buf[2][kChunk];
  int64_t found;
  float total;
};

// Returns the fp32 sum  ((v0 + v1) + v2) + ...  in index order.
template <class F>
__device__ float serial_sum(F f, int64_t V, ChainShared &sh) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t nch = (V + kChunk - 1) / kChunk;
  auto fill = [&](int64_t ch) {
    const int64_t base = ch * kChunk;
    const int n = (int)((V - base) < kChunk ? (V - base) : kChunk);
    float *dst = sh.buf[ch & 1];
    for (int j = tid - 32; j < n; j += kDecideThreads - 32) dst[j] = f(base + j);
  };
  if (warp != 0) fill(0);
  float acc = 0.0f;
  __syncthreads();
  for (int64_t ch = 0; ch < nch; ++ch) {
    if (warp != 0) {
      if (ch + 1 < nch) fill(ch + 1);
    } else if (lane == 0) {
      const int n = (int)((V - ch * kChunk) < kChunk ? (V - ch * kChunk) : kChunk);
      const float *src = sh.buf[ch & 1];
      int j = 0;
      for (; j + 4 <= n; j += 4) {
        float4 v = *reinterpret_cast<const float4 *>(src + j);
        acc = __fadd_rn(acc, v.x);
        acc = __fadd_rn(acc, v.y);
        acc = __fadd_rn(acc, v.z);
        acc = __fadd_rn(acc, v.w);
      }
      for (; j < n; ++j) acc = __fadd_rn(acc, src[j]);
    }
    __syncthreads();
  }
  if (tid == 0) sh.total = acc;
  __syncthreads();
  float t = sh.total;
  __syncthreads();
  return t;
}

// Returns the first index i with r <= (v0 + ... + vi) (sequential fp32), or
// V-1 when no prefix reaches r.
template <class F>
__device__ int64_t serial_search(F f, int64_t V, float r, ChainShared &sh) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t nch = (V + kChunk - 1) / kChunk;
  auto fill = [&](int64_t ch) {
    const int64_t base = ch * kChunk;
    const int n = (int)((V - base) < kChunk ? (V - base) : kChunk);
    float *dst = sh.buf[ch & 1];
    for (int j = tid - 32; j < n; j += kDecideThreads - 32) dst[j] = f(base + j);
  };
  if (tid == 0) sh.found = -1;
  if (warp != 0) fill(0);
  float cum = 0.0f;
  __syncthreads();
  for (int64_t ch = 0; ch < nch; ++ch) {
    if (warp != 0) {
      if (ch + 1 < nch) fill(ch + 1);
    } else if (lane == 0) {
      const int64_t base = ch * kChunk;
      const int n = (int)((V - base) < kChunk ? (V - base) : kChunk);
      const float *src = sh.buf[ch & 1];
      int j = 0;
      int hit = -1;
      for (; j + 4 <= n; j += 4) {
        float4 v = *reinterpret_cast<const float4 *>(src + j);
        float c0 = __fadd_rn(cum, v.x);
        float c1 = __fadd_rn(c0, v.y);
        float c2 = __fadd_rn(c1, v.z);
        float c3 = __fadd_rn(c2, v.w);
        if (r <= c0) { hit = j; break; }
        if (r <= c1) { hit = j + 1; break; }
        if (r <= c2) { hit = j + 2; break; }
        if (r <= c3) { hit = j + 3; break; }
        cum = c3;
      }
      if (hit < 0) {
        for (; j < n; ++j) {
          cum = __fadd_rn(cum, src[j]);
          if (r <= cum) { hit = j; break; }
        }
      }
      if (hit >= 0) sh.found = base + hit;
    }
    __syncthreads();
    if (sh.found >= 0) break;
  }
  int64_t res = sh.found >= 0 ? sh.found : V - 1;
  __syncthreads();
  return res;
}

// First index of the largest P value in a row (std::max_element semantics).
template <typename T>
__device__ int64_t block_argmax(const T *x, int64_t V, float c, RowStat st) {
  const int tid = threadIdx.x;
  float best = -INFINITY;
  int64_t bi = INT64_MAX;
  for (int64_t i = tid; i < V; i += kDecideThreads) {
    float p = prob_of(cf::to_float(x[i]), c, st);
    if (p > best || bi == INT64_MAX) { best = p; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float b2 = __shfl_xor_sync(0xffffffffu, best, o);
    int64_t i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    if (b2 > best || (b2 == best && i2 < bi)) { best = b2; bi = i2; }
  }
  __shared__ float sb[kDecideThreads / 32];
  __shared__ int64_t si[kDecideThreads / 32];
  const int w = tid >> 5, l = tid & 31;
  if (l == 0) { sb[w] = best; si[w] = bi; }
  __syncthreads();
  if (tid == 0) {
    for (int k = 1; k < kDecideThreads / 32; ++k)
      if (sb[k] > sb[0] || (sb[k] == sb[0] && si[k] < si[0])) { sb[0] = sb[k]; si[0] = si[k]; }
  }
  __syncthreads();
  int64_t res = si[0];
  __syncthreads();
  return res;
}

enum Mode : int { kDone = 0, kResidual = 1, kBonus = 2 };

template <typename T>
__global__ void __launch_bounds__(kDecideThreads)
decide_kernel(cf_accept_args a, float c, const RowStat *stats) {
  __shared__ ChainShared sh;
  __shared__ int s_mode, s_row, s_na;
  __shared__ float s_r;
  const int b = blockIdx.x, tid = threadIdx.x;
  const int K = a.k, rows = 2 * K + 1;
  const int64_t V = a.vocab;
  const RowStat *st = stats + (int64_t)b * rows;
  const int32_t *dt = a.draft_tokens + (int64_t)b * K;
  int32_t *out = a.out_tokens + (int64_t)b * (K + 1);

  if (a.greedy) {
    // speculative.cpp:105-150: accept while draft == argmax(target row i).
    int na = 0;
    for (int i = 0; i <= K; ++i) {
      const T *xt = row_ptr<T>(a.target_logits, a.target_seq_stride, a.target_row_stride, b, i);
      int64_t am = block_argmax<T>(xt, V, c, st[K + i]);
      if (i == K) {
        if (tid == 0) { out[na] = (int32_t)am; a.out_num_accepted[b] = na; a.out_eos[b] = (am == a.eos_token_id); }
        return;
      }
      const int32_t tok = dt[i];  // compared only, never indexed (as the reference)
      if (tok == am) {
        if (tid == 0) out[na] = tok;
        ++na;
        if (tok == a.eos_token_id) {
          if (tid == 0) { out[na] = tok; a.out_num_accepted[b] = na; a.out_eos[b] = 1; }
          return;
        }
      } else {
        if (tid == 0) { out[na] = (int32_t)am; a.out_num_accepted[b] = na; a.out_eos[b] = (am == a.eos_token_id); }
        return;
      }
    }
    return;
  }

  // speculative.cpp:66-101: sequential tests (K is small; thread 0 does them).
  if (tid == 0) {
    const float *u = a.uniforms + (int64_t)b * (K + 1);
    int na = 0, used = 0, mode = kBonus, row = K;
    bool bad = false;
    for (int i = 0; i < K; ++i) {
      const int32_t tok = dt[i];
      if (tok < 0 || tok >= V) { bad = true; break; }
      const T *xd = row_ptr<T>(a.draft_logits, a.draft_seq_stride, a.draft_row_stride, b, i);
      const T *xt = row_ptr<T>(a.target_logits, a.target_seq_stride, a.target_row_stride, b, i);
      const float q = prob_of(cf::to_float(xd[tok]), c, st[i]);
      const float p = prob_of(cf::to_float(xt[tok]), c, st[K + i]);
      const float pq = __fdiv_rn(p, q);
      const float ratio = (q > 0.0f) ? ((pq < 1.0f) ? pq : 1.0f) : 0.0f;
      const float r = u[used++];
      if (r <= ratio) {
        out[na++] = tok;
        if (tok == a.eos_token_id) { mode = kDone; break; }
      } else {
        mode = kResidual;
        row = i;
        break;
      }
    }
    if (bad) {
      a.out_num_accepted[b] = -1;
      a.out_eos[b] = 0;
      s_mode = -1;
    } else {
      s_mode = mode;
      s_row = row;
      s_na = na;
      s_r = (mode == kDone) ? 0.0f : u[used];
      if (mode == kDone) { out[na] = a.eos_token_id; a.out_num_accepted[b] = na; a.out_eos[b] = 1; }
    }
  }
  __syncthreads();
  const int mode = s_mode;
  if (mode == kDone || mode < 0) return;
  const int row = s_row;
  const float r = s_r;
  int64_t tok;
  const T *xt = row_ptr<T>(a.target_logits, a.target_seq_stride, a.target_row_stride, b, row);
  const RowStat stt = st[K + row];
  auto p_of = [&](int64_t i) { return prob_of(cf::to_float(xt[i]), c, stt); };
  if (mode == kResidual) {
    // speculative.cpp:26-48
    const T *xd = row_ptr<T>(a.draft_logits, a.draft_seq_stride, a.draft_row_stride, b, row);
    const RowStat std_ = st[row];
    auto resid = [&](int64_t i) {
      float d = __fsub_rn(p_of(i), prob_of(cf::to_float(xd[i]), c, std_));
      return d > 0.0f ? d : 0.0f;  // std::max(0.0f, d)
    };
    const float sum = serial_sum(resid, V, sh);
    if (sum <= 1e-6f) {
      tok = serial_search(p_of, V, r, sh);
    } else {
      auto normed = [&](int64_t i) { return __fdiv_rn(resid(i), sum); };
      tok = serial_search(normed, V, r, sh);
    }
  } else {
    tok = serial_search(p_of, V, r, sh);  // bonus, speculative.cpp:97
  }
  if (tid == 0) {
    out[s_na] = (int32_t)tok;
    a.out_num_accepted[b] = s_na;
    a.out_eos[b] = (tok == a.eos_token_id);
  }
}

template <typename T>
int launch_accept(const cf_accept_args &a, cudaStream_t stream) {
  const float c = (float)(1.4426950408889634 / (double)a.temperature);
  RowStat *stats = reinterpret_cast<RowStat *>(a.workspace);
  dim3 g1(2 * a.k + 1, a.batch);
  row_stats_kernel<T><<<g1, kStatsThreads, 0, stream>>>(a, c, stats);
  if (a.probs_draft || a.probs_target) export_probs_kernel<T><<<g1, 256, 0, stream>>>(a, c, stats);
  decide_kernel<T><<<a.batch, kDecideThreads, 0, stream>>>(a, c, stats);
  return cf_launch_status();
}

}  // namespace

extern "C" size_t cf_accept_workspace_bytes(int32_t batch, int32_t k) {
  if (batch < 0 || k < 0) return 0;
  return (size_t)batch * (2 * (size_t)k + 1) * sizeof(RowStat);
}

extern "C" int cf_accept_sample(const cf_accept_args *args, void *stream) {
  if (!args) return CF_EINVAL;
  const cf_accept_args &a = *args;
  if (a.batch < 0 || a.k < 0 || a.vocab < 1 || a.vocab > INT32_MAX) return CF_EINVAL;
  if (a.batch == 0) return CF_OK;
  if (!(a.temperature > 0.0f) || !isfinite(a.temperature)) return CF_EINVAL;
  if (!a.target_logits || !a.out_tokens || !a.out_num_accepted || !a.out_eos || !a.workspace) return CF_EINVAL;
  if (a.k > 0 && (!a.draft_tokens || (!a.greedy && !a.draft_logits))) return CF_EINVAL;
  if (!a.greedy && !a.uniforms) return CF_EINVAL;
  if ((reinterpret_cast<uintptr_t>(a.workspace) & 15) != 0) return CF_EINVAL;
  if (a.target_row_stride < a.vocab || (a.k > 0 && a.draft_row_stride < a.vocab)) return CF_EINVAL;
  if (2 * (int64_t)a.k + 1 > 65535 || a.batch > 65535) return CF_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (a.logits_dtype) {
    case CF_F32: return launch_accept<float>(a, s);
    case CF_BF16: return launch_accept<__nv_bfloat16>(a, s);
    case CF_F16: return launch_accept<__half>(a, s);
    default: return CF_EINVAL;
  }
}
