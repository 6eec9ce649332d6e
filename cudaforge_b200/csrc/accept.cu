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

#include <limits.h>
#include <mutex>
#include <math.h>

namespace {

constexpr int kStatsThreads = 512;
constexpr int kDecideThreads = 512;

struct RowStat {
  float mc;  // max_i fl(x_i * c)
  float s;   // sum_i exp2f(fl(x_i * c) - mc), fixed reduction order
};

template <typename T>
__device__ __forceinline__ const T *row_ptr(const void *base, int64_t seq_stride,
                                            int64_t row_stride, int b, int r) {
  return reinterpret_cast<const T *>(base) + (int64_t)b * seq_stride + (int64_t)r * row_stride;
}

// Eight consecutive logits as floats (16-B vector load when aligned).
template <typename T>
__device__ __forceinline__ void load8(const T *x, int64_t i0, int64_t V, float (&o)[8]) {
  const T *p = x + i0;
  if (i0 + 8 <= V && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    if constexpr (sizeof(T) == 2) {
      cf::Vec16<T> pk;
      pk.raw = *reinterpret_cast<const uint4 *>(p);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = pk.get(j);
    } else {
      const float4 a = reinterpret_cast<const float4 *>(p)[0], b = reinterpret_cast<const float4 *>(p)[1];
      o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = (i0 + j < V) ? cf::to_float(p[j]) : 0.0f;
  }
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
row_stats_kernel(cf_accept_args a, float c, RowStat *stats, int ndraft, int ntarget) {
  const int r = blockIdx.x, b = blockIdx.y;
  const int rows = ndraft + ntarget;
  if (r < ndraft && a.draft_logits == nullptr) {  // greedy without draft logits
    if (threadIdx.x == 0) stats[(int64_t)b * rows + r] = RowStat{-INFINITY, 0.0f};
    return;
  }
  const T *x = (r < ndraft) ? row_ptr<T>(a.draft_logits, a.draft_seq_stride, a.draft_row_stride, b, r)
                            : row_ptr<T>(a.target_logits, a.target_seq_stride, a.target_row_stride, b, r - ndraft);
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
__global__ void export_probs_kernel(cf_accept_args a, float c, const RowStat *stats, int ndraft, int ntarget) {
  const int r = blockIdx.x, b = blockIdx.y;
  const int rows = ndraft + ntarget;
  const bool draft = r < ndraft;
  if (draft ? (a.probs_draft == nullptr || a.draft_logits == nullptr) : a.probs_target == nullptr) return;
  const T *x = draft ? row_ptr<T>(a.draft_logits, a.draft_seq_stride, a.draft_row_stride, b, r)
                     : row_ptr<T>(a.target_logits, a.target_seq_stride, a.target_row_stride, b, r - ndraft);
  float *out = draft ? a.probs_draft + ((int64_t)b * ndraft + r) * a.vocab
                     : a.probs_target + ((int64_t)b * ntarget + (r - ndraft)) * a.vocab;
  const RowStat st = stats[(int64_t)b * rows + r];
  for (int64_t i = threadIdx.x; i < a.vocab; i += blockDim.x) out[i] = prob_of(cf::to_float(x[i]), c, st);
}

// ---------------------------------------------------------------------------
// Pass 2: the reference's sequential fp32 accumulation, computed exactly in
// parallel.
//
// The reference accumulates `cum += v_i` left to right in fp32
// (speculative.cpp:16-21, :34-35).  All v_i here are >= 0, so cum never
// decreases.  While cum stays inside one binade [2^e, 2^(e+1)) (ulp u = 2^ue,
// ue = max(e, -126) - 23) every partial sum is an integer multiple C*u with
// C < 2^24, and fl(C*u + v) = (C + inc)*u where inc is v/u rounded to nearest,
// ties to the even RESULT: the increment depends on v and on C's parity only.
// Each element is therefore a map on (C mod 2) -> increment, and maps compose
// associatively: a block-wide scan of these maps gives every exact partial
// sum of a chunk at once.  An element whose sum leaves the binade (or meets a
// NaN / Inf) is applied directly in fp32 by the thread that owns it and the
// chunk resumes after it; the binade index only grows, so this happens a few
// dozen times per row at most.  The result is bit-identical to the serial
// loop.
// ---------------------------------------------------------------------------
constexpr int kScanThreads = 512;
constexpr int kPerThread = 8;
constexpr int kScanChunk = kScanThreads * kPerThread;
constexpr int kSat = 1 << 26;
constexpr int kTop = 1 << 24;

struct IncMap {
  int e, o;  // ulps added when the running integer is even / odd
};

__device__ __forceinline__ int sat_add(int a, int b) { return min(a + b, kSat); }

// f, then g
__device__ __forceinline__ IncMap compose(IncMap f, IncMap g) {
  IncMap r;
  r.e = sat_add(f.e, (f.e & 1) ? g.o : g.e);
  r.o = sat_add(f.o, ((1 + f.o) & 1) ? g.o : g.e);
  return r;
}

__device__ __forceinline__ int apply(IncMap f, int C) { return C + ((C & 1) ? f.o : f.e); }

// The increment map of adding v (>= 0) on the ulp grid 2^ue.  Values the grid
// model cannot represent (NaN, Inf, or a jump past the binade) saturate,
// which forces the direct fp32 path.
__device__ __forceinline__ IncMap elem_map(float v, int ue) {
  const uint32_t bits = __float_as_uint(v);
  const int ex = (bits >> 23) & 0xff;
  uint32_t m = bits & 0x7fffffu;
  if (ex == 0xff) return {kSat, kSat};
  if (ex) m |= 0x800000u;
  if (m == 0) return {0, 0};
  const int ulp_v = (ex ? ex : 1) - 127 - 23;
  const int s = ue - ulp_v;  // v / u = m * 2^-s
  if (s <= 0) {
    if (-s >= 3) return {kSat, kSat};
    const int A = (int)(m << (-s));
    return {A, A};
  }
  if (s >= 25) return {0, 0};  // v < u/2
  const uint32_t fl = m >> s, rem = m & ((1u << s) - 1u), half = 1u << (s - 1);
  if (rem < half) return {(int)fl, (int)fl};
  if (rem > half) return {(int)fl + 1, (int)fl + 1};
  return {(int)(fl + (fl & 1u)), (int)(fl + ((fl & 1u) ^ 1u))};  // tie: round to the even result
}

__device__ __forceinline__ void grid_of(float c, int &C, int &ue) {
  const uint32_t bits = __float_as_uint(c);
  const int ex = (bits >> 23) & 0xff;
  ue = (ex ? ex : 1) - 127 - 23;
  C = (int)((bits & 0x7fffffu) | (ex ? 0x800000u : 0u));
}

struct ScanShared {
  IncMap warp_tot[kScanThreads / 32];
  IncMap warp_pre[kScanThreads / 32];
  float c;    // running sum after the processed prefix
  int pos;    // first unprocessed chunk-local index
  int cross;  // first chunk-local index leaving the grid model
  int found;  // first chunk-local index with r <= cum
  int done;
};

// Exclusive block scan of IncMap (thread order).
__device__ __forceinline__ IncMap block_exclusive_scan(IncMap x, ScanShared &sh) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  IncMap inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    IncMap y;
    y.e = __shfl_up_sync(0xffffffffu, inc.e, o);
    y.o = __shfl_up_sync(0xffffffffu, inc.o, o);
    if (lane >= o) inc = compose(y, inc);
  }
  if (lane == 31) sh.warp_tot[w] = inc;
  __syncthreads();
  if (w == 0) {
    IncMap ti = lane < kScanThreads / 32 ? sh.warp_tot[lane] : IncMap{0, 0};
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      IncMap y;
      y.e = __shfl_up_sync(0xffffffffu, ti.e, o);
      y.o = __shfl_up_sync(0xffffffffu, ti.o, o);
      if (lane >= o) ti = compose(y, ti);
    }
    IncMap ex;
    ex.e = __shfl_up_sync(0xffffffffu, ti.e, 1);
    ex.o = __shfl_up_sync(0xffffffffu, ti.o, 1);
    if (lane == 0) ex = IncMap{0, 0};
    if (lane < kScanThreads / 32) sh.warp_pre[lane] = ex;
  }
  __syncthreads();
  IncMap lex;
  lex.e = __shfl_up_sync(0xffffffffu, inc.e, 1);
  lex.o = __shfl_up_sync(0xffffffffu, inc.o, 1);
  if (lane == 0) lex = IncMap{0, 0};
  return compose(sh.warp_pre[w], lex);
}

// Sequential fp32 accumulation cum += v_i for i in [lo, hi), starting from the
// exact value c0, of the values (all >= 0 or NaN/Inf) that f(i0, out[8])
// produces eight at a time.  Returns the running value after the range (or
// after the hit / the first NaN / Inf, which ends the chain: nothing later
// can match or change a NaN, and an Inf is final for the searches here).
// SEARCH: *hit = the first i in the range with r <= cum_i, else -1.
template <bool SEARCH, class F>
__device__ float exact_chain_range(F f, int64_t lo, int64_t hi, float c0, float r, int64_t *hit, ScanShared &sh) {
  const int tid = threadIdx.x;
  if (tid == 0) { sh.c = c0; sh.done = 0; }
  __syncthreads();
  int64_t result = -1;
  for (int64_t base = lo; base < hi; base += kScanChunk) {
    const int n = (int)((hi - base) < kScanChunk ? (hi - base) : kScanChunk);
    float v[kPerThread];
#pragma unroll
    for (int j = 0; j < kPerThread; j += 8) {
      const int li = tid * kPerThread + j;
      float t8[8];
      if (li < n) f(base + li, t8);
#pragma unroll
      for (int q = 0; q < 8; ++q) v[j + q] = (li + q < n) ? t8[q] : 0.0f;
    }
    if (tid == 0) sh.pos = 0;
    __syncthreads();
    while (true) {
      const int pos = sh.pos;
      const float c0 = sh.c;
      if (pos >= n) break;
      if (tid == 0) { sh.cross = INT_MAX; sh.found = INT_MAX; }
      int C0, ue;
      grid_of(c0, C0, ue);
      IncMap loc{0, 0};
      IncMap em[kPerThread];  // this thread's element maps on the current grid (0 outside [pos, n))
#pragma unroll
      for (int j = 0; j < kPerThread; ++j) {
        const int li = tid * kPerThread + j;
        em[j] = (li >= pos && li < n) ? elem_map(v[j], ue) : IncMap{0, 0};
        loc = compose(loc, em[j]);
      }
      const IncMap pre = block_exclusive_scan(loc, sh);  // its barriers order the resets above
      int C = apply(pre, C0);
      if (C >= kTop) C = kTop;  // a crossing lies before this thread's elements
      int my_cross = INT_MAX, my_found = INT_MAX;
      // The running value only grows, so the exact value after this thread's last element
      // (apply(loc, C), below kTop exactly when no element of the range leaves the grid) tells
      // whether the range holds a crossing or, when searching, the first r <= cum: most
      // threads then skip the element walk.
      const int Cend = C < kTop ? apply(loc, C) : kTop;
      const bool walk = C < kTop && (Cend >= kTop || (SEARCH && r <= ldexpf((float)Cend, ue)));
      if (walk) {
#pragma unroll
        for (int j = 0; j < kPerThread; ++j) {
          const int li = tid * kPerThread + j;
          if (li < pos || li >= n || my_cross != INT_MAX || my_found != INT_MAX) continue;
          const int Cn = apply(em[j], C);
          if (Cn >= kTop) { my_cross = li; continue; }
          C = Cn;
          if (SEARCH && r <= ldexpf((float)C, ue)) my_found = li;
        }
      } else if (C < kTop) {
        C = Cend;
      }
      if (my_cross != INT_MAX) atomicMin(&sh.cross, my_cross);
      if (my_found != INT_MAX) atomicMin(&sh.found, my_found);
      __syncthreads();
      const int cross = sh.cross, found = sh.found;
      if (SEARCH && found < cross) { result = base + found; break; }
      if (cross == INT_MAX) {
        // chunk finished: the owner of the last element publishes the sum
        if (tid == (n - 1) / kPerThread) {
          sh.c = ldexpf((float)C, ue);
          sh.pos = n;
        }
        __syncthreads();
        break;
      }
      // element `cross` leaves the grid: apply it directly in fp32
      if (tid == cross / kPerThread) {
        int Cp = apply(pre, C0);
#pragma unroll
        for (int j = 0; j < kPerThread; ++j) {
          const int li = tid * kPerThread + j;
          if (li >= pos && li < cross) Cp = apply(em[j], Cp);
        }
        const float cprev = ldexpf((float)Cp, ue);  // exact: Cp < 2^24 on the 2^ue grid
        float vx = 0.0f;
#pragma unroll
        for (int j = 0; j < kPerThread; ++j)
          if (tid * kPerThread + j == cross) vx = v[j];
        const float cn = __fadd_rn(cprev, vx);
        sh.c = cn;
        sh.pos = cross + 1;
        sh.done = (SEARCH && r <= cn) ? 1 : (isnan(cn) || isinf(cn)) ? 2 : 0;
        sh.found = cross;
      }
      __syncthreads();
      if (sh.done == 1) { result = base + sh.found; break; }
      if (sh.done == 2) break;  // NaN / Inf: nothing later can match, the sum is final
    }
    if (result >= 0 || sh.done == 2) break;
    __syncthreads();
  }
  const float total = sh.c;
  __syncthreads();
  if (SEARCH) *hit = result;
  return total;
}

// The whole row from 0: SEARCH falls back to V-1 when r is never reached
// (speculative.cpp:23).
template <bool SEARCH, class F>
__device__ float exact_chain(F f, int64_t V, float r, int64_t *hit, ScanShared &sh) {
  int64_t h = -1;
  const float total = exact_chain_range<SEARCH>(f, 0, V, 0.0f, r, &h, sh);
  if (SEARCH) *hit = h >= 0 ? h : V - 1;
  return total;
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
__global__ void __launch_bounds__(kDecideThreads, 1)
decide_kernel(cf_accept_args a, float c, const RowStat *stats) {
  __shared__ ScanShared sh;
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
  auto p8 = [&](int64_t i0, float (&o)[8]) {
    load8<T>(xt, i0, V, o);
#pragma unroll
    for (int q = 0; q < 8; ++q) o[q] = prob_of(o[q], c, stt);
  };
  if (mode == kResidual) {
    // speculative.cpp:26-48
    const T *xd = row_ptr<T>(a.draft_logits, a.draft_seq_stride, a.draft_row_stride, b, row);
    const RowStat std_ = st[row];
    auto resid8 = [&](int64_t i0, float (&o)[8]) {
      float d8[8];
      load8<T>(xt, i0, V, o);
      load8<T>(xd, i0, V, d8);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float d = __fsub_rn(prob_of(o[q], c, stt), prob_of(d8[q], c, std_));
        o[q] = d > 0.0f ? d : 0.0f;  // std::max(0.0f, d)
      }
    };
    const float sum = exact_chain<false>(resid8, V, r, nullptr, sh);
    if (sum <= 1e-6f) {
      exact_chain<true>(p8, V, r, &tok, sh);
    } else {
      auto normed8 = [&](int64_t i0, float (&o)[8]) {
        resid8(i0, o);
#pragma unroll
        for (int q = 0; q < 8; ++q) o[q] = __fdiv_rn(o[q], sum);
      };
      exact_chain<true>(normed8, V, r, &tok, sh);
    }
  } else {
    exact_chain<true>(p8, V, r, &tok, sh);  // bonus, speculative.cpp:97
  }
  if (tid == 0) {
    out[s_na] = (int32_t)tok;
    a.out_num_accepted[b] = s_na;
    a.out_eos[b] = (tok == a.eos_token_id);
  }
}

// ---------------------------------------------------------------------------
// The stochastic draw across many CTAs.
//
// The single-CTA chain above walks a row chunk after chunk; here every row is
// cut into kNch chunks and the chunks are worked on by separate CTAs:
//   prep_kernel     grid (kNch, B): the K acceptance tests (every CTA of a
//                   sequence evaluates them; block 0 publishes the outcome)
//                   and, per chunk, approximate sums of the values the draw
//                   will accumulate (any order: they only predict);
//   maps_kernel     grid (kNch, B): per chunk, the composed increment map of
//                   the whole chunk on the ulp grid of the binade its start
//                   value is PREDICTED to lie in (from the approximate sums);
//   resolve_kernel  grid (B): walks the chunks with the exact running value:
//                   a chunk whose start really lies on the predicted grid and
//                   whose end stays inside that binade is applied in O(1)
//                   from its map; any other chunk (the first, those where a
//                   binade is crossed, a wrong prediction, NaN / Inf) and the
//                   chunk holding the search hit are scanned exactly.
// The running value is exact at every chunk boundary, so the result is the
// same bit for bit as the sequential loop.  Stage 0 is the residual mass (or
// directly the bonus draw), stage 1 the residual draw.
// ---------------------------------------------------------------------------
constexpr int kNch = 32;
constexpr int kChainThreads = 256;
constexpr int kNoMap = INT_MIN;
constexpr int kSerial = 512;  // the first elements of a row cross many binades: done serially

struct SeqState {
  int mode;    // -1 bad draft token, kDone, kResidual, kBonus
  int row;     // the row of the draw (rejected position, or K for the bonus)
  int na;      // accepted drafts
  float r;     // the draw's uniform
  float sum;   // stage 0 result: exact residual mass
  int vkind;   // stage 1 values: 1 = residual / sum, 2 = target row (mass <= 1e-6)
  uint32_t tp_key;  // nucleus (top-p) bonus draw: logits with order key >= tp_key are kept
  float tp_sum;     // ... and their probability mass (0: no nucleus filter)
};

struct ChunkInfo {
  float approx[2];  // approximate chunk sums: [0] stage-0 values, [1] target probabilities (residual mode)
  int ue, me, mo;   // the chunk's composed map on the grid 2^ue (kNoMap: scan it)
  int pad[3];
};

__host__ __device__ inline size_t accept_stats_bytes(int64_t batch, int64_t k) {
  return ((size_t)batch * (2 * (size_t)k + 1) * sizeof(RowStat) + 255) & ~(size_t)255;
}

__device__ __forceinline__ void chunk_range(int64_t V, int j, int64_t &lo, int64_t &hi) {
  const int64_t cl = ((V + kNch - 1) / kNch + 7) & ~(int64_t)7;
  lo = (int64_t)j * cl;
  hi = lo + cl < V ? lo + cl : V;
}

// Fixed-order block sum (kChainThreads threads): warp butterflies, then warp
// results in warp order.
__device__ __forceinline__ float block_sum256(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.0f;
  if (threadIdx.x == 0)
    for (int i = 0; i < kChainThreads / 32; ++i) t += red[i];
  return t;  // valid in thread 0
}

// The values a chain accumulates, eight at a time, for sequence b:
//   kind 0: target probabilities of `row`
//   kind 1: residual max(0, p - q) of `row`
//   kind 2: residual / sum
// Order key of a float: unsigned comparison of keys = numeric comparison of values.
__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <typename T>
struct ChainVals {
  const T *xt, *xd;
  RowStat st_t, st_d;
  float c, sum;
  int64_t V;
  int kind;
  uint32_t tp_key;
  __device__ __forceinline__ void operator()(int64_t i0, float (&o)[8]) const {
    load8<T>(xt, i0, V, o);
    if (kind == 0) {
#pragma unroll
      for (int q = 0; q < 8; ++q) o[q] = prob_of(o[q], c, st_t);
      return;
    }
    if (kind == 3) {  // nucleus: kept probabilities / their mass, the rest 0
#pragma unroll
      for (int q = 0; q < 8; ++q) o[q] = order_key(o[q]) >= tp_key ? __fdiv_rn(prob_of(o[q], c, st_t), sum) : 0.0f;
      return;
    }
    float d8[8];
    load8<T>(xd, i0, V, d8);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float d = __fsub_rn(prob_of(o[q], c, st_t), prob_of(d8[q], c, st_d));
      o[q] = d > 0.0f ? d : 0.0f;  // std::max(0.0f, d)
      if (kind == 2) o[q] = __fdiv_rn(o[q], sum);
    }
  }
};

template <typename T>
__device__ __forceinline__ ChainVals<T> chain_vals(const cf_accept_args &a, float c, const RowStat *st, int b, int row,
                                                   int kind, float sum) {
  const int K = a.k;
  ChainVals<T> f;
  f.xt = row_ptr<T>(a.target_logits, a.target_seq_stride, a.target_row_stride, b, row);
  f.xd = kind == 0 ? f.xt : row_ptr<T>(a.draft_logits, a.draft_seq_stride, a.draft_row_stride, b, row);
  f.st_t = st[K + row];
  f.st_d = kind == 0 ? f.st_t : st[row];
  f.c = c;
  f.sum = sum;
  f.V = a.vocab;
  f.kind = kind;
  f.tp_key = 0;
  return f;
}

// The chain values of sequence state sq for value kind `kind`.
template <typename T>
__device__ __forceinline__ ChainVals<T> chain_vals_of(const cf_accept_args &a, float c, const RowStat *st, int b,
                                                      const SeqState &sq, int kind) {
  ChainVals<T> f = chain_vals<T>(a, c, st, b, sq.row, kind == 3 ? 0 : kind, kind == 3 ? sq.tp_sum : sq.sum);
  if (kind == 3) {
    f.kind = 3;
    f.tp_key = sq.tp_key;
  }
  return f;
}

template <typename T>
__global__ void __launch_bounds__(kChainThreads)
prep_kernel(cf_accept_args a, float c, const RowStat *stats, SeqState *seq, ChunkInfo *ci) {
  __shared__ float s_ratio[64];
  __shared__ int s_mode, s_row, s_na;
  __shared__ float s_r, red[kChainThreads / 32];
  const int j = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int K = a.k;
  const int64_t V = a.vocab;
  const RowStat *st = stats + (int64_t)b * (2 * K + 1);
  const int32_t *dt = a.draft_tokens + (int64_t)b * K;
  auto ratio_of = [&](int i) -> float {  // speculative.cpp:69-74; NaN marks a bad draft token
    const int32_t tok = dt[i];
    if (tok < 0 || tok >= V) return __int_as_float(0x7fffffff);
    const T *xd = row_ptr<T>(a.draft_logits, a.draft_seq_stride, a.draft_row_stride, b, i);
    const T *xt = row_ptr<T>(a.target_logits, a.target_seq_stride, a.target_row_stride, b, i);
    const float q = prob_of(cf::to_float(xd[tok]), c, st[i]);
    const float p = prob_of(cf::to_float(xt[tok]), c, st[K + i]);
    const float pq = __fdiv_rn(p, q);
    return (q > 0.0f) ? ((pq < 1.0f) ? pq : 1.0f) : 0.0f;
  };
  for (int i = tid; i < K && i < 64; i += kChainThreads) s_ratio[i] = ratio_of(i);
  __syncthreads();
  if (tid == 0) {
    // speculative.cpp:66-101: the tests in order, one uniform each
    const float *u = a.uniforms + (int64_t)b * (K + 1);
    int32_t *out = a.out_tokens + (int64_t)b * (K + 1);
    int na = 0, used = 0, mode = kBonus, row = K;
    for (int i = 0; i < K; ++i) {
      const float ratio = i < 64 ? s_ratio[i] : ratio_of(i);
      if (isnan(ratio)) { mode = -1; break; }
      const float r = u[used++];
      if (r <= ratio) {
        const int32_t tok = dt[i];
        if (j == 0) out[na] = tok;
        ++na;
        if (tok == a.eos_token_id) { mode = kDone; break; }
      } else {
        mode = kResidual;
        row = i;
        break;
      }
    }
    s_mode = mode;
    s_row = row;
    s_na = na;
    s_r = (mode == kDone || mode < 0) ? 0.0f : u[used];
    if (j == 0) {
      SeqState sq{};
      sq.mode = mode; sq.row = row; sq.na = na; sq.r = s_r; sq.sum = 0.0f; sq.vkind = 0;
      sq.tp_key = 0; sq.tp_sum = 0.0f;
      seq[b] = sq;
      if (mode < 0) { a.out_num_accepted[b] = -1; a.out_eos[b] = 0; }
      if (mode == kDone) { out[na] = a.eos_token_id; a.out_num_accepted[b] = na; a.out_eos[b] = 1; }
    }
  }
  __syncthreads();
  const int mode = s_mode;
  if (mode == kDone || mode < 0) return;
  int64_t lo, hi;
  chunk_range(V, j, lo, hi);
  const ChainVals<T> f = chain_vals<T>(a, c, st, b, s_row, mode == kResidual ? 1 : 0, 0.0f);
  const ChainVals<T> fp = chain_vals<T>(a, c, st, b, s_row, 0, 0.0f);
  float s0 = 0.0f, s1 = 0.0f;
  for (int64_t i0 = lo + (int64_t)tid * 8; i0 < hi; i0 += (int64_t)kChainThreads * 8) {
    float v[8];
    f(i0, v);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (i0 + q < hi) s0 += v[q];
    if (mode == kResidual) {
      fp(i0, v);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (i0 + q < hi) s1 += v[q];
    }
  }
  s0 = block_sum256(s0, red);
  s1 = block_sum256(s1, red);
  if (tid == 0) {
    ci[(int64_t)b * kNch + j].approx[0] = s0;
    ci[(int64_t)b * kNch + j].approx[1] = s1;
  }
}

// The chain a sequence runs in stage STAGE: kind of values (-1: none) and
// whether it searches.
__device__ __forceinline__ int chain_kind(const SeqState &sq, int stage, bool &search) {
  search = true;
  if (stage == 0) {
    if (sq.mode == kBonus) return sq.tp_sum > 0.0f ? 3 : 0;
    if (sq.mode == kResidual) { search = false; return 1; }
    return -1;
  }
  if (sq.mode != kResidual) return -1;
  return sq.vkind == 2 ? 0 : 2;
}

template <typename T, int STAGE>
__global__ void __launch_bounds__(kChainThreads)
maps_kernel(cf_accept_args a, float c, const RowStat *stats, const SeqState *seq, ChunkInfo *ci) {
  __shared__ int s_ue;
  __shared__ IncMap s_w[kChainThreads / 32];
  const int j = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const SeqState sq = seq[b];
  bool search;
  const int kind = chain_kind(sq, STAGE, search);
  if (kind < 0) return;
  ChunkInfo *info = ci + (int64_t)b * kNch;
  if (j == 0) {  // a row's first chunk always starts at 0 and is scanned
    if (tid == 0) info[0].ue = kNoMap;
    return;
  }
  const int64_t V = a.vocab;
  int64_t lo, hi;
  chunk_range(V, j, lo, hi);
  if (lo >= hi) return;
  if (tid == 0) {
    // predicted start value: approximate sums of the chunks before this one
    const int idx = (STAGE == 1 && kind == 0) ? 1 : 0;
    float pre = 0.0f;
    for (int i = 0; i < j; ++i) pre += info[i].approx[idx];
    if (STAGE == 1 && kind == 2) pre = pre / sq.sum;
    int C;
    grid_of(pre, C, s_ue);
  }
  __syncthreads();
  const int ue = s_ue;
  const RowStat *st = stats + (int64_t)b * (2 * a.k + 1);
  const ChainVals<T> f = chain_vals_of<T>(a, c, st, b, sq, kind);
  // thread t owns the contiguous elements [lo + t*per, lo + (t+1)*per): maps compose in thread order
  const int64_t per = ((hi - lo + kChainThreads - 1) / kChainThreads + 7) & ~(int64_t)7;
  IncMap m{0, 0};
  for (int64_t i0 = lo + tid * per; i0 < lo + (tid + 1) * per && i0 < hi; i0 += 8) {
    float v[8];
    f(i0, v);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (i0 + q < hi) m = compose(m, elem_map(v[q], ue));
  }
  // in-order composition across the warp (lane l holds [l, l + 2o) after step o), then across warps
  const int lane = tid & 31, w = tid >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    IncMap y;
    y.e = __shfl_down_sync(0xffffffffu, m.e, o);
    y.o = __shfl_down_sync(0xffffffffu, m.o, o);
    if ((lane & (2 * o - 1)) == 0 && lane + o < 32) m = compose(m, y);
  }
  if (lane == 0) s_w[w] = m;
  __syncthreads();
  if (tid == 0) {
    IncMap t{0, 0};
    for (int i = 0; i < kChainThreads / 32; ++i) t = compose(t, s_w[i]);
    info[j].ue = ue;
    info[j].me = t.e;
    info[j].mo = t.o;
  }
}

// Nucleus (top-p) filter of the bonus draw, one CTA per sequence in bonus
// mode.  The reference (speculative.py:58-84) sorts the row, keeps every token
// whose exclusive cumulative probability in descending order is <= top_p
// (the token that crosses top_p included) and renormalises.  Here a token x is
// kept when the probability mass of the logits strictly above it is <= top_p;
// for distinct logits that is the same set, and tied logits are kept or
// dropped together (independent of sort stability).  The kept set is
// {order_key(x) >= k*}, k* the smallest key whose strictly-greater mass is
// <= top_p, found by bisection over the 32-bit keys with fixed-order sums; the
// approximate chunk sums of the renormalised values then predict the maps.
template <typename T>
__global__ void __launch_bounds__(kScanThreads, 1)
nucleus_kernel(cf_accept_args a, float c, const RowStat *stats, SeqState *seq, ChunkInfo *ci) {
  __shared__ float red[kScanThreads / 32];
  __shared__ float s_tot;
  const int b = blockIdx.x, tid = threadIdx.x;
  SeqState sq = seq[b];
  if (sq.mode != kBonus) return;
  const int64_t V = a.vocab;
  const RowStat *st = stats + (int64_t)b * (2 * a.k + 1);
  const T *x = row_ptr<T>(a.target_logits, a.target_seq_stride, a.target_row_stride, b, sq.row);
  const RowStat stt = st[a.k + sq.row];
  // fixed-order mass of the logits whose key is > kgt (strict) or >= kge
  auto mass = [&](uint32_t k, bool strict) -> float {
    float m = 0.0f;
    for (int64_t i0 = (int64_t)tid * 8; i0 < V; i0 += (int64_t)kScanThreads * 8) {
      float v[8];
      load8<T>(x, i0, V, v);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t kk = order_key(v[q]);
        if (i0 + q < V && (strict ? kk > k : kk >= k)) m += prob_of(v[q], c, stt);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m += __shfl_xor_sync(0xffffffffu, m, o);
    __syncthreads();
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    if (tid == 0) {
      float t = 0.0f;
      for (int i = 0; i < kScanThreads / 32; ++i) t += red[i];
      s_tot = t;
    }
    __syncthreads();
    return s_tot;
  };
  // smallest k with mass(> k) <= top_p: the predicate is monotone in k
  uint32_t lo = 0, hi = 0xffffffffu;
  if (mass(0u, true) <= a.top_p) hi = 0u;
  while (lo + 1 < hi) {
    const uint32_t mid = lo + (hi - lo) / 2;
    if (mass(mid, true) <= a.top_p) hi = mid;
    else lo = mid;
  }
  const float kept = mass(hi, false);
  int64_t lo_c, hi_c;
  if (tid == 0) {
    sq.tp_key = hi;
    sq.tp_sum = kept > 0.0f ? kept : 1.0f;
    seq[b] = sq;
  }
  // approximate chunk sums of the renormalised kept values (they predict the maps' grids)
  const float inv = 1.0f / (kept > 0.0f ? kept : 1.0f);
  for (int j = 0; j < kNch; ++j) {
    chunk_range(V, j, lo_c, hi_c);
    float m = 0.0f;
    for (int64_t i0 = lo_c + (int64_t)tid * 8; i0 < hi_c; i0 += (int64_t)kScanThreads * 8) {
      float v[8];
      load8<T>(x, i0, V, v);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (i0 + q < hi_c && order_key(v[q]) >= hi) m += prob_of(v[q], c, stt) * inv;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m += __shfl_xor_sync(0xffffffffu, m, o);
    __syncthreads();
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    if (tid == 0) {
      float t = 0.0f;
      for (int i = 0; i < kScanThreads / 32; ++i) t += red[i];
      ci[(int64_t)b * kNch + j].approx[0] = t;
    }
  }
}

template <typename T, int STAGE>
__global__ void __launch_bounds__(kScanThreads, 1)
resolve_kernel(cf_accept_args a, float c, const RowStat *stats, SeqState *seq, const ChunkInfo *ci) {
  __shared__ ScanShared sh;
  __shared__ int s_ue[kNch], s_me[kNch], s_mo[kNch];
  __shared__ __align__(16) float s_buf[kSerial];
  __shared__ float s_cum;
  __shared__ long long s_hit;
  const int b = blockIdx.x, tid = threadIdx.x;
  const SeqState sq = seq[b];
  bool search;
  const int kind = chain_kind(sq, STAGE, search);
  if (kind < 0) return;
  const int64_t V = a.vocab;
  const RowStat *st = stats + (int64_t)b * (2 * a.k + 1);
  const ChainVals<T> f = chain_vals_of<T>(a, c, st, b, sq, kind);
  for (int i = tid; i < kNch; i += kScanThreads) {
    s_ue[i] = ci[(int64_t)b * kNch + i].ue;
    s_me[i] = ci[(int64_t)b * kNch + i].me;
    s_mo[i] = ci[(int64_t)b * kNch + i].mo;
  }
  const float r = search ? sq.r : 0.0f;
  // the first kSerial elements: one thread, the reference's loop itself
  const int64_t n0 = V < kSerial ? V : kSerial;
  for (int64_t i0 = (int64_t)tid * 8; i0 < n0; i0 += (int64_t)kScanThreads * 8) {
    float v[8];
    f(i0, v);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (i0 + q < n0) s_buf[i0 + q] = v[q];
  }
  __syncthreads();
  if (tid == 0) {
    float cum = 0.0f;
    long long hit = -1;
    // eight values per pair of 16-byte shared loads, so the dependent adds do not wait on each load
    for (int i = 0; i < n0 && hit < 0; i += 8) {
      const float4 x = reinterpret_cast<const float4 *>(s_buf)[i / 4];
      const float4 y = reinterpret_cast<const float4 *>(s_buf)[i / 4 + 1];
      const float v[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (i + q < n0 && hit < 0) {
          cum = __fadd_rn(cum, v[q]);
          if (search && r <= cum) hit = i + q;
        }
      }
    }
    s_cum = cum;
    s_hit = hit;
  }
  __syncthreads();
  float cum = s_cum;
  int64_t hit = s_hit;
  for (int j = 0; j < kNch && hit < 0 && isfinite(cum); ++j) {
    int64_t lo, hi;
    chunk_range(V, j, lo, hi);
    if (lo >= V) break;
    const bool whole = lo >= n0;  // the chunk's map covers it only if the serial prefix did not
    if (!whole) lo = n0;
    if (lo >= hi) continue;
    bool fast = false;
    float end = 0.0f;
    if (whole && s_ue[j] != kNoMap) {
      int C, ue;
      grid_of(cum, C, ue);
      if (ue == s_ue[j]) {
        const int Ce = apply(IncMap{s_me[j], s_mo[j]}, C);
        if (Ce < kTop) { fast = true; end = ldexpf((float)Ce, ue); }
      }
    }
    if (fast && !(search && r <= end)) { cum = end; continue; }
    // scan the chunk exactly from its exact start value (and find the hit, searching)
    int64_t h = -1;
    if (search) cum = exact_chain_range<true>(f, lo, hi, cum, r, &h, sh);
    else cum = exact_chain_range<false>(f, lo, hi, cum, r, nullptr, sh);
    hit = h;
  }
  if (tid != 0) return;
  if (!search) {  // residual mass: speculative.cpp:34-41
    SeqState o = sq;
    o.sum = cum;
    o.vkind = (cum <= 1e-6f) ? 2 : 1;
    seq[b] = o;
    return;
  }
  const int64_t tok = hit >= 0 ? hit : V - 1;
  a.out_tokens[(int64_t)b * (a.k + 1) + sq.na] = (int32_t)tok;
  a.out_num_accepted[b] = sq.na;
  a.out_eos[b] = (tok == a.eos_token_id);
}

// ---------------------------------------------------------------------------
// Tree acceptance (no reference counterpart; a branching-1 tree reduces
// exactly to the chain rule above).  Nodes 0..N, node 0 the root, parent[i] <
// i, siblings tested in increasing node index.  Rows 0..N of the stats are
// the draft rows (distribution each node's children were drawn from), rows
// N+1..2N+1 the target rows.  The current distribution p is either a target
// row (through its stats) or, after a rejected sibling, the normalised
// residual held in this sequence's fp32 workspace row `resid`.
// ---------------------------------------------------------------------------
struct TreeArgs {
  cf_accept_args a;  // batch, vocab, dtype, logits (row u = node u), uniforms, temperature, eos, greedy
  int nodes;         // N + 1
  const int32_t *parent, *tokens;
  int32_t *out_path;
  float *resid;      // [B][V]
};

template <typename T>
__global__ void __launch_bounds__(kDecideThreads, 1)
decide_tree_kernel(TreeArgs ta, float c, const RowStat *stats) {
  __shared__ ScanShared sh;
  __shared__ int s_cur, s_moved, s_any, s_used, s_resid, s_done, s_na;
  __shared__ float s_r;
  const cf_accept_args &a = ta.a;
  const int b = blockIdx.x, tid = threadIdx.x;
  const int NN = ta.nodes;
  const int64_t V = a.vocab;
  const RowStat *st = stats + (int64_t)b * 2 * NN;
  const int32_t *par = ta.parent + (int64_t)b * NN;
  const int32_t *tk = ta.tokens + (int64_t)b * NN;
  const float *u = a.uniforms + (int64_t)b * NN;
  int32_t *outt = a.out_tokens + (int64_t)b * NN;
  int32_t *outp = ta.out_path + (int64_t)b * NN;
  float *R = ta.resid + (int64_t)b * V;
  if (tid == 0) { s_cur = 0; s_used = 0; s_resid = 0; s_done = 0; s_na = 0; outp[0] = 0; }
  __syncthreads();
  while (true) {
    const int cur = s_cur;
    const T *xt = row_ptr<T>(a.target_logits, a.target_seq_stride, a.target_row_stride, b, cur);
    const RowStat stt = st[NN + cur];
    if (a.greedy) {
      const int64_t am = block_argmax<T>(xt, V, c, stt);
      if (tid == 0) {
        int moved = -1;
        for (int ch = cur + 1; ch < NN; ++ch)
          if (par[ch] == cur && tk[ch] == am) { moved = ch; break; }
        if (moved < 0) {
          outt[s_na] = (int32_t)am; a.out_num_accepted[b] = s_na; a.out_eos[b] = (am == a.eos_token_id); s_done = 1;
        } else {
          outp[++s_na] = moved; outt[s_na - 1] = tk[moved]; s_cur = moved;
          if (tk[moved] == a.eos_token_id) { outt[s_na] = tk[moved]; a.out_num_accepted[b] = s_na; a.out_eos[b] = 1; s_done = 1; }
        }
      }
      __syncthreads();
      if (s_done) return;
      continue;
    }
    const T *xd = row_ptr<T>(a.draft_logits, a.draft_seq_stride, a.draft_row_stride, b, cur);
    const RowStat sdr = st[cur];
    if (tid == 0) { s_moved = -1; s_any = 0; s_resid = 0; }
    __syncthreads();
    for (int ch = cur + 1; ch < NN; ++ch) {
      if (par[ch] != cur) continue;  // uniform across the block
      if (tid == 0) {
        s_any = 1;
        const int32_t x = tk[ch];
        if (x < 0 || x >= V) { a.out_num_accepted[b] = -1; a.out_eos[b] = 0; s_done = 1; }
        else {
          const float qx = prob_of(cf::to_float(xd[x]), c, sdr);
          const float px = s_resid ? R[x] : prob_of(cf::to_float(xt[x]), c, stt);
          const float pq = __fdiv_rn(px, qx);
          const float ratio = (qx > 0.0f) ? ((pq < 1.0f) ? pq : 1.0f) : 0.0f;
          const float r = u[s_used++];
          if (r <= ratio) s_moved = ch;
        }
      }
      __syncthreads();
      if (s_done) return;
      if (s_moved >= 0) break;
      // rejected: p <- norm(max(0, p - q)) unless that sum is <= 1e-6
      const bool from_r = s_resid;
      auto d8 = [&](int64_t i0, float (&o)[8]) {
        float q8[8];
        if (from_r) load8<float>(R, i0, V, o);
        else {
          load8<T>(xt, i0, V, o);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = prob_of(o[j], c, stt);
        }
        load8<T>(xd, i0, V, q8);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float d = __fsub_rn(o[j], prob_of(q8[j], c, sdr));
          o[j] = d > 0.0f ? d : 0.0f;
        }
      };
      const float sum = exact_chain<false>(d8, V, 0.0f, nullptr, sh);
      if (sum > 1e-6f) {
        for (int64_t i0 = (int64_t)tid * 8; i0 < V; i0 += (int64_t)kDecideThreads * 8) {
          float o[8];
          d8(i0, o);  // reads the old R (if any) for exactly these elements before they are overwritten
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (i0 + j < V) R[i0 + j] = __fdiv_rn(o[j], sum);
        }
        __syncthreads();
        if (tid == 0) s_resid = 1;
        __syncthreads();
      }
    }
    const int moved = s_moved;
    if (moved >= 0) {
      if (tid == 0) {
        outp[++s_na] = moved;
        outt[s_na - 1] = tk[moved];
        s_cur = moved;
        if (tk[moved] == a.eos_token_id) {
          outt[s_na] = tk[moved]; a.out_num_accepted[b] = s_na; a.out_eos[b] = 1; s_done = 1;
        }
      }
      __syncthreads();
      if (s_done) return;
      continue;
    }
    // all children rejected (draw from the current p) or a leaf (bonus from its target row)
    if (tid == 0) s_r = u[s_used++];
    __syncthreads();
    const float r = s_r;
    int64_t tok;
    if (s_any && s_resid) {
      auto r8 = [&](int64_t i0, float (&o)[8]) { load8<float>(R, i0, V, o); };
      exact_chain<true>(r8, V, r, &tok, sh);
    } else {
      auto p8 = [&](int64_t i0, float (&o)[8]) {
        load8<T>(xt, i0, V, o);
#pragma unroll
        for (int q = 0; q < 8; ++q) o[q] = prob_of(o[q], c, stt);
      };
      exact_chain<true>(p8, V, r, &tok, sh);
    }
    if (tid == 0) {
      outt[s_na] = (int32_t)tok;
      a.out_num_accepted[b] = s_na;
      a.out_eos[b] = (tok == a.eos_token_id);
    }
    return;
  }
}

template <typename T>
int launch_accept_tree(const TreeArgs &ta, cudaStream_t stream) {
  const cf_accept_args &a = ta.a;
  const float c = (float)(1.4426950408889634 / (double)a.temperature);
  RowStat *stats = reinterpret_cast<RowStat *>(a.workspace);
  dim3 g1(2 * ta.nodes, a.batch);
  row_stats_kernel<T><<<g1, kStatsThreads, 0, stream>>>(a, c, stats, ta.nodes, ta.nodes);
  if (a.probs_draft || a.probs_target)
    export_probs_kernel<T><<<g1, 256, 0, stream>>>(a, c, stats, ta.nodes, ta.nodes);
  decide_tree_kernel<T><<<a.batch, kDecideThreads, 0, stream>>>(ta, c, stats);
  return cf_launch_status();
}

template <typename T>
int launch_accept(const cf_accept_args &a, cudaStream_t stream) {
  const float c = (float)(1.4426950408889634 / (double)a.temperature);
  RowStat *stats = reinterpret_cast<RowStat *>(a.workspace);
  dim3 g1(2 * a.k + 1, a.batch);
  row_stats_kernel<T><<<g1, kStatsThreads, 0, stream>>>(a, c, stats, a.k, a.k + 1);
  if (a.probs_draft || a.probs_target) export_probs_kernel<T><<<g1, 256, 0, stream>>>(a, c, stats, a.k, a.k + 1);
  if (a.greedy) {
    decide_kernel<T><<<a.batch, kDecideThreads, 0, stream>>>(a, c, stats);
    return cf_launch_status();
  }
  uint8_t *base = reinterpret_cast<uint8_t *>(a.workspace) + accept_stats_bytes(a.batch, a.k);
  SeqState *seq = reinterpret_cast<SeqState *>(base);
  ChunkInfo *ci = reinterpret_cast<ChunkInfo *>(base + (size_t)a.batch * sizeof(SeqState));
  const dim3 gc(kNch, a.batch);
  prep_kernel<T><<<gc, kChainThreads, 0, stream>>>(a, c, stats, seq, ci);
  if (a.top_p > 0.0f && a.top_p < 1.0f) nucleus_kernel<T><<<a.batch, kScanThreads, 0, stream>>>(a, c, stats, seq, ci);
  maps_kernel<T, 0><<<gc, kChainThreads, 0, stream>>>(a, c, stats, seq, ci);
  resolve_kernel<T, 0><<<a.batch, kScanThreads, 0, stream>>>(a, c, stats, seq, ci);
  maps_kernel<T, 1><<<gc, kChainThreads, 0, stream>>>(a, c, stats, seq, ci);
  resolve_kernel<T, 1><<<a.batch, kScanThreads, 0, stream>>>(a, c, stats, seq, ci);
  return cf_launch_status();
}

}  // namespace

static size_t tree_stats_bytes(int32_t batch, int32_t nodes) {
  return ((size_t)batch * 2 * (size_t)nodes * sizeof(RowStat) + 255) & ~(size_t)255;
}

extern "C" size_t cf_accept_tree_workspace_bytes(int32_t batch, int32_t nodes, int64_t vocab) {
  if (batch < 0 || nodes < 1 || vocab < 1) return 0;
  return tree_stats_bytes(batch, nodes) + (size_t)batch * (size_t)vocab * sizeof(float);
}

extern "C" int cf_accept_tree(const cf_accept_tree_args *t, void *stream) {
  if (!t) return CF_EINVAL;
  cf_accept_args a{};
  a.batch = t->batch;
  a.k = 0;
  a.vocab = t->vocab;
  a.logits_dtype = t->logits_dtype;
  a.draft_logits = t->draft_logits;
  a.draft_seq_stride = t->draft_seq_stride;
  a.draft_row_stride = t->draft_row_stride;
  a.target_logits = t->target_logits;
  a.target_seq_stride = t->target_seq_stride;
  a.target_row_stride = t->target_row_stride;
  a.uniforms = t->uniforms;
  a.temperature = t->temperature;
  a.eos_token_id = t->eos_token_id;
  a.greedy = t->greedy;
  a.out_tokens = t->out_tokens;
  a.out_num_accepted = t->out_num_accepted;
  a.out_eos = t->out_eos;
  a.workspace = t->workspace;
  a.probs_draft = t->probs_draft;
  a.probs_target = t->probs_target;
  if (a.batch < 0 || t->nodes < 1 || a.vocab < 1 || a.vocab > INT32_MAX || t->nodes > 65535 / 2) return CF_EINVAL;
  if (a.batch == 0) return CF_OK;
  if (!(a.temperature > 0.0f) || !isfinite(a.temperature)) return CF_EINVAL;
  if (!a.target_logits || !t->parent || !t->tokens || !t->out_path || !a.out_tokens || !a.out_num_accepted ||
      !a.out_eos || !a.workspace)
    return CF_EINVAL;
  if (!a.greedy && (!a.uniforms || !a.draft_logits)) return CF_EINVAL;
  if ((reinterpret_cast<uintptr_t>(a.workspace) & 255) != 0 || a.batch > 65535) return CF_EINVAL;
  if (a.target_row_stride < a.vocab || (a.draft_logits && a.draft_row_stride < a.vocab)) return CF_EINVAL;
  TreeArgs ta;
  ta.a = a;
  ta.nodes = t->nodes;
  ta.parent = t->parent;
  ta.tokens = t->tokens;
  ta.out_path = t->out_path;
  ta.resid = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(a.workspace) + tree_stats_bytes(a.batch, t->nodes));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (a.logits_dtype) {
    case CF_F32: return launch_accept_tree<float>(ta, s);
    case CF_BF16: return launch_accept_tree<__nv_bfloat16>(ta, s);
    case CF_F16: return launch_accept_tree<__half>(ta, s);
    default: return CF_EINVAL;
  }
}

extern "C" size_t cf_accept_workspace_bytes(int32_t batch, int32_t k) {
  if (batch < 0 || k < 0) return 0;
  return accept_stats_bytes(batch, k) + (size_t)batch * (sizeof(SeqState) + kNch * sizeof(ChunkInfo));
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

// ---------------------------------------------------------------------------
// Allocation-free variant.  Some callers cannot allocate device memory at
// all: code running where cudaMalloc is off limits (an allocator hook, a
// host runtime that owns every byte of device memory, a plugin that may only
// touch the buffers it is handed).  For them the acceptance scratch (row
// statistics, per-sequence state, per-chunk maps) lives in a fixed 2 MiB
// array inside this library instead of a caller workspace, on every GPU that
// loads the library, held until the process exits.
// ---------------------------------------------------------------------------
namespace {
constexpr size_t kAcceptScratchBytes = size_t(2) << 20;  // cf_accept_workspace_bytes(batch, k) must fit
static __device__ __align__(256) uint8_t g_accept_scratch[kAcceptScratchBytes];

constexpr int kMaxDevices = 64;
void *g_scratch_ptr[kMaxDevices];
std::mutex g_scratch_mu;

// Device address of g_accept_scratch on the current device (looked up once
// per device; the host-side symbol itself is not a device address).
int scratch_ptr(void **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CF_ECUDA;
  std::lock_guard<std::mutex> g(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_accept_scratch) != cudaSuccess || !p) return CF_ECUDA;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return CF_OK;
}
}  // namespace

extern "C" int cf_accept_sample_noalloc(const cf_accept_args *args, void *stream) {
  if (!args) return CF_EINVAL;
  if (args->batch < 0 || args->k < 0) return CF_EINVAL;
  if (cf_accept_workspace_bytes(args->batch, args->k) > kAcceptScratchBytes) return CF_ERANGE;
  void *ws = nullptr;
  const int rc = scratch_ptr(&ws);
  if (rc != CF_OK) return rc;
  cf_accept_args a = *args;
  // every scratch word a call reads was written earlier in that same call: nothing to clear
  a.workspace = ws;
  return cf_accept_sample(&a, stream);
}

extern "C" size_t cf_accept_noalloc_max_bytes(void) { return kAcceptScratchBytes; }
