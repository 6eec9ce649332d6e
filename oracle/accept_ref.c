/*
 * TEST INFRASTRUCTURE ONLY -- CPU oracle for speculative acceptance.
 *
 * This file restates the reference's native acceptance algorithm so the tests
 * can check the CUDA kernels bit-for-bit.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / reference arm may load it; the product path
 * never does.
 *
 * Reference: csrc/src/scheduler/speculative.cpp (CUDAForge)
 *   sample_from_distribution       :12-24
 *   sample_adjusted_distribution   :26-48
 *   verify_candidates              :50-103
 *   verify_candidates_greedy       :105-150
 *
 * The only change of form: the reference draws its uniforms from a private
 * std::mt19937; here they are an explicit argument `u[K+1]`, consumed in the
 * same order (acceptance test i uses u[i]; the single draw of the final
 * sample uses u[n_tests], where n_tests = j+1 after a rejection at j, or K
 * after full acceptance; an accepted EOS draws nothing more).  The pinning
 * test replays the reference's own mt19937 stream through this contract and
 * requires identical results from the unmodified reference code.
 *
 * All arithmetic is IEEE fp32 in the reference's order (sequential sums, one
 * rounding per operation); build without -ffast-math and without FMA
 * contraction (-ffp-contract=off).
 */
#include <stdint.h>
#include <stddef.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* speculative.cpp:12-24: inverse CDF by a sequential fp32 cumulative sum,
 * first index with r <= cum, falling back to the last index. */
static int32_t sample_from(const float *probs, int64_t V, float r) {
  float cum = 0.0f;
  for (int64_t i = 0; i < V; ++i) {
    cum += probs[i];
    if (r <= cum) return (int32_t)i;
  }
  return (int32_t)(V - 1);
}

/* speculative.cpp:26-48: residual max(0, p - q), sequential fp32 sum, fallback
 * to the target when the sum is <= 1e-6, else normalise element-wise and
 * sample. */
static int32_t sample_adjusted(const float *p, const float *q, int64_t V,
                               float r, float *work) {
  float sum = 0.0f;
  for (int64_t i = 0; i < V; ++i) {
    float d = p[i] - q[i];
    work[i] = d > 0.0f ? d : 0.0f;
    sum += work[i];
  }
  if (sum <= 1e-6f) return sample_from(p, V, r);
  for (int64_t i = 0; i < V; ++i) work[i] /= sum;
  return sample_from(work, V, r);
}

/* Result layout shared with the CUDA path: tokens[0..num_accepted-1] are the
 * accepted drafts, tokens[num_accepted] the final (resampled / bonus / EOS)
 * token. */
int oref_accept_one(int32_t K, int64_t V, const int32_t *draft_tokens,
                    const float *draft_probs,  /* [K][V]   */
                    const float *target_probs, /* [K+1][V] */
                    int32_t eos, const float *u, int32_t *tokens,
                    int32_t *num_accepted, uint8_t *eos_flag,
                    int32_t *n_uniforms_used) {
  float *work = (float *)malloc(sizeof(float) * (size_t)(V > 0 ? V : 1));
  if (!work) return -1;
  int32_t na = 0;
  uint8_t e = 0;
  int32_t used = 0;
  int32_t final_tok;
  int done = 0;
  for (int32_t i = 0; i < K && !done; ++i) {
    int32_t c = draft_tokens[i];
    float q = draft_probs[(size_t)i * V + c];
    float p = target_probs[(size_t)i * V + c];
    float pq = p / q;
    /* std::min(1.0f, p / q) == (p/q < 1) ? p/q : 1 (NaN -> 1) */
    float ratio = (q > 0.0f) ? ((pq < 1.0f) ? pq : 1.0f) : 0.0f; /* :71 */
    float r = u[used++];
    if (r <= ratio) { /* :74 */
      tokens[na++] = c;
      if (c == eos) { /* :79-83 */
        e = 1;
        final_tok = eos;
        done = 1;
      }
    } else { /* :84-92 */
      final_tok = sample_adjusted(target_probs + (size_t)i * V,
                                  draft_probs + (size_t)i * V, V, u[used++],
                                  work);
      if (final_tok == eos) e = 1;
      done = 1;
    }
  }
  if (!done) { /* :96-101 bonus */
    final_tok = sample_from(target_probs + (size_t)K * V, V, u[used++]);
    if (final_tok == eos) e = 1;
  }
  tokens[na] = final_tok;
  *num_accepted = na;
  *eos_flag = e;
  if (n_uniforms_used) *n_uniforms_used = used;
  free(work);
  return 0;
}

/* std::max_element: first index of the largest value. */
static int32_t argmax_first(const float *x, int64_t V) {
  int64_t best = 0;
  for (int64_t i = 1; i < V; ++i)
    if (x[best] < x[i]) best = i;
  return (int32_t)best;
}

/* speculative.cpp:105-150 */
int oref_accept_greedy_one(int32_t K, int64_t V, const int32_t *draft_tokens,
                           const float *target_probs, int32_t eos,
                           int32_t *tokens, int32_t *num_accepted,
                           uint8_t *eos_flag) {
  int32_t na = 0;
  uint8_t e = 0;
  for (int32_t i = 0; i < K; ++i) {
    int32_t c = draft_tokens[i];
    int32_t am = argmax_first(target_probs + (size_t)i * V, V);
    if (c == am) {
      tokens[na++] = c;
      if (c == eos) {
        tokens[na] = eos;
        *num_accepted = na;
        *eos_flag = 1;
        return 0;
      }
    } else {
      tokens[na] = am;
      *num_accepted = na;
      *eos_flag = (am == eos);
      return 0;
    }
  }
  int32_t b = argmax_first(target_probs + (size_t)K * V, V);
  tokens[na] = b;
  *num_accepted = na;
  *eos_flag = (b == eos);
  (void)e;
  return 0;
}

/* Batched front ends: rows of sequence b start at b*K*V (draft) and
 * b*(K+1)*V (target); tokens is [B][K+1]; u is [B][K+1]. */
int oref_accept_batch(int32_t B, int32_t K, int64_t V,
                      const int32_t *draft_tokens, const float *draft_probs,
                      const float *target_probs, int32_t eos, const float *u,
                      int32_t *tokens, int32_t *num_accepted,
                      uint8_t *eos_flag) {
  for (int32_t b = 0; b < B; ++b) {
    int rc = oref_accept_one(K, V, draft_tokens + (size_t)b * K,
                             draft_probs + (size_t)b * K * V,
                             target_probs + (size_t)b * (K + 1) * V, eos,
                             u + (size_t)b * (K + 1),
                             tokens + (size_t)b * (K + 1), num_accepted + b,
                             eos_flag + b, NULL);
    if (rc) return rc;
  }
  return 0;
}

int oref_accept_greedy_batch(int32_t B, int32_t K, int64_t V,
                             const int32_t *draft_tokens,
                             const float *target_probs, int32_t eos,
                             int32_t *tokens, int32_t *num_accepted,
                             uint8_t *eos_flag) {
  for (int32_t b = 0; b < B; ++b)
    oref_accept_greedy_one(K, V, draft_tokens + (size_t)b * K,
                           target_probs + (size_t)b * (K + 1) * V, eos,
                           tokens + (size_t)b * (K + 1), num_accepted + b,
                           eos_flag + b);
  return 0;
}

/* Temperature softmax of one row in a fixed, documented order:
 *   y_i = x_i / T ; m = max y ; e_i = expf(y_i - m) ; s = sequential sum e ;
 *   p_i = e_i / s.
 * This mirrors F.softmax(logits / T) (speculative.py:118, :145) closely but
 * not bit-for-bit; the acceptance parity contract therefore feeds the CUDA
 * kernel's own exported probabilities to oref_accept_*.  This function is
 * used only to time the CPU baseline. */
void oref_softmax_row(const float *x, int64_t V, float T, float *p) {
  float m = -INFINITY;
  for (int64_t i = 0; i < V; ++i) {
    float y = x[i] / T;
    p[i] = y;
    if (y > m) m = y;
  }
  float s = 0.0f;
  for (int64_t i = 0; i < V; ++i) {
    p[i] = expf(p[i] - m);
    s += p[i];
  }
  for (int64_t i = 0; i < V; ++i) p[i] /= s;
}

/* ---------------------------------------------------------------------------
 * Tree acceptance (no counterpart in the reference; defined by this build so
 * that a branching-1 tree reduces exactly to oref_accept_one).
 *
 * Nodes 0..N: node 0 is the root (the last emitted token), node i > 0 has
 * parent par[i] < i and token tok[i]; siblings are tested in increasing node
 * index (the builder numbers them in draft-rank order).  target_probs[u] is
 * the target distribution after node u, draft_probs[u] the draft
 * distribution node u's children were drawn from.  Walk from the root with
 * p = target_probs[u]:
 *   for each child c: ratio = q[x_c] > 0 ? min(1, p[x_c] / q[x_c]) : 0,
 *     accept iff u_next <= ratio  -> move to c (p = target_probs[c]);
 *       an accepted EOS stops (final = EOS, no further draw);
 *     reject -> d = max(0, p - q); s = sequential fp32 sum;
 *       if s > 1e-6: p = d / s (element-wise)   (else p is kept)
 *   all children rejected: final = sample_from(p, u_next)
 *   leaf reached:          final = sample_from(target_probs[u], u_next)
 * Outputs: path[0..na] = accepted node ids with path[0] = 0 (root), tokens of
 * the accepted nodes then the final token, na accepted drafts, eos flag.
 * ------------------------------------------------------------------------- */
int oref_accept_tree_one(int32_t N, int64_t V, const int32_t *par, const int32_t *tok,
                         const float *draft_probs,  /* [N+1][V] */
                         const float *target_probs, /* [N+1][V] */
                         int32_t eos, const float *u, int32_t *path, int32_t *tokens,
                         int32_t *num_accepted, uint8_t *eos_flag) {
  float *p = (float *)malloc(sizeof(float) * (size_t)(V > 0 ? V : 1));
  float *d = (float *)malloc(sizeof(float) * (size_t)(V > 0 ? V : 1));
  if (!p || !d) { free(p); free(d); return -1; }
  int32_t cur = 0, na = 0, used = 0, final_tok = -1;
  uint8_t e = 0;
  path[0] = 0;
  memcpy(p, target_probs, sizeof(float) * (size_t)V);
  for (;;) {
    const float *q = draft_probs + (size_t)cur * V;
    int32_t moved = -1, any_child = 0;
    for (int32_t c = cur + 1; c <= N; ++c) {
      if (par[c] != cur) continue;
      any_child = 1;
      const int32_t x = tok[c];
      const float qx = q[x], px = p[x];
      const float pq = px / qx;
      const float ratio = (qx > 0.0f) ? ((pq < 1.0f) ? pq : 1.0f) : 0.0f;
      const float r = u[used++];
      if (r <= ratio) { moved = c; break; }
      float s = 0.0f;
      for (int64_t i = 0; i < V; ++i) {
        const float t = p[i] - q[i];
        d[i] = t > 0.0f ? t : 0.0f;
        s += d[i];
      }
      if (s > 1e-6f)
        for (int64_t i = 0; i < V; ++i) p[i] = d[i] / s;
    }
    if (moved >= 0) {
      cur = moved;
      path[++na] = cur;
      tokens[na - 1] = tok[cur];
      if (tok[cur] == eos) { final_tok = eos; e = 1; break; }
      memcpy(p, target_probs + (size_t)cur * V, sizeof(float) * (size_t)V);
      continue;
    }
    final_tok = sample_from(any_child ? p : target_probs + (size_t)cur * V, V, u[used++]);
    if (final_tok == eos) e = 1;
    break;
  }
  tokens[na] = final_tok;
  *num_accepted = na;
  *eos_flag = e;
  free(p);
  free(d);
  return 0;
}

/* Greedy tree: at node u move to the first child whose token equals the
 * first-max argmax of target_probs[u]; otherwise final = that argmax (a leaf
 * gives its own argmax as the bonus). */
int oref_accept_tree_greedy_one(int32_t N, int64_t V, const int32_t *par, const int32_t *tok,
                                const float *target_probs, int32_t eos, int32_t *path, int32_t *tokens,
                                int32_t *num_accepted, uint8_t *eos_flag) {
  int32_t cur = 0, na = 0;
  path[0] = 0;
  for (;;) {
    const int32_t am = argmax_first(target_probs + (size_t)cur * V, V);
    int32_t moved = -1;
    for (int32_t c = cur + 1; c <= N; ++c)
      if (par[c] == cur && tok[c] == am) { moved = c; break; }
    if (moved < 0) {
      tokens[na] = am;
      *num_accepted = na;
      *eos_flag = (am == eos);
      return 0;
    }
    cur = moved;
    path[++na] = cur;
    tokens[na - 1] = tok[cur];
    if (tok[cur] == eos) {
      tokens[na] = eos;
      *num_accepted = na;
      *eos_flag = 1;
      return 0;
    }
  }
}
