// Host-side speculative verification engine: the reference's native
// SpeculativeEngine (csrc/include/cudaforge/scheduler/speculative.h:14-85,
// csrc/src/scheduler/speculative.cpp:8-150, bound in
// csrc/bindings/pybind_module.cpp:199-239) behind the C ABI.
//
// One engine owns a configuration and a std::mt19937 stream seeded once with
// config.rng_seed; every call of cf_spec_engine_verify draws its uniforms
// from that stream with std::uniform_real_distribution<float>(0, 1) in the
// reference's order (one per acceptance test, then one for the final
// sample, none after an accepted EOS), so a sequence of calls reproduces the
// reference engine's outputs exactly.  Calls on one engine are serialised by
// its mutex.  The per-sequence probability rows arrive as the reference
// receives them (one vector per row, possibly ragged).
//
// This is the reference's per-sequence CPU API, kept for drop-in
// compatibility.  Batches of logits go through the GPU acceptance kernel
// (cf_accept_sample); cf_spec_engine_draw_uniforms feeds that kernel from
// this engine's stream.
#include "cf_api.h"

#include <algorithm>
#include <mutex>
#include <new>
#include <random>
#include <vector>

struct cf_spec_engine {
  cf_spec_config cfg;
  std::mt19937 rng;
  std::mutex mu;
};

namespace {

bool valid_config(const cf_spec_config *c) { return c != nullptr && c->gamma >= 0; }

// First index i with r <= (v_0 + ... + v_i) accumulated left to right in
// fp32; the last index when the running sum never reaches r.
int32_t inverse_cdf(const float *v, int64_t n, float r) {
  float cum = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    cum += v[i];
    if (r <= cum) return static_cast<int32_t>(i);
  }
  return static_cast<int32_t>(n - 1);
}

// std::max_element: the first element that no later element exceeds.
int32_t first_argmax(const float *v, int64_t n) {
  int64_t best = 0;
  for (int64_t i = 1; i < n; ++i)
    if (v[best] < v[i]) best = i;
  return static_cast<int32_t>(best);
}

}  // namespace

extern "C" int cf_spec_engine_create(const cf_spec_config *config, cf_spec_engine **out) {
  if (!out || !valid_config(config)) return CF_EINVAL;
  cf_spec_engine *e = new (std::nothrow) cf_spec_engine;
  if (!e) return CF_ENOMEM;
  e->cfg = *config;
  e->rng.seed(static_cast<std::mt19937::result_type>(config->rng_seed));
  *out = e;
  return CF_OK;
}

extern "C" void cf_spec_engine_destroy(cf_spec_engine *e) { delete e; }

extern "C" int cf_spec_engine_set_config(cf_spec_engine *e, const cf_spec_config *config) {
  if (!e || !valid_config(config)) return CF_EINVAL;
  std::lock_guard<std::mutex> g(e->mu);
  e->cfg = *config;  // the stream is not reseeded (speculative.h:70-73)
  return CF_OK;
}

extern "C" int cf_spec_engine_get_config(cf_spec_engine *e, cf_spec_config *out) {
  if (!e || !out) return CF_EINVAL;
  std::lock_guard<std::mutex> g(e->mu);
  *out = e->cfg;
  return CF_OK;
}

extern "C" int cf_spec_engine_verify(cf_spec_engine *e, int32_t k, const int32_t *draft_tokens,
                                     const float *const *draft_rows, const int64_t *draft_lens, int32_t n_draft,
                                     const float *const *target_rows, const int64_t *target_lens, int32_t n_target,
                                     int32_t eos_token_id, int32_t greedy, int32_t *out_accepted,
                                     int32_t *out_num_accepted, int32_t *out_final_token, int32_t *out_eos) {
  if (!e || k < 0 || !out_num_accepted || !out_final_token || !out_eos || (k > 0 && (!draft_tokens || !out_accepted)))
    return CF_EINVAL;
  // speculative.cpp:58-62 (the greedy path of the reference checks nothing; here it needs K+1 rows too)
  if ((!greedy && n_draft != k) || n_target < k + 1 || !target_rows || !target_lens) return CF_EINVAL;
  if (!greedy && k > 0 && (!draft_rows || !draft_lens)) return CF_EINVAL;
  for (int32_t i = 0; i <= k; ++i)
    if (target_lens[i] < 1 || !target_rows[i]) return CF_EINVAL;
  std::lock_guard<std::mutex> g(e->mu);
  std::uniform_real_distribution<float> uni(0.0f, 1.0f);
  int32_t na = 0;
  *out_eos = 0;
  for (int32_t i = 0; i < k; ++i) {
    const int32_t tok = draft_tokens[i];
    const float *t = target_rows[i];
    const int64_t V = target_lens[i];
    if (greedy) {  // speculative.cpp:105-150
      const int32_t am = first_argmax(t, V);
      if (tok != am) {
        *out_final_token = am;
        *out_eos = am == eos_token_id;
        *out_num_accepted = na;
        return CF_OK;
      }
    } else {  // speculative.cpp:66-92
      const float *d = draft_rows[i];
      const int64_t Vd = draft_lens[i];
      if (tok < 0 || tok >= V || tok >= Vd) return CF_ERANGE;  // the reference reads out of bounds here
      const float q = d[tok], p = t[tok];
      const float ratio = (q > 0.0f) ? std::min(1.0f, p / q) : 0.0f;
      const float r = uni(e->rng);
      if (!(r <= ratio)) {
        // rejected: resample from norm(max(0, p - q)), or from p when that mass is <= 1e-6
        if (Vd < V) return CF_EINVAL;
        std::vector<float> adj(static_cast<size_t>(V));
        float sum = 0.0f;
        for (int64_t x = 0; x < V; ++x) {
          adj[x] = std::max(0.0f, t[x] - d[x]);
          sum += adj[x];
        }
        int32_t fin;
        if (sum <= 1e-6f) {
          fin = inverse_cdf(t, V, uni(e->rng));
        } else {
          for (int64_t x = 0; x < V; ++x) adj[x] /= sum;
          fin = inverse_cdf(adj.data(), V, uni(e->rng));
        }
        *out_final_token = fin;
        *out_eos = fin == eos_token_id;
        *out_num_accepted = na;
        return CF_OK;
      }
    }
    out_accepted[na++] = tok;
    if (tok == eos_token_id) {  // an accepted EOS ends the sequence; nothing more is drawn
      *out_final_token = eos_token_id;
      *out_eos = 1;
      *out_num_accepted = na;
      return CF_OK;
    }
  }
  // all K accepted: the bonus token from target row K
  const int32_t fin = greedy ? first_argmax(target_rows[k], target_lens[k])
                             : inverse_cdf(target_rows[k], target_lens[k], uni(e->rng));
  *out_final_token = fin;
  *out_eos = fin == eos_token_id;
  *out_num_accepted = na;
  return CF_OK;
}

extern "C" int cf_spec_engine_draw_uniforms(cf_spec_engine *e, int64_t n, float *out) {
  if (!e || n < 0 || (n > 0 && !out)) return CF_EINVAL;
  std::lock_guard<std::mutex> g(e->mu);
  std::uniform_real_distribution<float> uni(0.0f, 1.0f);
  for (int64_t i = 0; i < n; ++i) out[i] = uni(e->rng);
  return CF_OK;
}
