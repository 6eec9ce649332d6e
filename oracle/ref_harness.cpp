// TEST INFRASTRUCTURE ONLY -- C entry points around the UNMODIFIED reference
// acceptance code (CUDAForge csrc/src/scheduler/speculative.cpp), compiled
// from the reference sources by oracle/Makefile into oracle/_ref/.  Used to
// pin oracle/accept_ref.c and to time the reference CPU path.
#include "cudaforge/scheduler/speculative.h"

#include <cstdint>
#include <random>
#include <vector>

using cudaforge::scheduler::SpeculativeConfig;
using cudaforge::scheduler::SpeculativeEngine;

extern "C" {

// One call of SpeculativeEngine::verify_candidates (speculative.cpp:50-103)
// on a fresh engine seeded with `seed`.  tokens[0..na-1] accepted, tokens[na]
// final.  Returns 0, or -1 if the reference threw.
int ref_verify(uint64_t seed, int32_t K, int64_t V, const int32_t *draft_tokens,
               const float *draft_probs, const float *target_probs,
               int32_t eos, int32_t *tokens, int32_t *num_accepted,
               uint8_t *eos_flag) {
  SpeculativeConfig cfg;
  cfg.gamma = (size_t)K;
  cfg.rng_seed = seed;
  SpeculativeEngine eng(cfg);
  std::vector<int32_t> dt(draft_tokens, draft_tokens + K);
  std::vector<std::vector<float>> dp(K), tp(K + 1);
  for (int i = 0; i < K; ++i)
    dp[i].assign(draft_probs + (size_t)i * V, draft_probs + (size_t)(i + 1) * V);
  for (int i = 0; i <= K; ++i)
    tp[i].assign(target_probs + (size_t)i * V,
                 target_probs + (size_t)(i + 1) * V);
  try {
    auto r = eng.verify_candidates(dt, dp, tp, eos);
    for (size_t i = 0; i < r.accepted_tokens.size(); ++i)
      tokens[i] = r.accepted_tokens[i];
    tokens[r.num_accepted] = r.final_token;
    *num_accepted = (int32_t)r.num_accepted;
    *eos_flag = r.end_of_sequence ? 1 : 0;
  } catch (...) {
    return -1;
  }
  return 0;
}

// verify_candidates_greedy (speculative.cpp:105-150).
int ref_verify_greedy(int32_t K, int64_t V, const int32_t *draft_tokens,
                      const float *target_probs, int32_t eos, int32_t *tokens,
                      int32_t *num_accepted, uint8_t *eos_flag) {
  SpeculativeConfig cfg;
  SpeculativeEngine eng(cfg);
  std::vector<int32_t> dt(draft_tokens, draft_tokens + K);
  std::vector<std::vector<float>> tp(K + 1);
  for (int i = 0; i <= K; ++i)
    tp[i].assign(target_probs + (size_t)i * V,
                 target_probs + (size_t)(i + 1) * V);
  auto r = eng.verify_candidates_greedy(dt, tp, eos);
  for (size_t i = 0; i < r.accepted_tokens.size(); ++i)
    tokens[i] = r.accepted_tokens[i];
  tokens[r.num_accepted] = r.final_token;
  *num_accepted = (int32_t)r.num_accepted;
  *eos_flag = r.end_of_sequence ? 1 : 0;
  return 0;
}

// The first n draws the reference engine would make: std::mt19937(seed)
// through std::uniform_real_distribution<float>(0,1), the same engine and
// distribution the reference constructs (speculative.cpp:9, :13, :64).
void ref_uniforms(uint64_t seed, int32_t n, float *out) {
  std::mt19937 rng(seed);
  std::uniform_real_distribution<float> d(0.0f, 1.0f);
  for (int i = 0; i < n; ++i) out[i] = d(rng);
}

// Time-oriented batch call: B sequences through one engine per call, as a
// serving loop would use it (probabilities already computed).
int ref_verify_batch(uint64_t seed, int32_t B, int32_t K, int64_t V,
                     const int32_t *draft_tokens, const float *draft_probs,
                     const float *target_probs, int32_t eos, int32_t *tokens,
                     int32_t *num_accepted, uint8_t *eos_flag) {
  for (int b = 0; b < B; ++b) {
    int rc = ref_verify(seed + (uint64_t)b, K, V, draft_tokens + (size_t)b * K,
                        draft_probs + (size_t)b * K * V,
                        target_probs + (size_t)b * (K + 1) * V, eos,
                        tokens + (size_t)b * (K + 1), num_accepted + b,
                        eos_flag + b);
    if (rc) return rc;
  }
  return 0;
}

// B consecutive verify_candidates calls on ONE engine seeded with `seed`
// (the engine's stream carries over between calls, speculative.h:70-82);
// sequence b is call b.
int ref_verify_stream(uint64_t seed, int32_t B, int32_t K, int64_t V,
                      const int32_t *draft_tokens, const float *draft_probs,
                      const float *target_probs, int32_t eos, int32_t *tokens,
                      int32_t *num_accepted, uint8_t *eos_flag) {
  SpeculativeConfig cfg;
  cfg.gamma = (size_t)K;
  cfg.rng_seed = seed;
  SpeculativeEngine eng(cfg);
  for (int b = 0; b < B; ++b) {
    std::vector<int32_t> dt(draft_tokens + (size_t)b * K, draft_tokens + (size_t)(b + 1) * K);
    std::vector<std::vector<float>> dp(K), tp(K + 1);
    const float *d = draft_probs + (size_t)b * K * V, *t = target_probs + (size_t)b * (K + 1) * V;
    for (int i = 0; i < K; ++i) dp[i].assign(d + (size_t)i * V, d + (size_t)(i + 1) * V);
    for (int i = 0; i <= K; ++i) tp[i].assign(t + (size_t)i * V, t + (size_t)(i + 1) * V);
    try {
      auto r = eng.verify_candidates(dt, dp, tp, eos);
      int32_t *o = tokens + (size_t)b * (K + 1);
      for (size_t i = 0; i < r.accepted_tokens.size(); ++i) o[i] = r.accepted_tokens[i];
      o[r.num_accepted] = r.final_token;
      num_accepted[b] = (int32_t)r.num_accepted;
      eos_flag[b] = r.end_of_sequence ? 1 : 0;
    } catch (...) {
      return -1;
    }
  }
  return 0;
}
}
