// TEST INFRASTRUCTURE ONLY -- C entry points around the UNMODIFIED reference
// scheduler and model runner (CUDAForge csrc/src/scheduler/continuous_batcher.cpp,
// csrc/src/engine/model_runner.cpp), compiled from the reference sources by
// oracle/Makefile into oracle/_ref/libsched_ref.so.  Used to pin
// cudaforge_b200.serving against the reference on scripted operation sequences.
#include "cudaforge/engine/model_runner.h"
#include "cudaforge/scheduler/continuous_batcher.h"

#include <cstdint>
#include <memory>
#include <vector>

using cudaforge::engine::ModelRunner;
using cudaforge::engine::StreamOutput;
using cudaforge::scheduler::ContinuousBatcher;
using cudaforge::scheduler::Request;

struct RefSched {
  std::shared_ptr<ContinuousBatcher> batcher;
  std::shared_ptr<ModelRunner> runner;
};

extern "C" {

void *rs_create(uint64_t max_seqs, uint64_t max_tokens, uint64_t vocab, int32_t eos) {
  auto *h = new RefSched;
  h->batcher = std::make_shared<ContinuousBatcher>(max_seqs, max_tokens);
  h->runner = std::make_shared<ModelRunner>(h->batcher, vocab, eos);
  return h;
}

void rs_destroy(void *h) { delete static_cast<RefSched *>(h); }

int rs_add(void *h, uint64_t id, const int32_t *prompt, int32_t n, int32_t max_tokens, int32_t priority) {
  auto req = std::make_shared<Request>(id, std::vector<int32_t>(prompt, prompt + n), max_tokens, priority);
  return static_cast<RefSched *>(h)->batcher->add_request(req) ? 1 : 0;
}

void rs_cancel(void *h, uint64_t id) { static_cast<RefSched *>(h)->runner->cancel_request(id); }

void rs_update(void *h, const uint64_t *ids, int32_t n) {
  static_cast<RefSched *>(h)->batcher->update_requests_state(std::vector<uint64_t>(ids, ids + n));
}

uint64_t rs_step(void *h) { return static_cast<RefSched *>(h)->runner->step(); }

// Pops every streamed output; returns how many (at most cap are written).
int32_t rs_pop(void *h, uint64_t *ids, int32_t *tokens, uint8_t *final_flags, int32_t cap) {
  auto outs = static_cast<RefSched *>(h)->runner->get_stream_buffer()->pop_all();
  int32_t n = 0;
  for (const StreamOutput &o : outs) {
    if (n < cap) {
      ids[n] = o.request_id;
      tokens[n] = o.token_id;
      final_flags[n] = o.is_final ? 1 : 0;
    }
    ++n;
  }
  return n;
}

uint64_t rs_pending(void *h) { return static_cast<RefSched *>(h)->batcher->get_pending_count(); }
uint64_t rs_running(void *h) { return static_cast<RefSched *>(h)->batcher->get_running_count(); }
}
