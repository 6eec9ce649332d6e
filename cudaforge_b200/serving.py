"""Engine-facing scheduler and streaming classes with the reference's semantics.

cudaforge/engine.py (LLMEngine, engine.py:149-253) constructs these from the
native module: Request / RequestState / BatchStepResult / ContinuousBatcher
(csrc/include/cudaforge/scheduler/continuous_batcher.h:17-124,
csrc/src/scheduler/continuous_batcher.cpp:8-159) and StreamOutput /
TokenStreamBuffer / ModelRunner (csrc/include/cudaforge/engine/model_runner.h,
csrc/src/engine/model_runner.cpp:10-173), bound at
csrc/bindings/pybind_module.cpp:104-194.  They are host bookkeeping around
the verify + accept path, kept so that engine.py runs unchanged against this
package:

  * ContinuousBatcher admits waiting requests by priority (higher first, then
    earlier arrival) under a sequence and a token budget, charges one token
    per running request, and preempts the lowest-priority running request
    when the decode budget runs out (the preempted request may still be in
    this step's decode list, as in the reference);
  * ModelRunner.step schedules, drops cancelled requests and emits one token
    per scheduled request into the stream buffer.  Its token rule is the
    reference stub's ((last token + 1) mod vocab, model_runner.cpp:106-173):
    the reference runner has no model, and the speculative step is driven
    through cudaforge_b200.verifier / speculative instead.

Vector fields of the bound C++ structs read as copies in Python (pybind's
def_readwrite); prompt_tokens and generated_tokens do the same here.
"""
from __future__ import annotations

import enum
import heapq
import itertools
import threading
from typing import Iterable, List, Optional


class RequestState(enum.IntEnum):
    WAITING = 0
    RUNNING = 1
    FINISHED = 2
    PREEMPTED = 3


_arrival = itertools.count()


class Request:
    """Request(req_id, prompt, max_tokens=128, priority=0)."""

    def __init__(self, req_id: int, prompt: Iterable[int], max_tokens: int = 128, priority: int = 0):
        self.id = int(req_id)
        self._prompt = [int(t) for t in prompt]
        self._generated: List[int] = []
        self.max_new_tokens = int(max_tokens)
        self.priority = int(priority)
        self.state = RequestState.WAITING
        self._arrival = next(_arrival)

    @property
    def prompt_tokens(self) -> List[int]:
        return list(self._prompt)

    @prompt_tokens.setter
    def prompt_tokens(self, v):
        self._prompt = [int(t) for t in v]

    @property
    def generated_tokens(self) -> List[int]:
        return list(self._generated)

    @generated_tokens.setter
    def generated_tokens(self, v):
        self._generated = [int(t) for t in v]

    def get_total_length(self) -> int:
        return len(self._prompt) + len(self._generated)

    def is_finished(self) -> bool:
        return self.state == RequestState.FINISHED or len(self._generated) >= self.max_new_tokens


class BatchStepResult:
    def __init__(self):
        self.prefill_requests: List[Request] = []
        self.decode_requests: List[Request] = []
        self.total_batched_tokens = 0
        self.preempted_count = 0


class ContinuousBatcher:
    """ContinuousBatcher(max_num_seqs=256, max_num_batched_tokens=8192)."""

    def __init__(self, max_num_seqs: int = 256, max_num_batched_tokens: int = 8192):
        self.max_num_seqs = int(max_num_seqs)
        self.max_num_batched_tokens = int(max_num_batched_tokens)
        self._mu = threading.Lock()
        self._waiting: list = []  # heap of (-priority, arrival, request)
        self._running: List[Request] = []
        self._map: dict = {}

    def _push(self, r: Request) -> None:
        heapq.heappush(self._waiting, (-r.priority, r._arrival, r))

    def add_request(self, request: Request) -> bool:
        if request is None or not request._prompt:
            return False
        with self._mu:
            if request.id in self._map:
                return False
            request.state = RequestState.WAITING
            self._map[request.id] = request
            self._push(request)
            return True

    def cancel_request(self, request_id: int) -> bool:
        with self._mu:
            r = self._map.pop(int(request_id), None)
            if r is None:
                return False
            r.state = RequestState.FINISHED  # stays in the waiting heap; skipped when popped
            self._running = [x for x in self._running if x.id != r.id]
            return True

    def _preempt(self, res: BatchStepResult) -> None:
        self._running.sort(key=lambda x: x.priority)  # lowest priority first
        if self._running:
            r = self._running.pop(0)
            r.state = RequestState.PREEMPTED
            self._push(r)
            res.preempted_count += 1

    def schedule_step(self) -> BatchStepResult:
        with self._mu:
            res = BatchStepResult()
            used = 0
            active = []
            for r in self._running:
                if not r.is_finished() and r.state == RequestState.RUNNING:
                    active.append(r)
                else:
                    r.state = RequestState.FINISHED
                    self._map.pop(r.id, None)
            self._running = active
            for r in list(self._running):
                if used + 1 <= self.max_num_batched_tokens:
                    res.decode_requests.append(r)
                    used += 1
                else:
                    self._preempt(res)
                    break
            deferred = []
            while self._waiting and len(self._running) < self.max_num_seqs:
                _, _, cand = heapq.heappop(self._waiting)
                if cand.state == RequestState.FINISHED:
                    continue
                n = len(cand._prompt)
                if used + n <= self.max_num_batched_tokens:
                    cand.state = RequestState.RUNNING
                    res.prefill_requests.append(cand)
                    self._running.append(cand)
                    used += n
                else:
                    deferred.append(cand)
                    break
            for r in deferred:
                self._push(r)
            res.total_batched_tokens = used
            return res

    def update_requests_state(self, finished_ids: Iterable[int]) -> None:
        with self._mu:
            for i in finished_ids:
                r = self._map.get(int(i))
                if r is not None:
                    r.state = RequestState.FINISHED

    def get_pending_count(self) -> int:
        with self._mu:
            return len(self._waiting)

    def get_running_count(self) -> int:
        with self._mu:
            return len(self._running)


class StreamOutput:
    """StreamOutput() / StreamOutput(req_id, tok_id, final_flag)."""

    def __init__(self, req_id: int = 0, tok_id: int = 0, final_flag: bool = False):
        self.request_id = int(req_id)
        self.token_id = int(tok_id)
        self.is_final = bool(final_flag)


class TokenStreamBuffer:
    """Thread-safe FIFO of StreamOutput (model_runner.cpp:14-60)."""

    def __init__(self):
        self._cv = threading.Condition()
        self._q: List[StreamOutput] = []

    def push(self, output: StreamOutput) -> None:
        with self._cv:
            self._q.append(output)
            self._cv.notify()

    def push_batch(self, outputs: Iterable[StreamOutput]) -> None:
        outputs = list(outputs)
        if not outputs:
            return
        with self._cv:
            self._q.extend(outputs)
            self._cv.notify_all()

    def pop_all(self) -> List[StreamOutput]:
        with self._cv:
            out, self._q = self._q, []
            return out

    def pop_timeout(self, timeout_ms: int) -> Optional[StreamOutput]:
        with self._cv:
            if not self._cv.wait_for(lambda: bool(self._q), timeout=timeout_ms / 1e3):
                return None
            return self._q.pop(0)

    def size(self) -> int:
        with self._cv:
            return len(self._q)

    def empty(self) -> bool:
        with self._cv:
            return not self._q


class ModelRunner:
    """ModelRunner(batcher, vocab_size, eos_token_id)."""

    def __init__(self, batcher: ContinuousBatcher, vocab_size: int, eos_token_id: int):
        self._batcher = batcher
        self._stream = TokenStreamBuffer()
        self.vocab_size = int(vocab_size)
        self.eos_token_id = int(eos_token_id)
        self._mu = threading.Lock()
        self._cancelled: set = set()

    def cancel_request(self, request_id: int) -> None:
        with self._mu:
            self._cancelled.add(int(request_id))
        if self._batcher is not None:
            self._batcher.cancel_request(request_id)

    def is_cancelled(self, request_id: int) -> bool:
        with self._mu:
            return int(request_id) in self._cancelled

    def get_stream_buffer(self) -> TokenStreamBuffer:
        return self._stream

    def _emit(self, r: Request, tok: int, outs: list, finished: list) -> None:
        r._generated.append(tok)
        final = tok == self.eos_token_id or len(r._generated) >= r.max_new_tokens
        outs.append(StreamOutput(r.id, tok, final))
        if final:
            r.state = RequestState.FINISHED
            finished.append(r.id)

    def step(self) -> int:
        if self._batcher is None:
            return 0
        res = self._batcher.schedule_step()
        with self._mu:
            if self._cancelled:
                res.prefill_requests = [r for r in res.prefill_requests if r.id not in self._cancelled]
                res.decode_requests = [r for r in res.decode_requests if r.id not in self._cancelled]
        total = len(res.prefill_requests) + len(res.decode_requests)
        if total == 0:
            return 0
        outs: List[StreamOutput] = []
        finished: List[int] = []
        for r in res.prefill_requests:
            tok = 0 if not r._prompt else (r._prompt[-1] + 1) % self.vocab_size
            self._emit(r, tok, outs, finished)
        for r in res.decode_requests:
            last = r._generated[-1] if r._generated else 0
            self._emit(r, (last + 1) % self.vocab_size, outs, finished)
        self._stream.push_batch(outs)
        if finished:
            self._batcher.update_requests_state(finished)
        return total
