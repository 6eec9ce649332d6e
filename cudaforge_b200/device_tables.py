"""Device-resident page tables for a fixed batch (no host round trip per step).

The host PagedKVCache (cudaforge_b200.kv_cache; reference semantics,
csrc/src/memory/paged_kv_cache.cpp:255-286 for the growth) stays the owner of
the page-table state.  While a DeviceTables is attached, the same growth runs
on the GPU every step (cf_kv_append_device: batch order, LIFO free stack, the
same blocks the host would hand out), so the step's commit reads tables that
are already on the device; the host cache replays the same growth later from
pinned copies of the per-step counts (catch_up), which keeps the two identical.

Contract: while attached, nothing else may change the cache (no register,
unregister, fork or append from elsewhere); call sync() before using the host
cache again.  Prefix caching must be off (the device path never evicts); a
batch that does not fit records CF_ENOMEM in the status word and changes
nothing."""
from __future__ import annotations

import collections
import ctypes
from typing import Sequence

import torch

from . import _lib


class CfKvAppendArgs(ctypes.Structure):
    _P = ctypes.c_void_p
    _fields_ = [("batch", ctypes.c_int32), ("block_size", ctypes.c_int32), ("n_append", _P), ("n_add", ctypes.c_int32),
                ("context_lens", _P), ("table_len", _P), ("tables", _P), ("max_blocks", ctypes.c_int32),
                ("free_stack", _P), ("free_top", _P), ("status", _P)]


def _L():
    L = _lib.lib()
    if not getattr(L, "_append_ready", False):
        L.cf_kv_append_device.argtypes = [ctypes.POINTER(CfKvAppendArgs), ctypes.c_void_p]
        L.cf_kvcache_export_free_stack.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32,
                                                   ctypes.POINTER(ctypes.c_uint32)]
        L._append_ready = True
    return L


class DeviceTables:
    def __init__(self, cache, seq_ids: Sequence[int], max_blocks: int, device, ring: int = 8):
        cfg = cache.get_config()
        if cfg.enable_prefix_caching:
            raise ValueError("device-resident page tables need prefix caching off (no eviction on the device)")
        self.cache, self.seq_ids = cache, list(seq_ids)
        self.B, self.cap, self.bs = len(self.seq_ids), int(max_blocks), cfg.block_size
        self.device = torch.device(device)
        self.tables = torch.full((self.B, self.cap), -1, dtype=torch.int32, device=self.device)
        self.table_len = torch.zeros(self.B, dtype=torch.int32, device=self.device)
        self.free_stack = torch.zeros(max(1, cfg.total_gpu_blocks), dtype=torch.int32, device=self.device)
        self.free_top = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._ring = [(torch.zeros(self.B, dtype=torch.int32).pin_memory(), torch.cuda.Event()) for _ in range(ring)]
        self._pending = collections.deque()  # (slot, n_add)
        self._next = 0
        self.emitted = 0  # tokens appended to the host cache so far

    # ---- host -> device ----
    def upload(self, context_lens: torch.Tensor) -> None:
        """Copy the host cache's tables and free stack to the device (after
        any host-side change; the pending growth must have been replayed)."""
        if self._pending:
            raise RuntimeError("DeviceTables.upload with growth still pending: call sync() first")
        pinned = torch.full((self.B * self.cap,), -1, dtype=torch.int32).pin_memory()
        ctx = torch.zeros(self.B, dtype=torch.int32).pin_memory()
        mb = self.cache.prepare_batch_into(self.seq_ids, pinned, ctx)
        if mb > self.cap:
            raise ValueError(f"a sequence needs {mb} blocks > max_blocks={self.cap}")
        full = torch.full((self.B, self.cap), -1, dtype=torch.int32)
        full[:, :mb] = pinned[: self.B * mb].view(self.B, mb)
        self.tables.copy_(full)
        self.table_len.copy_((full >= 0).sum(1).to(torch.int32))
        context_lens.copy_(ctx)
        L = _L()
        n = ctypes.c_uint32(0)
        h = self.cache._h
        _lib.check(L.cf_kvcache_export_free_stack(h, None, 0, ctypes.byref(n)), "export_free_stack")
        host = torch.zeros(max(1, n.value), dtype=torch.int32)
        _lib.check(L.cf_kvcache_export_free_stack(h, host.data_ptr(), n.value, ctypes.byref(n)), "export_free_stack")
        self.free_stack[: n.value].copy_(host[: n.value])
        self.free_top.fill_(n.value)
        torch.cuda.current_stream(self.device).synchronize()

    # ---- the device growth (stream-ordered, capturable) ----
    def append(self, counts: torch.Tensor, context_lens: torch.Tensor, n_add: int, status=None, stream=None) -> None:
        a = CfKvAppendArgs(batch=self.B, block_size=self.bs, n_append=counts.data_ptr(), n_add=int(n_add),
                           context_lens=context_lens.data_ptr(), table_len=self.table_len.data_ptr(),
                           tables=self.tables.data_ptr(), max_blocks=self.cap, free_stack=self.free_stack.data_ptr(),
                           free_top=self.free_top.data_ptr(), status=status.data_ptr() if status is not None else None)
        s = stream or torch.cuda.current_stream(self.device)
        _lib.check(_L().cf_kv_append_device(ctypes.byref(a), ctypes.c_void_p(s.cuda_stream)), "cf_kv_append_device")
        _lib.count()

    # ---- device -> host, lazily ----
    def record(self, counts: torch.Tensor, n_add: int) -> None:
        """Queue this step's counts for the host replay (async copy + event)."""
        if len(self._pending) == len(self._ring):
            self.catch_up(block_oldest=True)
        slot = self._next
        self._next = (self._next + 1) % len(self._ring)
        buf, ev = self._ring[slot]
        buf.copy_(counts, non_blocking=True)
        ev.record(torch.cuda.current_stream(self.device))
        self._pending.append((slot, n_add))

    def catch_up(self, block_oldest: bool = False, block_all: bool = False) -> int:
        """Replay the finished steps' growth on the host cache (in order).
        Returns the number of steps replayed."""
        done = 0
        while self._pending:
            slot, n_add = self._pending[0]
            buf, ev = self._ring[slot]
            if not ev.query():
                if not (block_all or (block_oldest and done == 0)):
                    break
                ev.synchronize()
            counts = [max(0, int(x)) + n_add for x in buf.tolist()]
            self.cache.append_batch(self.seq_ids, counts)
            self.emitted += sum(counts)
            self._pending.popleft()
            done += 1
        return done

    def sync(self) -> None:
        self.catch_up(block_all=True)
