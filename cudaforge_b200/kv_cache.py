"""Paged KV cache with the reference's interface and page-table semantics.

Mirrors the `_C` classes cudaforge/engine.py uses (KVCacheConfig,
KVCacheStats, BlockAllocator, PagedKVCache; bound in the reference at
csrc/bindings/pybind_module.cpp:27-99) over the C ABI cf_kvcache_*.  The K and
V pools are device tensors owned by this object, laid out as the reference
lays them out: [block][layer][kv_head][slot][head_dim].
"""
from __future__ import annotations

import ctypes
import dataclasses
from typing import List, Sequence

import torch

from . import _lib

_P = ctypes.c_void_p


class OutOfPagesException(RuntimeError):
    """The KV pool is exhausted (paged_kv_cache.h:31-34)."""


class CfKvConfig(ctypes.Structure):
    _fields_ = [("num_layers", ctypes.c_uint32), ("num_kv_heads", ctypes.c_uint32),
                ("head_dim", ctypes.c_uint32), ("block_size", ctypes.c_uint32),
                ("element_size_bytes", ctypes.c_uint64), ("total_gpu_blocks", ctypes.c_uint64),
                ("enable_prefix_caching", ctypes.c_int32), ("max_supported_batch_size", ctypes.c_uint64),
                ("max_blocks_per_sequence", ctypes.c_uint64)]


class CfKvStats(ctypes.Structure):
    _fields_ = [("total_blocks", ctypes.c_uint64), ("free_blocks", ctypes.c_uint64),
                ("allocated_blocks", ctypes.c_uint64), ("cached_prefix_blocks", ctypes.c_uint64),
                ("total_memory_bytes", ctypes.c_uint64), ("used_memory_bytes", ctypes.c_uint64),
                ("pool_utilization_ratio", ctypes.c_double), ("active_sequences_count", ctypes.c_uint32),
                ("prefix_cache_hits", ctypes.c_uint64), ("prefix_cache_misses", ctypes.c_uint64),
                ("lru_evictions_count", ctypes.c_uint64)]


@dataclasses.dataclass
class KVCacheConfig:
    """KVCacheConfig (paged_kv_cache.h:36-46), same fields and defaults."""

    num_layers: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    block_size: int = 16
    element_size_bytes: int = 2
    total_gpu_blocks: int = 1024
    enable_prefix_caching: bool = True
    max_supported_batch_size: int = 256
    max_blocks_per_sequence: int = 512


@dataclasses.dataclass
class KVCacheStats:
    """KVCacheStats (paged_kv_cache.h:63-75)."""

    total_blocks: int = 0
    free_blocks: int = 0
    allocated_blocks: int = 0
    cached_prefix_blocks: int = 0
    total_memory_bytes: int = 0
    used_memory_bytes: int = 0
    pool_utilization_ratio: float = 0.0
    active_sequences_count: int = 0
    prefix_cache_hits: int = 0
    prefix_cache_misses: int = 0
    lru_evictions_count: int = 0


class BlockAllocator:
    """Accepts the constructor engine.py calls, BlockAllocator(total_gpu_blocks,
    block_size) (engine.py:149-151), which the reference binding lacks.  Device
    memory is allocated through torch's caching allocator; the VRAM headroom
    default of the reference (0.05) is checked against the request."""

    def __init__(self, total_gpu_blocks: int = 0, block_size: int = 16, vram_headroom_fraction: float = 0.05,
                 device=None):
        self.total_gpu_blocks = int(total_gpu_blocks)
        self.block_size = int(block_size)
        self.vram_headroom_fraction = float(vram_headroom_fraction)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device()) \
            if torch.cuda.is_available() else torch.device("cpu")

    def allocate(self, nbytes: int, dtype=torch.uint8) -> torch.Tensor:
        if self.device.type == "cuda":
            free, total = torch.cuda.mem_get_info(self.device)
            if nbytes > free - self.vram_headroom_fraction * total:
                raise MemoryError(f"BlockAllocator: {nbytes} bytes exceed the VRAM safety budget")
        return torch.zeros(nbytes // torch.empty((), dtype=dtype).element_size(), dtype=dtype, device=self.device)


def _lib_kv():
    L = _lib.lib()
    if not getattr(L, "_kv_ready", False):
        L.cf_kvcache_create.restype = _P
        L.cf_kvcache_create.argtypes = [ctypes.POINTER(CfKvConfig), _P, _P]
        L.cf_kvcache_destroy.argtypes = [_P]
        L.cf_kvcache_register_sequence.argtypes = [_P, ctypes.c_uint64, _P, ctypes.c_uint32, _P]
        L.cf_kvcache_append_tokens.argtypes = [_P, ctypes.c_uint64, ctypes.c_uint32]
        L.cf_kvcache_append_batch.argtypes = [_P, _P, _P, ctypes.c_uint32]
        L.cf_kvcache_unregister_sequence.argtypes = [_P, ctypes.c_uint64]
        L.cf_kvcache_fork_sequence.argtypes = [_P, ctypes.c_uint64, ctypes.c_uint64]
        L.cf_kvcache_get_block_table.argtypes = [_P, ctypes.c_uint64, _P, ctypes.c_uint32, _P]
        L.cf_kvcache_prepare_batch.argtypes = [_P, _P, ctypes.c_uint32, _P, ctypes.c_uint32, _P, _P]
        L.cf_kvcache_get_stats.argtypes = [_P, ctypes.POINTER(CfKvStats)]
        L.cf_kvcache_key_block_ptr.restype = _P
        L.cf_kvcache_key_block_ptr.argtypes = [_P, ctypes.c_int32, ctypes.c_uint32]
        L.cf_kvcache_value_block_ptr.restype = _P
        L.cf_kvcache_value_block_ptr.argtypes = [_P, ctypes.c_int32, ctypes.c_uint32]
        L._kv_ready = True
    return L


class PagedKVCache:
    """PagedKVCache(config, allocator) with the reference's methods."""

    def __init__(self, config: KVCacheConfig, allocator: BlockAllocator | None = None, *, dtype=torch.bfloat16,
                 allocate_pools: bool = True):
        self._cfg = config
        self.dtype = dtype
        self.allocator = allocator or BlockAllocator(config.total_gpu_blocks, config.block_size)
        esz = torch.empty((), dtype=dtype).element_size()
        if esz != config.element_size_bytes:
            raise ValueError("element_size_bytes must match the pool dtype")
        self.layer_block_elems = config.num_kv_heads * config.block_size * config.head_dim
        self.block_elems = config.num_layers * self.layer_block_elems
        if allocate_pools:
            n = config.total_gpu_blocks * self.block_elems
            self.key_pool = self.allocator.allocate(n * esz, dtype=dtype)
            self.value_pool = self.allocator.allocate(n * esz, dtype=dtype)
        else:  # page tables only (host-side tests)
            self.key_pool = self.value_pool = None
        c = CfKvConfig(config.num_layers, config.num_kv_heads, config.head_dim, config.block_size,
                       config.element_size_bytes, config.total_gpu_blocks, int(bool(config.enable_prefix_caching)),
                       config.max_supported_batch_size, config.max_blocks_per_sequence)
        L = _lib_kv()
        self._h = L.cf_kvcache_create(ctypes.byref(c),
                                      self.key_pool.data_ptr() if self.key_pool is not None else None,
                                      self.value_pool.data_ptr() if self.value_pool is not None else None)
        if not self._h:
            raise ValueError("invalid KVCacheConfig")
        self._table_buf = None

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                _lib_kv().cf_kvcache_destroy(h)
            except Exception:  # interpreter shutdown: module globals may already be gone
                pass
            self._h = None

    @staticmethod
    def _check(rc, what):
        if rc == _lib.CF_ENOMEM:
            raise OutOfPagesException(f"OutOfPagesException: Physical KV Cache pool exhausted ({what})")
        if rc == _lib.CF_ERANGE:
            raise RuntimeError(f"{what}: sequence not registered / limit exceeded")
        _lib.check(rc, what)

    def register_sequence_with_prefix(self, sequence_id: int, prompt_tokens: Sequence[int]) -> int:
        t = (ctypes.c_int32 * len(prompt_tokens))(*[int(x) for x in prompt_tokens])
        m = ctypes.c_uint32(0)
        self._check(_lib_kv().cf_kvcache_register_sequence(self._h, sequence_id, t, len(prompt_tokens),
                                                           ctypes.byref(m)), "register_sequence_with_prefix")
        return m.value

    def append_tokens(self, sequence_id: int, num_tokens: int = 1) -> None:
        self._check(_lib_kv().cf_kvcache_append_tokens(self._h, sequence_id, num_tokens), "append_tokens")

    def append_batch(self, sequence_ids: Sequence[int], counts) -> None:
        """append_tokens(sequence_ids[i], counts[i]) for every i in order (counts <= 0 skipped)."""
        B = len(sequence_ids)
        ids = (ctypes.c_uint64 * max(1, B))(*sequence_ids)
        n = (ctypes.c_int32 * max(1, B))(*[int(x) for x in counts])
        self._check(_lib_kv().cf_kvcache_append_batch(self._h, ids, n, B), "append_tokens")

    def prepare_batch_into(self, sequence_ids: Sequence[int], tables: torch.Tensor, ctx: torch.Tensor) -> int:
        """prepare_batch_metadata into caller (pinned) CPU buffers: tables is a
        flat int32 buffer, filled as [B, max_blocks]; returns max_blocks."""
        B = len(sequence_ids)
        ids = (ctypes.c_uint64 * max(1, B))(*sequence_ids)
        mb = ctypes.c_uint32(0)
        self._check(_lib_kv().cf_kvcache_prepare_batch(self._h, ids, B, tables.data_ptr(), tables.numel(),
                                                       ctx.data_ptr(), ctypes.byref(mb)), "prepare_batch_metadata")
        return mb.value

    def unregister_sequence(self, sequence_id: int) -> None:
        self._check(_lib_kv().cf_kvcache_unregister_sequence(self._h, sequence_id), "unregister_sequence")

    def fork_sequence(self, parent_sequence_id: int, child_sequence_id: int) -> None:
        self._check(_lib_kv().cf_kvcache_fork_sequence(self._h, parent_sequence_id, child_sequence_id),
                    "fork_sequence")

    def get_block_table(self, sequence_id: int) -> List[int]:
        n = ctypes.c_uint32(0)
        self._check(_lib_kv().cf_kvcache_get_block_table(self._h, sequence_id, None, 0, ctypes.byref(n)),
                    "get_block_table")
        buf = (ctypes.c_int32 * max(1, n.value))()
        self._check(_lib_kv().cf_kvcache_get_block_table(self._h, sequence_id, buf, n.value, ctypes.byref(n)),
                    "get_block_table")
        return list(buf[: n.value])

    def prepare_batch_host(self, sequence_ids: Sequence[int]):
        """Host half of prepare_batch_metadata: (tables [B, max_blocks] int32
        padded with -1, context_lens [B] int32), as CPU tensors."""
        B = len(sequence_ids)
        ids = (ctypes.c_uint64 * max(1, B))(*sequence_ids)
        mb = ctypes.c_uint32(0)
        ctx = torch.zeros(B, dtype=torch.int32)
        L = _lib_kv()
        self._check(L.cf_kvcache_prepare_batch(self._h, ids, B, None, 0, ctx.data_ptr() if B else None,
                                               ctypes.byref(mb)), "prepare_batch_metadata")
        tables = torch.full((B, mb.value), -1, dtype=torch.int32)
        self._check(L.cf_kvcache_prepare_batch(self._h, ids, B, tables.data_ptr() if tables.numel() else None,
                                               tables.numel(), ctx.data_ptr() if B else None, ctypes.byref(mb)),
                    "prepare_batch_metadata")
        return tables, ctx

    def prepare_batch_metadata(self, sequence_ids: Sequence[int], device=None, non_blocking: bool = True):
        """prepare_batch_metadata (paged_kv_cache.cpp:318-396): device copies of
        the padded block table and the context lengths."""
        tables, ctx = self.prepare_batch_host(sequence_ids)
        dev = device or (self.key_pool.device if self.key_pool is not None else "cuda")
        return (tables.pin_memory().to(dev, non_blocking=non_blocking),
                ctx.pin_memory().to(dev, non_blocking=non_blocking))

    def get_config(self) -> KVCacheConfig:
        return self._cfg

    def get_stats(self) -> KVCacheStats:
        s = CfKvStats()
        self._check(_lib_kv().cf_kvcache_get_stats(self._h, ctypes.byref(s)), "get_stats")
        return KVCacheStats(**{f: getattr(s, f) for f, _ in CfKvStats._fields_})

    def get_key_block_ptr(self, block_id: int, layer_idx: int) -> int:
        return _lib_kv().cf_kvcache_key_block_ptr(self._h, block_id, layer_idx) or 0

    def get_value_block_ptr(self, block_id: int, layer_idx: int) -> int:
        return _lib_kv().cf_kvcache_value_block_ptr(self._h, block_id, layer_idx) or 0

    # pool geometry for the kernels
    @property
    def bytes_per_block(self) -> int:
        return self.block_elems * self._cfg.element_size_bytes

    @property
    def layer_block_bytes(self) -> int:
        return self.layer_block_elems * self._cfg.element_size_bytes
