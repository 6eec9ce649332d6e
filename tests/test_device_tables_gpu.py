"""GPU: device-resident page tables (cf_kv_append_device, DeviceTables,
BatchVerifier(device_tables=True)).

The device growth must hand out exactly the blocks the host cache hands out
(the host cache is itself pinned to the compiled reference PagedKVCache by
tests/test_kv_cache.py): random per-step counts in batch order, across many
steps, leave identical tables and an identical free stack; a batch that does
not fit records CF_ENOMEM and changes nothing.  A verifier with device tables
(one CUDA graph per step, no host round trip) gives the same acceptance
results, page tables and pool contents as the host-table verifier."""
import numpy as np
import pytest
import torch

from cudaforge_b200 import _lib
from cudaforge_b200.device_tables import DeviceTables
from cudaforge_b200.kv_cache import KVCacheConfig, PagedKVCache

pytestmark = pytest.mark.gpu


def _host_tables(cache, ids, cap):
    out = torch.full((len(ids), cap), -1, dtype=torch.int32)
    for i, s in enumerate(ids):
        t = cache.get_block_table(s)
        out[i, : len(t)] = torch.tensor(t, dtype=torch.int32)
    return out


@pytest.mark.parametrize("seed", range(4))
def test_device_growth_matches_host_cache(seed):
    rng = np.random.default_rng(seed)
    B, bs, cap = int(rng.integers(1, 40)), 16, 64
    cfg = KVCacheConfig(num_layers=1, num_kv_heads=1, head_dim=16, block_size=bs, total_gpu_blocks=B * 40,
                        enable_prefix_caching=False, max_supported_batch_size=256, max_blocks_per_sequence=cap)
    cache = PagedKVCache(cfg, allocate_pools=False)
    ids = list(range(100, 100 + B))
    for s in ids:
        cache.register_sequence_with_prefix(s, rng.integers(0, 99, size=int(rng.integers(1, 70))).tolist())
    cache.unregister_sequence(ids[0])  # a non-trivial free stack
    cache.register_sequence_with_prefix(ids[0], [1, 2, 3])
    dev = torch.device("cuda")
    dt = DeviceTables(cache, ids, cap, dev)
    ctx = torch.zeros(B, dtype=torch.int32, device=dev)
    dt.upload(ctx)
    for step in range(30):
        na = torch.tensor(rng.integers(-1, 6, size=B), dtype=torch.int32, device=dev)  # num_accepted (-1: bad draft)
        dt.append(na, ctx, 1)
        ctx += na.clamp_min(0) + 1
        dt.record(na, 1)
    dt.sync()
    torch.cuda.synchronize()
    assert torch.equal(dt.tables.cpu(), _host_tables(cache, ids, cap))
    ref_ctx = torch.zeros(B, dtype=torch.int32)
    cache.prepare_batch_into(ids, torch.zeros(B * cap, dtype=torch.int32), ref_ctx)
    assert torch.equal(ctx.cpu(), ref_ctx)
    import ctypes
    n = ctypes.c_uint32(0)
    host = torch.zeros(cfg.total_gpu_blocks, dtype=torch.int32)
    _lib.lib().cf_kvcache_export_free_stack(cache._h, host.data_ptr(), cfg.total_gpu_blocks, ctypes.byref(n))
    assert int(dt.free_top.item()) == n.value
    assert torch.equal(dt.free_stack[: n.value].cpu(), host[: n.value])


def test_device_growth_pool_exhausted_changes_nothing():
    B, bs, cap = 4, 16, 16
    cfg = KVCacheConfig(num_layers=1, num_kv_heads=1, head_dim=16, block_size=bs, total_gpu_blocks=9,
                        enable_prefix_caching=False, max_blocks_per_sequence=cap)
    cache = PagedKVCache(cfg, allocate_pools=False)
    ids = [0, 1, 2, 3]
    for s in ids:
        cache.register_sequence_with_prefix(s, list(range(16)))  # exactly one full block each
    dev = torch.device("cuda")
    dt = DeviceTables(cache, ids, cap, dev)
    ctx = torch.zeros(B, dtype=torch.int32, device=dev)
    dt.upload(ctx)
    before = (dt.tables.clone(), dt.table_len.clone(), int(dt.free_top.item()))
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    dt.append(torch.full((B,), 40, dtype=torch.int32, device=dev), ctx, 1, status=st)  # 3 blocks each: 12 > 5
    torch.cuda.synchronize()
    assert st.item() == _lib.CF_ENOMEM
    assert torch.equal(dt.tables, before[0]) and torch.equal(dt.table_len, before[1])
    assert int(dt.free_top.item()) == before[2]


def test_verifier_device_tables_matches_host_tables():
    from cudaforge_b200.model import LlamaConfig, LlamaModel
    from cudaforge_b200.verifier import BatchVerifier
    cfg = LlamaConfig(2, 512, 8, 2, 128, 768, 2048)
    m = LlamaModel(cfg, seed=8)
    B, K, P = 5, 4, 29
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, cfg.vocab, (B, P), generator=g)
    vs = []
    for dev_tab in (False, True):
        cache = m.make_cache(B * 12, max_batch=B)
        v = BatchVerifier(m, cache, list(range(B)), K, max_blocks_per_seq=10, use_graph=True, device_tables=dev_tab)
        v.register_context(prompts[:, :-1].tolist(), prompts[:, -1])
        v.fill_synthetic_kv(torch.Generator(device="cuda").manual_seed(2))
        vs.append(v)
    gd = torch.Generator(device="cuda").manual_seed(3)
    dlog = torch.randn(B, K, cfg.vocab, generator=gd, device="cuda").to(cfg.dtype)
    for step in range(7):
        dtok = torch.randint(0, cfg.vocab, (B, K), generator=gd, device="cuda", dtype=torch.int32)
        u = torch.rand(B, K + 1, generator=gd, device="cuda") * 0.05
        outs = []
        for v in vs:
            r = v.step(dtok, dlog, u)
            torch.cuda.synchronize()
            outs.append((r.num_accepted.cpu().clone(), r.tokens.cpu().clone(), v.tables().cpu().clone(),
                         v.ctx.cpu().clone()))
        a, b = outs
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]), step
        assert torch.equal(a[2], b[2]) and torch.equal(a[3], b[3]), step
    vs[1].check_status()
    assert vs[1].graphs is not None and vs[1].graphs[1] is None  # one graph per step
    assert vs[0].ctx_host == vs[1].ctx_host
    assert torch.equal(_host_tables(vs[0].cache, list(range(B)), 10), _host_tables(vs[1].cache, list(range(B)), 10))
    for pa, pb in ((vs[0].cache.key_pool, vs[1].cache.key_pool), (vs[0].cache.value_pool, vs[1].cache.value_pool)):
        assert torch.equal(pa, pb)
