"""CPU: page-table parity of cudaforge_b200.kv_cache.PagedKVCache with the
UNMODIFIED reference PagedKVCache (compiled from its sources into
oracle/_ref/ with a host-memory CUDA runtime).  Random interleavings of
register (with shared prefixes), append (1..K+1 tokens, the commit pattern of
a speculative step), fork, unregister and batch preparation must leave
identical block tables, context lengths and statistics, including pool
exhaustion and LRU eviction of cached prefix blocks."""
import numpy as np
import pytest

import oracle
from cudaforge_b200.kv_cache import KVCacheConfig, OutOfPagesException, PagedKVCache

pytestmark = pytest.mark.skipif(not oracle.RefKV.available(), reason="reference KV build absent")


def _pair(total, prefix=True, bs=16, max_batch=256, max_blocks=512):
    cfg = KVCacheConfig(num_layers=2, num_kv_heads=2, head_dim=8, block_size=bs, total_gpu_blocks=total,
                        enable_prefix_caching=prefix, max_supported_batch_size=max_batch,
                        max_blocks_per_sequence=max_blocks)
    return PagedKVCache(cfg, allocate_pools=False), oracle.RefKV(2, 2, 8, bs, total, prefix, max_batch, max_blocks)


def _stats(ours):
    s = ours.get_stats()
    return [s.total_blocks, s.free_blocks, s.allocated_blocks, s.cached_prefix_blocks,
            s.active_sequences_count, s.prefix_cache_hits, s.prefix_cache_misses, s.lru_evictions_count]


@pytest.mark.parametrize("seed", range(12))
@pytest.mark.parametrize("prefix", [True, False])
def test_random_interleavings_match_reference(seed, prefix):
    rng = np.random.default_rng(seed)
    total = int(rng.integers(8, 200))
    ours, ref = _pair(total, prefix)
    prompts = [rng.integers(0, 50, size=int(rng.integers(0, 80))).tolist() for _ in range(6)]
    live = []
    next_id = 1
    for step in range(300):
        op = rng.random()
        if op < 0.3 or not live:
            p = list(prompts[int(rng.integers(0, len(prompts)))])
            if rng.random() < 0.5:
                p = p + rng.integers(0, 50, size=int(rng.integers(0, 40))).tolist()
            rc, m = ref.register(next_id, p)
            try:
                m2 = ours.register_sequence_with_prefix(next_id, p)
                assert rc == 0 and m == m2
            except OutOfPagesException:
                assert rc == -5
            if rc == 0:
                live.append(next_id)
            next_id += 1
        elif op < 0.7:
            s = live[int(rng.integers(0, len(live)))]
            n = int(rng.integers(1, 7))
            rc = ref.append(s, n)
            try:
                ours.append_tokens(s, n)
                assert rc == 0
            except OutOfPagesException:
                assert rc == -5
        elif op < 0.8:
            s = live[int(rng.integers(0, len(live)))]
            assert ref.fork(s, next_id) == 0
            ours.fork_sequence(s, next_id)
            live.append(next_id)
            next_id += 1
        else:
            s = live.pop(int(rng.integers(0, len(live))))
            ref.unregister(s)
            ours.unregister_sequence(s)
        for s in live:
            assert ours.get_block_table(s) == ref.table(s)[1]
        assert _stats(ours) == ref.stats()
        if live and step % 10 == 0:
            rc, tab, ctx = ref.prepare(live)
            t2, c2 = ours.prepare_batch_host(live)
            assert rc == 0 and (t2.numpy() == tab).all() and (c2.numpy() == ctx).all()


def test_reference_cpp_known_answer_context_lens():
    # tests/cpp/test_paged_kv_cache.cpp:39-74: prompts of 32 and 48 tokens
    ours, ref = _pair(64)
    ours.register_sequence_with_prefix(1, list(range(32)))
    ours.register_sequence_with_prefix(2, list(range(100, 148)))
    tables, ctx = ours.prepare_batch_host([1, 2])
    assert ctx.tolist() == [32, 48] and tables.shape[1] == 3
    assert tables[0, 2].item() == -1


def test_first_blocks_and_exact_multiple_tail():
    ours, _ = _pair(10)
    # LIFO initialised N-1..0 -> first allocations return 0, 1, 2
    ours.register_sequence_with_prefix(1, list(range(20)))
    assert ours.get_block_table(1) == [0, 1]
    # a prompt that is an exact multiple of the block size gets no tail block
    ours.register_sequence_with_prefix(2, list(range(200, 216)))
    assert ours.get_block_table(2) == [2]
    ours.append_tokens(2, 1)
    assert ours.get_block_table(2) == [2, 3]


def test_unknown_sequence_and_batch_limits():
    ours, _ = _pair(10, max_batch=2)
    with pytest.raises(RuntimeError):
        ours.append_tokens(99, 1)
    for i in range(3):
        ours.register_sequence_with_prefix(i, [1])
    with pytest.raises(RuntimeError):
        ours.prepare_batch_host([0, 1, 2])
