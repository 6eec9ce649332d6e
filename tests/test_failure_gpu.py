"""GPU: the failure paths, driven without faulting the GPU.

Every mbarrier wait in the GEMM and attention kernels is bounded: when the
limit runs out the kernel records CF_ETIMEOUT in the caller's status word,
lets its own copies land, frees TMEM and returns, so the context stays
usable.  These tests make the waits run out with a 1 ns limit (nothing the
kernel waits for can arrive that fast), check the status word, and then
check that the next normal call on the same context is correct.  Invalid
page ids and negative positions record CF_ERANGE instead of touching memory
outside the pools.  The host layers (BatchVerifier, DeviceStatus) turn a
non-zero status word into DeviceError."""
import pytest
import torch

from cudaforge_b200 import _lib, ops
from cudaforge_b200.gemm import pack_int4_reference, repack_int4, w4a16_gemm
from cudaforge_b200.kv_cache import KVCacheConfig, PagedKVCache

pytestmark = pytest.mark.gpu


def _cache(L=2, Hkv=8, D=128, blocks=200, seed=0):
    cfg = KVCacheConfig(num_layers=L, num_kv_heads=Hkv, head_dim=D, block_size=16, total_gpu_blocks=blocks,
                        enable_prefix_caching=False)
    c = PagedKVCache(cfg, dtype=torch.bfloat16)
    g = torch.Generator(device="cuda").manual_seed(seed)
    c.key_pool.copy_(torch.randn(c.key_pool.shape, generator=g, device="cuda").to(torch.bfloat16))
    c.value_pool.copy_(torch.randn(c.value_pool.shape, generator=g, device="cuda").to(torch.bfloat16))
    return c


def test_gemm_wait_timeout_then_normal_call():
    M, N, K = 384, 6144, 4096
    g = torch.Generator().manual_seed(3)
    wq = repack_int4(pack_int4_reference(torch.randint(0, 16, (K, N), generator=g)).cuda())
    sc = (torch.randn(K // 128, N, generator=g).abs() * 0.002).half().cuda()
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    good = w4a16_gemm(x, wq, sc, status=st).clone()
    torch.cuda.synchronize()
    assert st.item() == _lib.CF_OK
    for split in (0, 1):
        w4a16_gemm(x, wq, sc, status=st, timeout_ns=1, split_k=split)
        torch.cuda.synchronize()
        assert st.item() == _lib.CF_ETIMEOUT
        st.zero_()
    again = w4a16_gemm(x, wq, sc, status=st)
    torch.cuda.synchronize()
    assert st.item() == _lib.CF_OK
    assert torch.equal(again, good)


def _attn_inputs(c, B=4, R=6, Hq=32, ctxs=(300, 1000, 17, 640)):
    for i, n in enumerate(ctxs[:B]):
        c.register_sequence_with_prefix(i, list(range(n)))
    tables, ctx = c.prepare_batch_metadata(list(range(B)))
    g = torch.Generator(device="cuda").manual_seed(1)
    D, Hkv = c.get_config().head_dim, c.get_config().num_kv_heads
    q = torch.randn(B * R, Hq * D, generator=g, device="cuda").to(torch.bfloat16)
    kn = torch.randn(B, R, Hkv, D, generator=g, device="cuda").to(torch.bfloat16)
    vn = torch.randn(B, R, Hkv, D, generator=g, device="cuda").to(torch.bfloat16)
    return tables, ctx, q, kn, vn, max(ctxs[:B])


def test_attention_wait_timeout_then_normal_call():
    c = _cache()
    tables, ctx, q, kn, vn, mx = _attn_inputs(c)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    kw = dict(rows=6, num_q_heads=32, status=st)
    good = ops.verify_attention(c, 1, q, kn, vn, tables, ctx, mx, **kw).clone()
    torch.cuda.synchronize()
    assert st.item() == _lib.CF_OK
    for splits in (1, 3):
        ops.verify_attention(c, 1, q, kn, vn, tables, ctx, mx, num_splits=splits, timeout_ns=1, **kw)
        torch.cuda.synchronize()
        assert st.item() == _lib.CF_ETIMEOUT
        st.zero_()
    again = ops.verify_attention(c, 1, q, kn, vn, tables, ctx, mx, **kw)
    torch.cuda.synchronize()
    assert st.item() == _lib.CF_OK
    assert torch.equal(again, good)


def test_attention_bad_page_id_records_erange():
    c = _cache()
    tables, ctx, q, kn, vn, mx = _attn_inputs(c)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    good = ops.verify_attention(c, 0, q, kn, vn, tables, ctx, mx, rows=6, num_q_heads=32, status=st).clone()
    bad = tables.clone()
    bad[1, 3] = c.get_config().total_gpu_blocks + 7  # sequence 1 only
    out = ops.verify_attention(c, 0, q, kn, vn, bad, ctx, mx, rows=6, num_q_heads=32, status=st)
    torch.cuda.synchronize()
    assert st.item() == _lib.CF_ERANGE
    rows = out.view(4, 6, -1)
    ref = good.view(4, 6, -1)
    for b in (0, 2, 3):  # the other sequences are untouched by the bad id
        assert torch.equal(rows[b], ref[b])


def test_kv_commit_negative_start_records_erange():
    c = _cache(L=2, Hkv=8, D=128, blocks=40)
    B, R = 2, 4
    for i in range(B):
        c.register_sequence_with_prefix(i, list(range(40)))
    tables, ctx = c.prepare_batch_metadata(list(range(B)))
    kn = torch.randn(2, B, R, 8, 128, device="cuda").to(torch.bfloat16)
    vn = torch.randn_like(kn)
    kp, vp = c.key_pool.clone(), c.value_pool.clone()
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    n = torch.tensor([2, 2], dtype=torch.int32, device="cuda")
    start = torch.tensor([-3, -1], dtype=torch.int32, device="cuda")
    ops.kv_commit(c, kn, vn, n, start, tables, status=st)
    torch.cuda.synchronize()
    assert st.item() == _lib.CF_ERANGE
    # positions -3, -2 and -1 are refused; position 0 (the second row of sequence 1) is valid
    cfg = c.get_config()
    shp = (cfg.total_gpu_blocks, cfg.num_layers, cfg.num_kv_heads, cfg.block_size, cfg.head_dim)
    changed = (c.key_pool.view(shp) != kp.view(shp)).flatten(2).any(-1)  # [block, layer]
    blk0 = int(tables[1, 0])
    assert changed.nonzero().tolist() == [[blk0, 0], [blk0, 1]]
    assert torch.equal(c.value_pool.view(shp)[blk0, :, :, 1:], vp.view(shp)[blk0, :, :, 1:])


def test_device_status_raises_and_clears():
    st = _lib.DeviceStatus(torch.device("cuda"))
    st.dev.fill_(_lib.CF_ETIMEOUT)
    with pytest.raises(_lib.DeviceError) as e:
        st.sync_check("probe")
    assert e.value.code == _lib.CF_ETIMEOUT
    st.sync_check("probe")  # cleared: no error the second time


def test_verifier_step_raises_on_device_error():
    from cudaforge_b200.model import LlamaConfig, LlamaModel
    from cudaforge_b200.verifier import BatchVerifier
    cfg = LlamaConfig(2, 256, 4, 2, 64, 512, 1024)
    model = LlamaModel(cfg, seed=0)
    B, K = 3, 4
    cache = model.make_cache(64, max_batch=B, max_blocks_per_seq=16)
    ver = BatchVerifier(model, cache, list(range(B)), K, max_blocks_per_seq=16)
    ver.register_context([list(range(20))] * B, [1, 2, 3])
    ver.fill_synthetic_kv(torch.Generator(device="cuda").manual_seed(0))
    g = torch.Generator(device="cuda").manual_seed(1)
    dt = torch.randint(0, cfg.vocab, (B, K), generator=g, device="cuda", dtype=torch.int32)
    dl = torch.randn(B, K, cfg.vocab, generator=g, device="cuda").to(torch.bfloat16)
    u = torch.rand(B, K + 1, generator=g, device="cuda")
    ver.step(dt, dl, u)
    ctx_before = list(ver.ctx_host)
    ver.status.fill_(_lib.CF_ERANGE)  # as a kernel of the step would record it
    with pytest.raises(_lib.DeviceError):
        ver.step(dt, dl, u)
    assert ver.ctx_host == ctx_before  # the failed step committed nothing on the host
    ver.step(dt, dl, u)  # the status word was cleared; the next step runs
    ver.check_status()


def test_tree_attention_tcgen05_wait_timeout_and_bad_page():
    """The tcgen05 path (>= 128 rows per kv head: 65 tree rows x 4 heads): waits driven to
    expiry record CF_ETIMEOUT and the next call is correct; an invalid page id records
    CF_ERANGE and leaves the other sequences' outputs untouched."""
    c = _cache(L=2, Hkv=8, D=128, blocks=300)
    R, Hq = 65, 32
    tables, ctx, q, kn, vn, mx = _attn_inputs(c, B=3, R=R, Hq=Hq, ctxs=(300, 1000, 17))
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    kw = dict(rows=R, num_q_heads=Hq, status=st)
    good = ops.verify_attention(c, 1, q, kn, vn, tables, ctx, mx, **kw).clone()
    torch.cuda.synchronize()
    assert st.item() == _lib.CF_OK
    ops.verify_attention(c, 1, q, kn, vn, tables, ctx, mx, timeout_ns=1, **kw)
    torch.cuda.synchronize()
    assert st.item() == _lib.CF_ETIMEOUT
    st.zero_()
    again = ops.verify_attention(c, 1, q, kn, vn, tables, ctx, mx, **kw)
    torch.cuda.synchronize()
    assert st.item() == _lib.CF_OK
    assert torch.equal(again, good)
    bad = tables.clone()
    bad[1, 5] = c.get_config().total_gpu_blocks + 3  # sequence 1 only
    out = ops.verify_attention(c, 1, q, kn, vn, bad, ctx, mx, **kw)
    torch.cuda.synchronize()
    assert st.item() == _lib.CF_ERANGE
    rows, ref = out.view(3, R, -1), good.view(3, R, -1)
    for b in (0, 2):
        assert torch.equal(rows[b], ref[b])
