"""GPU: verify attention, KV commit and the fused elementwise kernels against
the torch fp32 restatement (oracle/llama_ref.py).  Attention tolerance:
max-abs 2e-2 on O(1) outputs (bf16 inputs, fp32 accumulation); commit and
embedding are bit-exact copies."""
import pytest
import torch

from cudaforge_b200 import ops
from cudaforge_b200.kv_cache import KVCacheConfig, PagedKVCache
from oracle import llama_ref

pytestmark = pytest.mark.gpu


def _cache(L, Hkv, D, blocks, dtype=torch.bfloat16, seed=0):
    cfg = KVCacheConfig(num_layers=L, num_kv_heads=Hkv, head_dim=D, block_size=16, total_gpu_blocks=blocks,
                        enable_prefix_caching=False)
    c = PagedKVCache(cfg, dtype=dtype)
    g = torch.Generator(device="cuda").manual_seed(seed)
    c.key_pool.copy_(torch.randn(c.key_pool.shape, generator=g, device="cuda").to(dtype))
    c.value_pool.copy_(torch.randn(c.value_pool.shape, generator=g, device="cuda").to(dtype))
    return c


def _pool5(c):
    cfg = c.get_config()
    shp = (cfg.total_gpu_blocks, cfg.num_layers, cfg.num_kv_heads, cfg.block_size, cfg.head_dim)
    return c.key_pool.view(shp), c.value_pool.view(shp)


@pytest.mark.parametrize("D,Hq,Hkv,R", [(128, 32, 8, 6), (128, 8, 1, 5), (64, 8, 8, 5), (128, 32, 8, 65), (64, 4, 4, 17)])
@pytest.mark.parametrize("splits", [0, 1, 3])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_verify_attention_chain(D, Hq, Hkv, R, splits, dtype):
    L, B = 3, 5
    ctxs = [0, 1, 16, 37, 300][:B]
    c = _cache(L, Hkv, D, 80, dtype)
    for i, n in enumerate(ctxs):
        c.register_sequence_with_prefix(i, list(range(n)))
    tables, ctx = c.prepare_batch_metadata(list(range(B)))
    g = torch.Generator(device="cuda").manual_seed(1)
    q = torch.randn(B * R, Hq * D, generator=g, device="cuda").to(dtype)
    kn = torch.randn(B, R, Hkv, D, generator=g, device="cuda").to(dtype)
    vn = torch.randn(B, R, Hkv, D, generator=g, device="cuda").to(dtype)
    layer = 1
    out = ops.verify_attention(c, layer, q, kn, vn, tables, ctx, max(ctxs), rows=R, num_q_heads=Hq, num_splits=splits)
    torch.cuda.synchronize()
    kp, vp = _pool5(c)
    ref = llama_ref.verify_attention(q.view(B, R, Hq, D), kp, vp, layer, tables.cpu(), ctx.cpu(), kn, vn)
    err = (out.view(B, R, Hq, D).float() - ref).abs().max().item()
    assert err < 2e-2, err


@pytest.mark.parametrize("splits", [0, 2])
def test_verify_attention_tree_mask(splits):
    D, Hq, Hkv, R, B, L = 128, 32, 8, 65, 3, 2
    c = _cache(L, Hkv, D, 100)
    ctxs = [100, 4, 257]
    for i, n in enumerate(ctxs):
        c.register_sequence_with_prefix(i, list(range(n)))
    tables, ctx = c.prepare_batch_metadata(list(range(B)))
    # random tree: parent[j] < j, node 0 = root; mask = ancestors + self
    g = torch.Generator().manual_seed(3)
    mask = torch.zeros(B, R, R, dtype=torch.bool)
    for b in range(B):
        par = [-1] + [int(torch.randint(0, j, (1,), generator=g)) for j in range(1, R)]
        for j in range(R):
            k = j
            while k >= 0:
                mask[b, j, k] = True
                k = par[k]
    words = torch.zeros(B, R, 2, dtype=torch.int64)
    for j in range(R):
        bit = torch.tensor(1 << (j % 64), dtype=torch.int64) if j % 64 != 63 else torch.tensor(-(1 << 63), dtype=torch.int64)
        words[:, :, j // 64] |= torch.where(mask[:, :, j], bit, torch.zeros((), dtype=torch.int64))
    gq = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn(B * R, Hq * D, generator=gq, device="cuda").to(torch.bfloat16)
    kn = torch.randn(B, R, Hkv, D, generator=gq, device="cuda").to(torch.bfloat16)
    vn = torch.randn(B, R, Hkv, D, generator=gq, device="cuda").to(torch.bfloat16)
    out = ops.verify_attention(c, 0, q, kn, vn, tables, ctx, max(ctxs), rows=R, num_q_heads=Hq,
                               tree_mask=words.cuda(), num_splits=splits)
    torch.cuda.synchronize()
    kp, vp = _pool5(c)
    ref = llama_ref.verify_attention(q.view(B, R, Hq, D), kp, vp, 0, tables.cpu(), ctx.cpu(), kn, vn,
                                     tree_mask=mask.cuda())
    assert (out.view(B, R, Hq, D).float() - ref).abs().max().item() < 2e-2


@pytest.mark.parametrize("qscale", [1.0, 6.0])
def test_verify_attention_tcgen05_wide_tree(qscale):
    """>= 128 rows per kv head (65 tree rows x 4 heads) take the tcgen05 path
    (attention_tc.cu): long contexts (several 128-key blocks, ring wrap-around,
    partial last blocks, an empty context), a random tree mask, and scaled-up
    queries that force the lazy running-max rescale of O.  Checked against the
    fp32 restatement and against the warp-MMA kernel (selected by an explicit
    KV split)."""
    D, Hq, Hkv, R, L = 128, 32, 8, 65, 2
    ctxs = [1500, 129, 0, 2048]
    B = len(ctxs)
    c = _cache(L, Hkv, D, sum((n + R) // 16 + 2 for n in ctxs) + 8, seed=5)
    for i, n in enumerate(ctxs):
        c.register_sequence_with_prefix(i, list(range(n)))
    tables, ctx = c.prepare_batch_metadata(list(range(B)))
    g = torch.Generator().manual_seed(11)
    mask = torch.zeros(B, R, R, dtype=torch.bool)
    for b in range(B):
        par = [-1] + [int(torch.randint(0, j, (1,), generator=g)) for j in range(1, R)]
        for j in range(R):
            k = j
            while k >= 0:
                mask[b, j, k] = True
                k = par[k]
    bits = (mask.to(torch.int64) << torch.arange(64).repeat(2)[:R].view(1, 1, R))  # bit j % 64
    words = torch.stack([bits[..., :64].sum(-1), bits[..., 64:].sum(-1)], -1)
    gq = torch.Generator(device="cuda").manual_seed(12)
    q = (torch.randn(B * R, Hq * D, generator=gq, device="cuda") * qscale).to(torch.bfloat16)
    kn = torch.randn(B, R, Hkv, D, generator=gq, device="cuda").to(torch.bfloat16)
    vn = torch.randn(B, R, Hkv, D, generator=gq, device="cuda").to(torch.bfloat16)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    kw = dict(rows=R, num_q_heads=Hq, tree_mask=words.cuda(), status=st)
    out = ops.verify_attention(c, 1, q, kn, vn, tables, ctx, max(ctxs), **kw).clone()
    old = ops.verify_attention(c, 1, q, kn, vn, tables, ctx, max(ctxs), num_splits=2, **kw)
    torch.cuda.synchronize()
    assert st.item() == 0
    kp, vp = _pool5(c)
    ref = llama_ref.verify_attention(q.view(B, R, Hq, D), kp, vp, 1, tables.cpu(), ctx.cpu(), kn, vn,
                                     tree_mask=mask.cuda())
    err = (out.view(B, R, Hq, D).float() - ref).abs().max().item()
    err_old = (old.view(B, R, Hq, D).float() - ref).abs().max().item()
    print(f"tcgen05 tree attention max-abs {err:.3e} (warp-MMA kernel {err_old:.3e})")
    assert err < 2e-2 and err_old < 2e-2


def test_kv_commit_chain_and_tree():
    L, Hkv, D, B, R = 3, 2, 128, 4, 6
    c = _cache(L, Hkv, D, 40)
    ctxs = [0, 15, 16, 33]
    for i, n in enumerate(ctxs):
        c.register_sequence_with_prefix(i, list(range(n)))
    n_acc = torch.tensor([5, 0, 2, 3], dtype=torch.int32)
    for i in range(B):  # host commit of n_acc + 1 tokens in batch order
        c.append_tokens(i, int(n_acc[i]) + 1)
    tables, _ = c.prepare_batch_metadata(list(range(B)))
    g = torch.Generator(device="cuda").manual_seed(5)
    kn = torch.randn(L, B, R, Hkv, D, generator=g, device="cuda").to(torch.bfloat16)
    vn = torch.randn(L, B, R, Hkv, D, generator=g, device="cuda").to(torch.bfloat16)
    row_index = torch.tensor([[0, 2, 3, 5, 1, 4]] * B, dtype=torch.int32).cuda()
    for ri in (None, row_index):
        ops.kv_commit(c, kn, vn, n_acc.cuda(), torch.tensor(ctxs, dtype=torch.int32).cuda(), tables,
                      n_commit_add=1, row_index=ri)
        torch.cuda.synchronize()
        kp, vp = _pool5(c)
        for b in range(B):
            for j in range(int(n_acc[b]) + 1):
                pos = ctxs[b] + j
                blk = int(tables[b, pos // 16])
                src = j if ri is None else int(row_index[b, j])
                assert torch.equal(kp[blk, :, :, pos % 16], kn[:, b, src])
                assert torch.equal(vp[blk, :, :, pos % 16], vn[:, b, src])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_elementwise(dtype):
    g = torch.Generator(device="cuda").manual_seed(7)
    M, d, V = 37, 512, 1000
    tab = torch.randn(V, d, generator=g, device="cuda").to(dtype)
    ids = torch.randint(0, V, (M,), generator=g, device="cuda", dtype=torch.int32)
    e = ops.embedding(ids, tab)
    assert torch.equal(e, tab[ids.long()])
    w = torch.randn(d, generator=g, device="cuda").to(dtype)
    y = ops.rmsnorm(e, w)
    assert (y.float() - llama_ref.rmsnorm(e, w)).abs().max().item() < 3e-2
    Hq, Hkv, D = 8, 2, 64
    qkv = torch.randn(M, (Hq + 2 * Hkv) * D, generator=g, device="cuda").to(dtype)
    pos = torch.randint(0, 4096, (M,), generator=g, device="cuda", dtype=torch.int32)
    kn = torch.empty(M, Hkv, D, dtype=dtype, device="cuda")
    vn = torch.empty_like(kn)
    orig = qkv.clone()
    ops.rope_qkv(qkv, pos, Hq, Hkv, D, kn, vn)
    rq = llama_ref.rope(orig[:, : Hq * D].view(M, Hq, D).float(), pos.view(M, 1))
    rk = llama_ref.rope(orig[:, Hq * D:(Hq + Hkv) * D].view(M, Hkv, D).float(), pos.view(M, 1))
    tol = 2e-2 if dtype == torch.bfloat16 else 4e-3
    assert (qkv[:, : Hq * D].view(M, Hq, D).float() - rq).abs().max().item() < tol * 4
    assert (kn.float() - rk).abs().max().item() < tol * 4
    assert torch.equal(vn.view(M, -1), orig[:, (Hq + Hkv) * D:])
    F = 1408
    gu = torch.randn(M, 2 * F, generator=g, device="cuda").to(dtype)
    h = ops.silu_mul(gu, F)
    ref = torch.nn.functional.silu(gu[:, :F].float()) * gu[:, F:].float()
    assert (h.float() - ref).abs().max().item() < tol * 4
