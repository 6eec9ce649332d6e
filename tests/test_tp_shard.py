"""CPU: tensor-parallel sharding of the Llama projections.

The shards a rank keeps must tile the single-GPU model of the same seed:
column-parallel shards (QKV heads, gate|up features, vocabulary) select the
right output features, row-parallel shards (O, down) the right input
features, and the all-reduce of the row-parallel partial products (emulated
with gloo ranks over the fp32 restatement) reproduces the unsharded
projection."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cudaforge_b200.model import (LlamaConfig, LlamaModel, TensorParallel, linear_weight_fp32, tp_local_config)

CFG = LlamaConfig(2, 256, 8, 4, 64, 512, 1024)          # INT4
CFG_DENSE = LlamaConfig(2, 256, 8, 4, 64, 512, 1024, quant="dense", dtype=torch.float16)


@pytest.mark.parametrize("cfg", [CFG, CFG_DENSE], ids=["int4", "dense"])
@pytest.mark.parametrize("size", [2, 4])
def test_shards_tile_the_full_model(cfg, size):
    full = LlamaModel(cfg, device="cpu", seed=5)
    lc = tp_local_config(cfg, size)
    D = cfg.head_dim
    for r in range(size):
        m = LlamaModel(cfg, device="cpu", seed=5, tp=TensorParallel(r, size))
        assert m.lcfg == lc
        for li in range(cfg.layers):
            F = {k: linear_weight_fp32(full.layers[li][k]) for k in ("qkv", "o", "gate_up", "down")}
            S = {k: linear_weight_fp32(m.layers[li][k]) for k in ("qkv", "o", "gate_up", "down")}
            hq, hk = lc.n_heads, lc.n_kv_heads
            q = F["qkv"][r * hq * D:(r + 1) * hq * D]
            k0 = cfg.n_heads * D
            k = F["qkv"][k0 + r * hk * D:k0 + (r + 1) * hk * D]
            v0 = k0 + cfg.n_kv_heads * D
            v = F["qkv"][v0 + r * hk * D:v0 + (r + 1) * hk * D]
            assert torch.equal(S["qkv"], torch.cat([q, k, v]))
            f = lc.ffn
            assert torch.equal(S["gate_up"], torch.cat([F["gate_up"][r * f:(r + 1) * f],
                                                        F["gate_up"][cfg.ffn + r * f:cfg.ffn + (r + 1) * f]]))
            assert torch.equal(S["o"], F["o"][:, r * hq * D:(r + 1) * hq * D])
            assert torch.equal(S["down"], F["down"][:, r * f:(r + 1) * f])
        lm = linear_weight_fp32(m.lm_head)
        vl = cfg.vocab // size
        assert lm.shape[0] % 128 == 0 and lm.shape[0] >= vl
        assert torch.equal(lm[:vl], linear_weight_fp32(full.lm_head)[r * vl:(r + 1) * vl])
        assert not lm[vl:].any()  # padded output features are exact zeros
        assert torch.equal(m.embed, full.embed)


def _rank_main(rank, size, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=size)
    try:
        cfg = CFG
        m = LlamaModel(cfg, device="cpu", seed=9, tp=TensorParallel(rank, size))
        full = LlamaModel(cfg, device="cpu", seed=9)
        g = torch.Generator().manual_seed(1)
        x = torch.randn(6, cfg.n_heads * cfg.head_dim, generator=g)
        h = torch.randn(6, cfg.d_model, generator=g)
        D, hq = cfg.head_dim, cfg.n_heads // size
        # O projection: this rank's heads only, rank 0 adds the residual, then all-reduce
        part = x[:, rank * hq * D:(rank + 1) * hq * D] @ linear_weight_fp32(m.layers[0]["o"]).T
        if rank == 0:
            part = part + h
        dist.all_reduce(part)
        ref = h + x @ linear_weight_fp32(full.layers[0]["o"]).T
        out[rank] = float((part - ref).abs().max())
    finally:
        dist.destroy_process_group()


def test_row_parallel_all_reduce_gloo():
    size = 2
    out = mp.Manager().dict()
    mp.spawn(_rank_main, args=(size, 29517, out), nprocs=size, join=True)
    assert max(out.values()) < 1e-4
