"""GPU (2 GPUs, NCCL): the tensor-parallel verify forward and step.

Each of 2 ranks holds half the heads / FFN features / vocabulary of a small
INT4 Llama; the verify logits (all-reduced residual stream, all-gathered
vocabulary) must match the fp32 restatement of the same-seed single-GPU model
within the model tests' tolerance, and a BatchVerifier step must give
identical acceptance results and page tables on both ranks."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

needs2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                            reason="needs 2 GPUs")


def _worker(rank, size, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=size, device_id=dev)
    try:
        from cudaforge_b200.model import LlamaConfig, LlamaModel, TensorParallel
        from cudaforge_b200.runner import PagedRunner
        from cudaforge_b200.verifier import BatchVerifier
        from oracle import llama_ref

        cfg = LlamaConfig(2, 512, 8, 2, 128, 768, 2000)  # vocab shard 1000 -> padded to 1024
        m = LlamaModel(cfg, device=dev, seed=4, tp=TensorParallel(rank, size))
        B, S0, K = 3, 21, 4
        g = torch.Generator().manual_seed(2)
        prompt = torch.randint(0, cfg.vocab, (B, S0), generator=g)
        drafts = torch.randint(0, cfg.vocab, (B, K), generator=g)
        runner = PagedRunner(m, m.make_cache(32), seq_ids=[0, 1, 2])
        runner.prefill(prompt[:, :-1].tolist())
        ids = torch.cat([prompt, drafts], 1)
        logits = runner.forward(ids).float()
        torch.cuda.synchronize()
        res = {"status": int(runner.status.item())}
        if rank == 0:
            full = LlamaModel(cfg, device=dev, seed=4)
            ref = llama_ref.forward_full(full, ids.to(dev))[:, -(K + 1):]
            scale = max(1.0, ref.abs().max().item())
            res["err"] = (logits - ref).abs().max().item() / scale
            top2 = ref.topk(2, dim=-1).values
            clear = (top2[..., 0] - top2[..., 1]) > 2e-2 * scale
            res["agree"] = bool((logits.argmax(-1) == ref.argmax(-1))[clear].all())
        # a device-resident verify + accept + commit step, identical on both ranks
        cache = m.make_cache(64, max_batch=B)
        ver = BatchVerifier(m, cache, [0, 1, 2], K)
        ver.register_context(prompt[:, :-1].tolist(), prompt[:, -1])
        ver.fill_synthetic_kv(torch.Generator(device=dev).manual_seed(3))
        dl = torch.randn(B, K, cfg.vocab, generator=torch.Generator(device=dev).manual_seed(5), device=dev)
        u = torch.rand(B, K + 1, generator=torch.Generator(device=dev).manual_seed(6), device=dev)
        r = ver.step(drafts.to(dev, torch.int32), dl.to(cfg.dtype), u)
        torch.cuda.synchronize()
        res["n"] = r.num_accepted.cpu().tolist()
        res["tok"] = r.tokens.cpu().tolist()
        res["tables"] = ver.tables().cpu().tolist()
        # two micro-batches on two streams (one NCCL group each) == one batch, over 3 steps
        B2 = 4
        g2 = torch.Generator().manual_seed(8)
        prompt2 = torch.randint(0, cfg.vocab, (B2, S0), generator=g2)
        outs = []
        for mb in (1, 2):
            cache2 = m.make_cache(64, max_batch=B2)
            v2 = BatchVerifier(m, cache2, list(range(B2)), K, micro_batches=mb)
            v2.register_context(prompt2[:, :-1].tolist(), prompt2[:, -1])
            v2.fill_synthetic_kv(torch.Generator(device=dev).manual_seed(3))
            gd = torch.Generator(device=dev).manual_seed(9)
            steps = []
            for _ in range(3):
                dt2 = torch.randint(0, cfg.vocab, (B2, K), generator=gd, device=dev, dtype=torch.int32)
                dl2 = torch.randn(B2, K, cfg.vocab, generator=gd, device=dev).to(cfg.dtype)
                u2 = torch.rand(B2, K + 1, generator=gd, device=dev) * 0.05
                r2 = v2.step(dt2, dl2, u2)
                torch.cuda.synchronize()
                steps.append((r2.num_accepted.cpu().tolist(), r2.tokens.cpu().tolist()))
            outs.append((v2.mb, steps, v2.tables().cpu().tolist(), cache2.key_pool.float().sum().item()))
        res["mb_used"] = outs[1][0]
        res["mb_equal"] = outs[0][1:] == outs[1][1:]
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


@needs2
def test_tp2_forward_and_step():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, 29611, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert out[0]["status"] == 0 and out[1]["status"] == 0
    assert out[0]["err"] <= 2e-2, out[0]["err"]
    assert out[0]["agree"]
    for key in ("n", "tok", "tables"):
        assert out[0][key] == out[1][key], key
    assert out[0]["mb_used"] == 2 and out[0]["mb_equal"] and out[1]["mb_equal"]
