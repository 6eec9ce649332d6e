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
