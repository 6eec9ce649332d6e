#!/usr/bin/env python
"""Benchmark: accepted tokens/s of the speculative verify + accept step on
the Llama-3-8B-shaped W4A16 target (batch 64 per GPU,
random 1024-token prompts, K=5 chain drafts from the 1B-shaped INT4 draft,
T=1.0, paged KV block 16).

A step = target verify forward over K+1 rows per sequence + fused acceptance
+ page-table commit and K/V commit (cudaforge_b200.BatchVerifier.step).  The
draft model (cudaforge_b200.BatchDrafter) drafts once before timing and its
cost is excluded from the metric; every step uses fresh uniforms.  A second
timed loop reports full rounds (draft loop + verify step + draft advance) as
`speculative_round`.  Requests are batch-sharded: each rank owns
64 sequences with its own weights, pools and page tables and no collective
(weak scaling).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "accepted tok/s of verify+accept at 8B-INT4"
UNIT = "tokens/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.idx = gpu_index
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower() == "active"})
        loaded = [r for r in rows if r[2] > 200.0] or rows
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------- timing helpers
class KernelTimer:
    """CUDA events around launch groups on the launching (current) stream."""

    def __init__(self):
        self.ev = {}

    def __call__(self, kind):
        timer = self

        class _C:
            def __enter__(self_):
                self_.a = torch.cuda.Event(enable_timing=True)
                self_.a.record()
                return self_

            def __exit__(self_, *exc):
                b = torch.cuda.Event(enable_timing=True)
                b.record()
                timer.ev.setdefault(kind, []).append((self_.a, b))
                return False

        return _C()

    def total_ms(self, kind):
        return sum(a.elapsed_time(b) for a, b in self.ev.get(kind, []))

    def count(self, kind):
        return len(self.ev.get(kind, []))


def fill_random(cache, gen: torch.Generator) -> None:
    """Seeded N(0,1) K/V in every pool slot, in chunks (no full-size fp32 temporary)."""
    for pool in (cache.key_pool, cache.value_pool):
        flat = pool.view(-1)
        for i in range(0, flat.numel(), 1 << 28):
            seg = flat[i: i + (1 << 28)]
            seg.copy_(torch.randn(seg.numel(), generator=gen, device=seg.device).to(seg.dtype))


def setup(args, rank, device, world=1):
    from cudaforge_b200.model import DRAFT_1B, LLAMA_8B, TINY_DRAFT, TINY_TARGET, LlamaModel
    from cudaforge_b200.runner import PagedRunner
    from cudaforge_b200.speculative import SpeculativeEngine
    from cudaforge_b200.verifier import BatchVerifier

    from cudaforge_b200.shard import rank_sequence_ids
    tcfg, dcfg = (LLAMA_8B, DRAFT_1B) if args.config == "8b" else (TINY_TARGET, TINY_DRAFT)
    B, P, K = args.batch, args.ctx, args.k
    steps_total = args.warmup + 3 * args.steps + 8
    blocks_per_seq = math.ceil((P + steps_total * (K + 1)) / 16) + 2
    ids = rank_sequence_ids(rank, B)  # global sequence ids of this rank's shard
    # every rank holds a replica of the same weights; the prompts are this rank's rows of one global set
    target = LlamaModel(tcfg, device=device, seed=1000)
    cache = target.make_cache(B * blocks_per_seq + 8, max_batch=B, max_blocks_per_seq=blocks_per_seq + 4)
    ver = BatchVerifier(target, cache, ids, K, temperature=args.temperature,
                        max_blocks_per_seq=blocks_per_seq + 4, use_graph=not args.no_graph,
                        device_tables=not args.host_tables)
    g = torch.Generator().manual_seed(7)
    prompts = torch.randint(0, tcfg.vocab, (B * world, P), generator=g)[ids[0]: ids[-1] + 1]
    ver.register_context(prompts[:, :-1].tolist(), prompts[:, -1])
    gd = torch.Generator(device=device).manual_seed(11 + rank)
    ver.fill_synthetic_kv(gd)
    # draft: the 1B-shaped INT4 model proposes K tokens per sequence through the device-resident
    # draft loop (its first round gives the drafts the verify steps reuse; rounds are timed separately)
    from cudaforge_b200.drafter import BatchDrafter
    draft = LlamaModel(dcfg, device=device, seed=2000)
    dcache = draft.make_cache(B * blocks_per_seq + 8, max_batch=B, max_blocks_per_seq=blocks_per_seq + 4)
    drafter = BatchDrafter(draft, dcache, ids, K, temperature=args.temperature,
                           max_blocks_per_seq=blocks_per_seq + 4, use_graph=not args.no_graph)
    drafter.register_context(prompts[:, :-1].tolist(), prompts[:, -1])
    fill_random(dcache, gd)
    du = torch.rand(B, K, generator=gd, device=device)
    draft_tokens, draft_logits = drafter.draft(du)
    return tcfg, target, cache, ver, draft_tokens.clone(), draft_logits.clone(), drafter


def setup_tp(args, rank, world, device):
    """cfg5: Llama-3-70B-shaped W4A16 target, tensor-parallel over the ranks
    (TP = world size; 1 rank holds the whole model), B=128, 2048-token
    contexts, K=4; drafts from an 8B-shaped INT4 draft replicated on every
    rank (same seed everywhere, untimed)."""
    from cudaforge_b200.model import LLAMA_8B, LLAMA_70B, LlamaModel, TensorParallel
    from cudaforge_b200.runner import PagedRunner
    from cudaforge_b200.speculative import SpeculativeEngine
    from cudaforge_b200.verifier import BatchVerifier

    tcfg, dcfg = LLAMA_70B, LLAMA_8B
    B, P, K = args.batch, args.ctx, args.k
    steps_total = args.warmup + 2 * args.steps + 4
    blocks_per_seq = math.ceil((P + steps_total * (K + 1)) / 16) + 2
    target = LlamaModel(tcfg, device=device, seed=1000, tp=TensorParallel(rank, world))
    cache = target.make_cache(B * blocks_per_seq + 8, max_batch=B, max_blocks_per_seq=blocks_per_seq + 4)
    ver = BatchVerifier(target, cache, list(range(B)), K, temperature=args.temperature,
                        max_blocks_per_seq=blocks_per_seq + 4, micro_batches=args.tp_microbatches)
    g = torch.Generator().manual_seed(7)
    prompts = torch.randint(0, tcfg.vocab, (B, P), generator=g)
    ver.register_context(prompts[:, :-1].tolist(), prompts[:, -1])
    gd = torch.Generator(device=device).manual_seed(11 + rank)
    ver.fill_synthetic_kv(gd)
    draft = LlamaModel(dcfg, device=device, seed=2000)
    dcache = draft.make_cache(B * (math.ceil((P + K + 2) / 16) + 2) + 8, max_batch=B)
    dr = PagedRunner(draft, dcache, list(range(B)))
    dr.register(prompts[:, :-1].tolist())
    fill_random(dcache, torch.Generator(device=device).manual_seed(13))
    eng = SpeculativeEngine(dr, None, num_speculative_tokens=K, temperature=args.temperature, seed=3)
    eng.target_runner = dr  # device lookup only
    draft_tokens, draft_logits = eng.draft(prompts.tolist())
    del dr, dcache, draft
    torch.cuda.empty_cache()
    return tcfg, target, cache, ver, draft_tokens.contiguous(), draft_logits.contiguous()


def setup_tree(args, rank, device):
    """cfg4: the 8B-INT4 target verifies a 64-node top-k tree (4/4/4, breadth-first
    truncated) per sequence; the tree comes from the 1B draft (untimed)."""
    from cudaforge_b200.model import DRAFT_1B, LLAMA_8B, LlamaModel
    from cudaforge_b200.runner import PagedRunner
    from cudaforge_b200.tree import TreeSpeculativeEngine, TreeVerifier, topk_tree_shape

    tcfg, dcfg = LLAMA_8B, DRAFT_1B
    B, P = args.batch, args.ctx
    shape = topk_tree_shape((4, 4, 4), 64)
    steps_total = args.warmup + 2 * args.steps + 4
    blocks_per_seq = math.ceil((P + steps_total * 4) / 16) + 2
    target = LlamaModel(tcfg, device=device, seed=1000 + rank)
    cache = target.make_cache(B * blocks_per_seq + 8, max_batch=B, max_blocks_per_seq=blocks_per_seq + 4)
    ver = TreeVerifier(target, cache, list(range(B)), shape, temperature=args.temperature,
                       max_blocks_per_seq=blocks_per_seq + 4)
    g = torch.Generator().manual_seed(7 + rank)
    prompts = torch.randint(0, tcfg.vocab, (B, P), generator=g)
    ver.register_context(prompts[:, :-1].tolist(), prompts[:, -1])
    gd = torch.Generator(device=device).manual_seed(11 + rank)
    ver.fill_synthetic_kv(gd)
    draft = LlamaModel(dcfg, device=device, seed=2000 + rank)
    dcache = draft.make_cache(B * (math.ceil((P + 8) / 16) + 2) + 8, max_batch=B)
    dr = PagedRunner(draft, dcache, list(range(B)))
    dr.register(prompts[:, :-1].tolist())
    fill_random(dcache, gd)
    eng = TreeSpeculativeEngine(dr, dr, shape, temperature=args.temperature, seed=3 + rank)
    ttok, tlog = eng.draft_tree(prompts.tolist())
    del eng, dr, dcache, draft
    torch.cuda.empty_cache()
    return tcfg, target, cache, ver, ttok.contiguous(), tlog.contiguous()


def run_ours(args):
    import torch.distributed as dist

    from cudaforge_b200 import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    tree = args.config == "8b-tree"
    tp = args.config == "70b-tp"
    drafter = None
    if tp:
        tcfg, target, cache, ver, dtok, dlog = setup_tp(args, rank, world, device)
    elif tree:
        tcfg, target, cache, ver, dtok, dlog = setup_tree(args, rank, device)
    else:
        tcfg, target, cache, ver, dtok, dlog, drafter = setup(args, rank, device, world)
    B = args.batch
    R = dlog.shape[1] if tree else args.k + 1
    K = R - 1
    total_steps = args.warmup + args.steps
    gen = torch.Generator(device=device).manual_seed(99 + rank)
    uni = torch.rand(total_steps + args.steps + 1, B, K + 1, generator=gen, device=device)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    for i in range(args.warmup):
        ver.step(dtok, dlog, uni[i])
    barrier()
    # ---- timed region (device-resident inputs) ----
    clk = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ else local)
    clk.start()
    time.sleep(0.5)  # nvidia-smi's first sample takes a moment; the samples span every timed loop below
    tokens_per_step = []
    l0 = _lib.LAUNCHES[0]
    dev_tab = getattr(ver, "dtab", None) is not None
    if dev_tab:
        ver.sync()  # the warm-up steps' counts are replayed on the host before the timed region starts
    em0 = ver.dtab.emitted if dev_tab else 0
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    step_ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    e0.record()
    step_ev[0].record()
    for i in range(args.steps):
        res = ver.step(dtok, dlog, uni[args.warmup + i])
        step_ev[i + 1].record()
        if not dev_tab:  # host tables: the step already synchronised for its counts
            tokens_per_step.append(int((ver.n_pinned.clamp_min(0) + 1).sum()))
    e1.record()
    barrier()
    ver.check_status()  # a timed-out wait or a bad page id voids the measurement
    if dev_tab:  # device tables: the host replayed the steps' counts lazily
        tokens_per_step = [(ver.dtab.emitted - em0) / args.steps] * args.steps
    launches = _lib.LAUNCHES[0] - l0
    ms = e0.elapsed_time(e1)
    step_ms = sorted(step_ev[i].elapsed_time(step_ev[i + 1]) for i in range(args.steps))
    # ---- per-kernel timing pass: the same step launched eagerly with CUDA events around every
    # launch group; a device-side sleep queued first keeps the GPU busy while the host enqueues
    # the step, so each event pair brackets device time only (no host launch gaps) ----
    kt = KernelTimer()
    kp = max(2, min(args.steps, 4))
    ctx_sums = []
    for i in range(kp):
        if hasattr(ver, "sync"):
            ver.sync()
        ctx_sums.append(sum(ver.ctx_host))  # context of the step's attention (before its commit)
        torch.cuda._sleep(60_000_000)  # ~30 ms of device time at 1.9 GHz
        ver.step(dtok, dlog, uni[total_steps + i], timer=kt)
    torch.cuda.synchronize(device)
    ver.check_status()
    # ---- e2e: host inputs (pinned) -> device, results -> host, every step ----
    h_tok = dtok.cpu().pin_memory()
    h_uni = uni[total_steps: total_steps + args.steps].cpu().pin_memory()
    h_out_tok = torch.empty(B, R, dtype=torch.int32).pin_memory()
    h_out_n = torch.empty(B, dtype=torch.int32).pin_memory()
    d_tok = torch.empty_like(dtok)
    d_uni = torch.empty(B, K + 1, device=device)
    barrier()
    x0 = torch.cuda.Event(enable_timing=True)
    x1 = torch.cuda.Event(enable_timing=True)
    x0.record()
    e2e_tokens = 0
    for i in range(args.steps):
        d_tok.copy_(h_tok, non_blocking=True)
        d_uni.copy_(h_uni[i], non_blocking=True)
        r = ver.step(d_tok, dlog, d_uni)
        h_out_tok.copy_(r.tokens, non_blocking=True)
        h_out_n.copy_(r.num_accepted, non_blocking=True)
        torch.cuda.current_stream(device).synchronize()
        e2e_tokens += int((h_out_n.clamp_min(0) + 1).sum())
    x1.record()
    barrier()
    ver.check_status()
    e2e_ms = x0.elapsed_time(x1)
    # the host gathers every rank's emitted tokens of the last e2e step (outside the timed regions)
    from cudaforge_b200.shard import gather_emitted
    nl = h_out_n.tolist()
    gathered = gather_emitted(ver.seq_ids, [h_out_tok[b, : max(0, nl[b]) + 1].tolist() for b in range(B)]) \
        if not tp else None
    h2d = dtok.numel() * 4 + B * R * 4
    d2h = B * R * 4 + B * 4

    # ---- full speculative rounds: draft loop (K steps of the 1B draft) + verify + accept + advance ----
    round_info = None
    if drafter is not None and not args.no_rounds:
        ud = torch.rand(args.steps + 2, B, K, generator=gen, device=device)
        for i in range(2):  # the drafter captures its graph on its second round
            dt_, dl_ = drafter.draft(ud[i])
            r = ver.step(dt_, dl_, uni[i])
            drafter.advance(r, (r.num_accepted.clamp_min(0) + 1).tolist())
        barrier()
        d_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        r0 = torch.cuda.Event(enable_timing=True)
        r1 = torch.cuda.Event(enable_timing=True)
        round_tokens = 0
        r0.record()
        for i in range(args.steps):
            d_ev[i][0].record()
            dt_, dl_ = drafter.draft(ud[2 + i])
            d_ev[i][1].record()
            r = ver.step(dt_, dl_, uni[i])
            n_host = (r.num_accepted.clamp_min(0) + 1).tolist()  # the draft tables grow on the host
            round_tokens += sum(n_host)
            drafter.advance(r, n_host)
        r1.record()
        barrier()
        ver.check_status()
        drafter.st.sync_check("BatchDrafter")
        round_ms = r0.elapsed_time(r1)
        draft_ms = sum(a.elapsed_time(b) for a, b in d_ev)
        round_info = [round_ms, draft_ms, float(round_tokens)]

    clocks = clk.stop()
    clocks["window"] = "headline, per-kernel, e2e and full-round timed loops"
    # max over ranks of the device times, sum of the emitted tokens (batch-sharded, no data-path collective)
    from cudaforge_b200.shard import reduce_step_metrics
    (ms_max, e2e_max), (tok_all, e2e_tok_all) = reduce_step_metrics(
        [ms, e2e_ms], [float(sum(tokens_per_step)), float(e2e_tokens)], device=device)
    if tp:  # every rank verifies the same batch: count its tokens once
        tok_all, e2e_tok_all = tok_all / world, e2e_tok_all / world
    value = tok_all / (ms_max / 1e3)
    round_out = None
    if round_info is not None:
        (rms, dms), (rtok,) = reduce_step_metrics(round_info[:2], round_info[2:], device=device)
        round_out = {"what": "full speculative round: device-resident draft loop (K steps of the 1B INT4 draft, "
                             "CUDA graph) + verify + accept + KV commit + draft advance, device-resident inputs",
                     "accepted_tok_s": round(rtok / (rms / 1e3), 1), "ms_per_round": round(rms / args.steps, 3),
                     "draft_ms_per_round": round(dms / args.steps, 3)}
    e2e_value = e2e_tok_all / (e2e_max / 1e3)

    # roofline of the dominant kernel (W4A16 GEMM, tensor bound) and the others
    peaks, peak_src = load_peaks()
    M = B * R
    gemm_flops = tcfg.gemm_flops(M) / (world if tp else 1)  # per rank
    kms = {k: kt.total_ms(k) / kp for k in ("gemm", "attn", "accept", "commit", "other", "comm")}
    gemm_ms, attn_ms = kms["gemm"], kms["attn"]
    achieved_tf = gemm_flops / (gemm_ms / 1e3) / 1e12
    # burst peak for kernels that ran at the maximum SM clock (a short timed window), the
    # sustained (power-capped) one when the clocks show the cap
    at_max = (clocks.get("sm_mhz") or 0) >= 0.97 * (clocks.get("sm_max_mhz") or 1) \
        and "sw_power_cap" not in clocks.get("reasons", [])
    peak_key = "bf16_tflops" if at_max else "bf16_tflops_sustained"
    peak_tf = float(peaks.get(peak_key, FALLBACK_PEAKS[peak_key]))
    lc = target.lcfg
    # attention reads every context token's K and V of every layer once, plus the new rows
    ctx_mean_sum = statistics.mean(ctx_sums)
    attn_bytes = tcfg.layers * (ctx_mean_sum + B * R) * lc.n_kv_heads * tcfg.head_dim * 2 * 2  # per rank
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    elem = 2  # bf16 logits
    acc_rows = (tree and 2 * R or 2 * K + 1)
    acc_bytes = B * acc_rows * tcfg.vocab * elem
    commit_bytes = statistics.mean(tokens_per_step) * tcfg.layers * lc.n_kv_heads \
        * tcfg.head_dim * 2 * 2 * 2  # K and V rows, read from scratch + written to the pool
    # DRAM bytes of the step's GEMM launches as captured by ncu at the cfg3 shapes (B=64, K=5):
    # a committed profile figure, not measured by this run
    traffic = None
    tr_path = os.path.join(ROOT, "profiles", "w4a16_gemm_traffic_cfg3.md")
    if not tree and not tp and B == 64 and K == 5 and os.path.exists(tr_path):
        import re
        m = re.search(r"traffic_bytes_per_step:\s*(\d+)", open(tr_path).read())
        traffic = int(m.group(1)) if m else None

    def hbm_entry(byts, ms_):
        if not ms_:
            return None
        gbs = byts / (ms_ / 1e3) / 1e9
        return {"bound": "hbm", "bytes_per_step": round(byts), "ms_per_step": round(ms_, 4),
                "achieved_gbs": round(gbs, 1), "peak_gbs": hbm, "frac": round(gbs / hbm, 4),
                "peak_source": f"{peak_src} hbm_gbs"}

    out = None
    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3), "higher_is_better": True,
            "scaling": "strong" if (tp or args.global_batch) else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: random-init weights (INT4 uniform [-8,7], |N(0,0.002)| fp16 scales), random "
                    "prompt ids, context K/V seeded random (stands in for a prefill), drafts from the random-init "
                    "1B INT4 draft model",
            "config": {"workload": ("cfg4 8B-INT4 tree verify+accept (64-node top-k tree 4/4/4)" if tree
                                    else f"cfg5 70B-INT4 TP-{world} verify+accept" if tp
                                    else "cfg3 8B-INT4 verify+accept"),
                       "model": "Llama-3-70B-shaped W4A16 g128" if tp else "Llama-3-8B-shaped W4A16 g128",
                       "draft": ("8B-shaped W4A16 replicated per rank" if tp else "1B-shaped W4A16")
                                + " (excluded from timing)",
                       "global_batch": B if tp else B * world,
                       **({"sequences_gathered_on_rank0": len(gathered)} if gathered is not None else {}),
                       "batch_per_gpu": B, "seq_len": args.ctx, **({"tree_nodes": K} if tree else {"k": K}),
                       "temperature": args.temperature,
                       "parallelism": (f"tensor-parallel tp{world} (NCCL all-reduce after O and down, "
                                       "all-gather of the vocabulary shards; "
                                       f"{args.tp_microbatches} micro-batch(es) on separate streams)" if tp
                                       else f"batch-sharded dp{world} (no collective; "
                                       + ("fixed global batch split over the ranks" if args.global_batch
                                          else "fixed batch per GPU") + ")"),
                       "l2": "inputs larger than L2 (GB-sized INT4 weights + KV pools per GPU)",
                       "page_tables": "host (round trip per step)" if args.host_tables or tp or tree
                                      else "device-resident (one CUDA graph per step)",
                       "mean_accepted_per_seq_step": round(tok_all / (args.steps * B * (1 if tp else world)) - 1, 3)},
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "verify_latency_ms": {"p50": round(statistics.median(step_ms), 3),
                                  "p95": round(step_ms[min(len(step_ms) - 1, math.ceil(0.95 * len(step_ms)) - 1)], 3),
                                  "min": round(step_ms[0], 3), "max": round(step_ms[-1], 3),
                                  "what": "per-step CUDA-event time of the headline loop (rank 0)"},
            "gpu_launches": launches,
            **({"speculative_round": round_out} if round_out else {}),
            "clocks": clocks,
            "roofline": {"bound": "tensor", "kernel": f"w4a16_gemm (tcgen05, all {4 * tcfg.layers + 1} GEMMs of a step"
                                   + (", per rank)" if tp else ")"),
                         "achieved": round(achieved_tf, 1), "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": round(achieved_tf / peak_tf, 4), "traffic": traffic,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the step's GEMM "
                                           "launches at B=64, K=5 (profiles/w4a16_gemm_traffic_cfg3.md); a committed "
                                           "profile figure, not measured by this run",
                         "algorithmic_bytes_per_step": round(tcfg.weight_bytes() / (world if tp else 1)
                                                             + 2 * M * sum(n + k for _, n, k in lc.linear_shapes())
                                                             * tcfg.layers),
                         "peak_source": f"{peak_src} {peak_key} (burst when the timed window ran at max SM clock "
                                        "without a power cap, else sustained)",
                         "algorithmic_flops_per_step": gemm_flops, "gemm_ms_per_step": round(gemm_ms, 3),
                         "splitk_reduction": "fused into the consuming RoPE / residual+RMSNorm / SwiGLU launches "
                                             "(timed under kernels.other_ms, not in gemm_ms)"},
            "kernels": {
                "timing": "eager instrumented pass: CUDA events around each launch group, the GPU kept ahead of "
                          "the host (device-side sleep queued first), so the sums are device time",
                "step_ms_instrumented": round(sum(kms.values()), 3),
                **{f"{k}_ms": round(v, 3) for k, v in kms.items() if v or k != "comm"},
                "attention": hbm_entry(attn_bytes, attn_ms),
                "acceptance": hbm_entry(acc_bytes, kms["accept"]),
                "kv_commit": hbm_entry(commit_bytes, kms["commit"]),
            },
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return out


# ---------------------------------------------------------------- CPU baseline / reference arm
def cpu_step_sample(args, threads: int, parity_out=None):
    """One bounded CPU sample of the verify+accept step at the bench shapes:
    one transformer layer of the 8B-shaped model (torch fp32 on the host,
    weights dequantised from INT4) over the 64 x 6 verify rows with a
    1024-token context, the lm_head, and the acceptance of all sequences by
    the reference's own compiled verify_candidates (oracle/_ref) fed the
    fp32 softmaxes, or the oracle restatement when that build is absent.
    Returns (seconds for a full step extrapolated to 32 layers, accepted
    tokens of the step, description)."""
    import numpy as np

    import oracle

    torch.set_num_threads(threads)
    from cudaforge_b200.model import LLAMA_8B
    c = LLAMA_8B
    B, K, P = args.batch, args.k, args.ctx
    R = K + 1
    M = B * R
    g = torch.Generator().manual_seed(5)

    def w4(n, k):
        q = torch.randint(0, 16, (k, n), generator=g, dtype=torch.int8).float() - 8.0
        s = (torch.randn(k // 128, n, generator=g).abs() * 0.002).half().float().repeat_interleave(128, 0)
        return (q * s).T.contiguous()  # [n, k] fp32

    W = {name: w4(n, k) for name, n, k in c.linear_shapes()}
    x = torch.randn(M, c.d_model, generator=g) * 0.02
    kc = torch.randn(B, P, c.n_kv_heads, c.head_dim, generator=g)
    vc = torch.randn(B, P, c.n_kv_heads, c.head_dim, generator=g)
    from oracle import llama_ref
    t0 = time.perf_counter()
    xn = llama_ref.rmsnorm(x, torch.ones(c.d_model))
    qkv = xn @ W["qkv"].T
    q = qkv[:, : c.n_heads * c.head_dim].view(B, R, c.n_heads, c.head_dim)
    kn = qkv[:, c.n_heads * c.head_dim:(c.n_heads + c.n_kv_heads) * c.head_dim].view(B, R, c.n_kv_heads, c.head_dim)
    vn = qkv[:, (c.n_heads + c.n_kv_heads) * c.head_dim:].view(B, R, c.n_kv_heads, c.head_dim)
    G = c.n_heads // c.n_kv_heads
    k_all = torch.cat([kc, kn], 1).repeat_interleave(G, 2)
    v_all = torch.cat([vc, vn], 1).repeat_interleave(G, 2)
    s = torch.einsum("brhd,bthd->bhrt", q, k_all) / math.sqrt(c.head_dim)
    mask = torch.ones(R, P + R, dtype=torch.bool)
    mask[:, P:] = torch.tril(torch.ones(R, R, dtype=torch.bool))
    s = s.masked_fill(~mask, float("-inf"))
    a = torch.einsum("bhrt,bthd->brhd", torch.softmax(s, -1), v_all).reshape(M, -1)
    x = x + a @ W["o"].T
    xn = llama_ref.rmsnorm(x, torch.ones(c.d_model))
    gu = xn @ W["gate_up"].T
    x = x + (torch.nn.functional.silu(gu[:, : c.ffn]) * gu[:, c.ffn:]) @ W["down"].T
    t_layer = time.perf_counter() - t0
    del W
    lm = torch.randn(c.vocab, c.d_model, generator=g) * 0.007
    t1 = time.perf_counter()
    logits = (llama_ref.rmsnorm(x, torch.ones(c.d_model)) @ lm.T).view(B, R, c.vocab)
    t_lm = time.perf_counter() - t1
    del lm
    # acceptance: softmax(/T) of the target rows and K draft rows, then verify_candidates per sequence
    dl = (logits[:, :K] + torch.randn(B, K, c.vocab, generator=g) * 0.5).numpy()
    tl = logits.numpy()
    dt = np.stack([np.argmax(dl[b], -1) for b in range(B)]).astype(np.int32)
    u = torch.rand(B, K + 1, generator=g).numpy()
    t2 = time.perf_counter()
    dp = oracle.softmax_rows(dl, args.temperature)
    tp = oracle.softmax_rows(tl, args.temperature)
    tokens = 0
    if oracle.ref_available():
        from concurrent.futures import ThreadPoolExecutor

        def one(b):
            tok, na, ef = oracle.ref_verify(42 + b, dt[b], dp[b], tp[b], -1)
            return na + 1

        with ThreadPoolExecutor(max_workers=threads) as ex:
            tokens = sum(ex.map(one, range(B)))
        kind_acc = "reference verify_candidates (compiled from the reference sources)"
    else:
        tok, na, ef = oracle.accept(dt, dp, tp, u, -1)
        tokens = int((na + 1).sum())
        kind_acc = "oracle restatement of verify_candidates"
    t_acc = time.perf_counter() - t2
    if parity_out is not None:  # untimed: the GPU acceptance kernel on this sample's logits
        parity_out.update(acceptance_parity(args, dl, tl, dt))
    step_s = c.layers * t_layer + t_lm + t_acc
    desc = (f"1 of {c.layers} layers at M={M} rows (ctx {P}) timed and x{c.layers}, + lm_head + acceptance of "
            f"{B} seqs ({kind_acc}); forward is the torch fp32 restatement (the reference has no model forward)")
    return step_s, tokens, desc, {"layer_s": t_layer, "lm_head_s": t_lm, "accept_s": t_acc}


def acceptance_parity(args, dl, tl, dt):
    """Acceptance parity at the bench shape (B sequences, K drafts, the full
    vocabulary), inside the CPU-baseline leg: the library's GPU acceptance
    kernel (cf_accept_sample) on the sample's fp32 logits, each sequence's
    uniforms drawn from the library's mt19937 engine seeded 42 + b (the
    reference engine's seed for that sequence), its softmax probabilities
    exported; the reference's compiled verify_candidates (or the oracle
    restatement when that build is absent) then decides on those same
    probabilities.  Accepted counts and emitted tokens must agree exactly."""
    import numpy as np

    import oracle
    from cudaforge_b200._C import SpeculativeConfig, SpeculativeEngine
    from cudaforge_b200.accept import accept_sample
    dev = torch.device("cuda", 0)
    B, K = dt.shape
    U = np.stack([_engine_uniforms(SpeculativeConfig, SpeculativeEngine, 42 + b, K + 1, args.temperature)
                  for b in range(B)])
    r = accept_sample(torch.from_numpy(np.ascontiguousarray(dl)).to(dev),
                      torch.from_numpy(np.ascontiguousarray(tl)).to(dev), torch.from_numpy(dt).to(dev),
                      torch.from_numpy(U).to(dev), temperature=args.temperature, export_probs=True)
    torch.cuda.synchronize()
    pd, pt = r.probs_draft.cpu().numpy(), r.probs_target.cpu().numpy()
    na_gpu = r.num_accepted.cpu().numpy()
    if oracle.ref_available():
        kind = "reference verify_candidates (compiled from the reference sources), engine seed 42 + b"
        res = [oracle.ref_verify(42 + b, dt[b], pd[b], pt[b], -1) for b in range(B)]
        tok = np.stack([t for t, _, _ in res])
        na = np.array([n for _, n, _ in res])
    else:
        kind = "oracle restatement of verify_candidates on the same uniforms"
        tok, na, _ = oracle.accept(dt, pd, pt, U, -1)
    same = [int(na_gpu[b]) == int(na[b]) and r.emitted(b) == tok[b, : int(na[b]) + 1].tolist() for b in range(B)]
    return {"acceptance": {"sequences": int(B), "k": int(K), "vocab": int(tl.shape[-1]),
                           "bit_exact_sequences": int(sum(same)), "bit_exact": bool(all(same)),
                           "mean_accepted": round(float(np.mean(na)), 3), "compared_with": kind},
            "logits": "not compared in this run: the 8B-width logits vs the fp32 restatement are the "
                      "GPU test tests/test_cfg3_parity_gpu.py (max-abs and argmax agreement)"}


def _engine_uniforms(cfg_cls, eng_cls, seed, n, temperature):
    cfg = cfg_cls()
    cfg.rng_seed = seed
    cfg.temperature = temperature
    return eng_cls(cfg).draw_uniforms(n)


def run_reference(args):
    """--impl reference: the reference path's CPU implementation on the host
    cores (rank 0 only; other ranks exit without work)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    samples = []
    toks = []
    for i in range(args.warmup + args.steps):
        s, t, desc, parts = cpu_step_sample(args, threads)
        if i >= args.warmup:
            samples.append(s)
            toks.append(t)
    tot_s = sum(samples)
    value = sum(toks) / tot_s
    return {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * tot_s / args.steps, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "cfg3 8B-INT4 verify+accept", "batch": args.batch,
                                            "seq_len": args.ctx, "k": args.k},
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def generate_cfg2(tcfg, dcfg, prompts, K, new_tokens, temperature, greedy, device, seed=0):
    """speculative generation with the tiny fp16 pair.  Both
    models prefill the prompts (all but the last token) through the paged
    runner; then full rounds -- the device-resident K-step draft loop, the
    verify + accept + commit step, the draft advance -- run until every
    sequence has `new_tokens` emitted tokens.  Returns (emitted token lists,
    device ms of the rounds, rounds, the verifier, the models)."""
    from cudaforge_b200.drafter import BatchDrafter
    from cudaforge_b200.model import LlamaModel
    from cudaforge_b200.runner import PagedRunner
    from cudaforge_b200.verifier import BatchVerifier
    B, P = prompts.shape
    ids = list(range(B))
    bps = math.ceil((P + new_tokens + 2 * (K + 1)) / 16) + 2
    target = LlamaModel(tcfg, device=device, seed=1000 + seed)
    draft = LlamaModel(dcfg, device=device, seed=2000 + seed)
    tcache = target.make_cache(B * bps + 8, max_batch=B, max_blocks_per_seq=bps + 4)
    dcache = draft.make_cache(B * (bps + 1) + 8, max_batch=B, max_blocks_per_seq=bps + 4)
    head = prompts[:, :-1].tolist()
    PagedRunner(target, tcache, ids).prefill(head)
    PagedRunner(draft, dcache, ids).prefill(head)
    ver = BatchVerifier(target, tcache, ids, K, temperature=temperature, greedy=greedy,
                        max_blocks_per_seq=bps + 4, use_graph=True)
    ver.register_context(head, prompts[:, -1], registered=True)
    dr = BatchDrafter(draft, dcache, ids, K, temperature=temperature, greedy=greedy, max_blocks_per_seq=bps + 4,
                      use_graph=True)
    dr.register_context(head, prompts[:, -1], registered=True)
    gen = torch.Generator(device=device).manual_seed(77 + seed)
    out = [[] for _ in range(B)]
    rounds = 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    while min(len(o) for o in out) < new_tokens:
        ud = None if greedy else torch.rand(B, K, generator=gen, device=device)
        uv = None if greedy else torch.rand(B, K + 1, generator=gen, device=device)
        dt, dl = dr.draft(ud)
        res = ver.step(dt, dl, uv)
        n = (ver.n_pinned.clamp_min(0) + 1).tolist()
        toks = res.tokens.cpu().tolist()
        for b in range(B):
            out[b].extend(toks[b][: n[b]])
        dr.advance(res, n)
        rounds += 1
    e1.record()
    torch.cuda.synchronize(device)
    ver.check_status()
    return out, e0.elapsed_time(e1), rounds, ver, target


def run_cfg2(args):
    """--config tiny: BASELINE config 2 on one GPU -- the tiny fp16 target /
    draft pair (random init), B=8, 128-token random prompts, K=4 chain
    drafting, 128 new tokens per sequence, greedy and at T=0.8.  The metric is
    whole-job generated tokens per second of the speculative rounds (device
    time, prefill excluded).  Logits parity for this workload is the GPU test
    tests/test_cfg2_gpu.py."""
    from cudaforge_b200.model import TINY_DRAFT, TINY_TARGET
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    B, P, K, N = 8, 128, 4, 128
    prompts = torch.randint(0, TINY_TARGET.vocab, (B, P), generator=torch.Generator().manual_seed(7))
    modes = {}
    for name, greedy, T in (("greedy", True, 1.0), ("t0.8", False, 0.8)):
        generate_cfg2(TINY_TARGET, TINY_DRAFT, prompts, K, 16, T, greedy, device)  # warm-up (captures graphs)
        out, ms, rounds, ver, _ = generate_cfg2(TINY_TARGET, TINY_DRAFT, prompts, K, N, T, greedy, device)
        emitted = sum(len(o) for o in out)
        modes[name] = {"generated_tok_s": round(emitted / (ms / 1e3), 1), "ms": round(ms, 2), "rounds": rounds,
                       "tokens_per_round_per_seq": round(emitted / (rounds * B), 3)}
    return {"metric": "generated tok/s of speculative decoding (cfg2 tiny fp16 pair)",
            "value": modes["t0.8"]["generated_tok_s"], "unit": UNIT, "n_gpus": 1, "higher_is_better": True,
            "dtype": "f16", "data": "synthetic: random-init fp16 weights N(0,0.02), random prompt ids",
            "config": {"workload": "cfg2 tiny pair: target L4/d512/8x64/FFN1408, draft L1/d256/4x64/FFN704, "
                                   "V 32000, B=8, 128-token prompts, K=4, 128 new tokens", "batch": B, "k": K},
            "modes": modes}


def _reference_kernel_module(name: str):
    """A Triton kernel module of the reference, from its offline install under
    baseline/_ref (the package's __init__ needs the reference's C++ extension,
    which is not built, so the module file is loaded by itself)."""
    import importlib.util
    path = os.path.join(ROOT, "baseline", "_ref", "cudaforge", "kernels", name + ".py")
    if not os.path.exists(path):
        raise RuntimeError(f"reference kernels not installed under baseline/_ref ({path})")
    spec = importlib.util.spec_from_file_location("cf_reference_" + name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _time_us(fn, iters):
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters * 1e3


def run_case_reference(args):
    """--case gemm|attention --impl reference: the reference's own GPU kernels
    (csrc/kernels/triton/int4_dequant_triton.py:80-131, flash_attn_triton.py:112-172)
    at the bench shapes, for a kernel-level comparison.  The INT4 kernel takes fp16
    activations (its tl.dot operand type) and its [K/8, N] packing; the attention
    kernel is self-attention over [B, H, S, D] with H_q = H_kv, so the verify shape
    (R query rows against a ctx-long cache) is run as causal self-attention over the
    ctx + R tokens -- more work than the verify step needs, which is all it can express."""
    from cudaforge_b200.model import LLAMA_8B
    dev = torch.device("cuda", 0)
    c = LLAMA_8B
    g = torch.Generator(device=dev).manual_seed(0)
    if args.case == "gemm":
        mod = _reference_kernel_module("int4_dequant_triton")
        M = args.batch * (args.k + 1)
        shapes = [(n, k) for _, n, k in c.linear_shapes()] + [(c.vocab, c.d_model)]
        x = (torch.randn(M, 14336, generator=g, device=dev) * 0.5).to(torch.float16)
        for n, k in shapes:
            wq = torch.randint(-2**31, 2**31 - 1, (k // 8, n), generator=g, device=dev, dtype=torch.int32)
            sc = (torch.randn(k // 128, n, generator=g, device=dev).abs() * 0.002).half()
            xs = x[:, :k].contiguous()
            us = _time_us(lambda: mod.int4_gemm_dequant_triton(xs, wq, sc), args.iters)
            print(json.dumps({"case": "int4_gemm_dequant_triton (reference)", "M": M, "N": n, "K": k,
                              "us": round(us, 1), "tflops": round(2 * M * n * k / us / 1e6, 1)}), flush=True)
    elif args.case == "attention":
        mod = _reference_kernel_module("flash_attn_triton")
        B, R, P = args.batch, args.k + 1, args.ctx
        S = P + R
        q = torch.randn(B, c.n_heads, S, c.head_dim, generator=g, device=dev).to(torch.float16)
        kk = torch.randn_like(q)
        vv = torch.randn_like(q)
        us = _time_us(lambda: mod.flash_attn_triton(q, kk, vv, causal=True), args.iters)
        print(json.dumps({"case": "flash_attn_triton (reference, causal self-attention)", "B": B, "H": c.n_heads,
                          "S": S, "us": round(us, 1),
                          "kv_bytes_of_the_verify_step": B * S * c.n_kv_heads * c.head_dim * 2 * 2}), flush=True)
    else:
        raise ValueError("--impl reference supports --case gemm and --case attention")


def run_case(args):
    """Single-kernel cases at the bench shapes (for ncu captures and per-shape
    timing); prints one JSON line per shape."""
    if args.impl == "reference":
        run_case_reference(args)
        return
    from cudaforge_b200 import ops
    from cudaforge_b200.gemm import w4a16_gemm
    from cudaforge_b200.model import LLAMA_8B
    dev = torch.device("cuda", 0)
    c = LLAMA_8B
    g = torch.Generator(device=dev).manual_seed(0)
    if args.case == "gemm":
        M = args.batch * (args.k + 1)
        shapes = [(n, k) for _, n, k in c.linear_shapes()] + [(c.vocab, c.d_model)]
        if args.shape:
            shapes = [tuple(int(v) for v in args.shape.split("x"))]
        x = (torch.randn(M, 14336, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        for n, k in shapes:
            wq = torch.randint(-2**31, 2**31 - 1, (k // 8, n), generator=g, device=dev, dtype=torch.int32)
            sc = (torch.randn(k // 128, n, generator=g, device=dev).abs() * 0.002).half()
            y = torch.empty(M, n, dtype=torch.bfloat16, device=dev)
            xs = x[:, :k]
            for _ in range(2):
                w4a16_gemm(xs, wq, sc, out=y)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.iters):
                w4a16_gemm(xs, wq, sc, out=y)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.iters
            print(json.dumps({"case": "w4a16_gemm", "M": M, "N": n, "K": k, "us": round(ms * 1e3, 1),
                              "tflops": round(2 * M * n * k / (ms / 1e3) / 1e12, 1),
                              "weight_gbs": round(n * k * (0.5 + 2 / 128) / (ms / 1e3) / 1e9, 1)}), flush=True)
    elif args.case == "attention":
        from cudaforge_b200.kv_cache import KVCacheConfig, PagedKVCache
        B, R, P = args.batch, args.k + 1, args.ctx
        bps = math.ceil((P + R) / 16) + 1
        cfg = KVCacheConfig(num_layers=1, num_kv_heads=c.n_kv_heads, head_dim=c.head_dim, block_size=16,
                            total_gpu_blocks=B * bps + 4, enable_prefix_caching=False, max_supported_batch_size=B)
        cache = PagedKVCache(cfg)
        for i in range(B):
            cache.register_sequence_with_prefix(i, list(range(P)))
        tables, ctx = cache.prepare_batch_metadata(list(range(B)))
        q = torch.randn(B * R, c.n_heads * c.head_dim, generator=g, device=dev).to(torch.bfloat16)
        kn = torch.randn(B, R, c.n_kv_heads, c.head_dim, generator=g, device=dev).to(torch.bfloat16)
        vn = torch.randn_like(kn)
        out = torch.empty_like(q)
        for _ in range(2):
            ops.verify_attention(cache, 0, q, kn, vn, tables, ctx, P, rows=R, num_q_heads=c.n_heads, out=out)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            ops.verify_attention(cache, 0, q, kn, vn, tables, ctx, P, rows=R, num_q_heads=c.n_heads, out=out)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.iters
        byts = B * (P + R) * c.n_kv_heads * c.head_dim * 2 * 2
        print(json.dumps({"case": "verify_attention", "B": B, "ctx": P, "R": R, "us": round(ms * 1e3, 1),
                          "gbs": round(byts / (ms / 1e3) / 1e9, 1)}), flush=True)
    elif args.case == "accept":
        from cudaforge_b200.accept import accept_sample
        B, K, V = args.batch, args.k, c.vocab
        d = (torch.randn(B, K, V, generator=g, device=dev) * 2).to(torch.bfloat16)
        t = (torch.randn(B, K + 1, V, generator=g, device=dev) * 2).to(torch.bfloat16)
        dt = torch.randint(0, V, (B, K), generator=g, device=dev, dtype=torch.int32)
        u = torch.rand(B, K + 1, generator=g, device=dev)
        for _ in range(2):
            accept_sample(d, t, dt, u)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            accept_sample(d, t, dt, u)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.iters
        byts = B * (2 * K + 1) * V * 2
        print(json.dumps({"case": "accept", "B": B, "K": K, "V": V, "us": round(ms * 1e3, 1),
                          "gbs": round(byts / (ms / 1e3) / 1e9, 1)}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="8b", choices=["8b", "tiny", "8b-tree", "70b-tp"],
                    help="8b = cfg3 chain (default); tiny = cfg2 generation with the tiny fp16 pair; 8b-tree = cfg4 (B=32, 4096 context, 64-node tree); "
                         "70b-tp = cfg5 (70B tensor-parallel over the ranks, B=128, 2048 context, K=4)")
    ap.add_argument("--batch", type=int, default=None, help="sequences per GPU (weak scaling)")
    ap.add_argument("--global-batch", type=int, default=None,
                    help="fixed global batch split evenly over the GPUs (strong scaling), e.g. 64 -> 32/16/8 per GPU")
    ap.add_argument("--ctx", type=int, default=None)
    ap.add_argument("--k", type=int, default=5)
    ap.add_argument("--temperature", type=float, default=1.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch every kernel eagerly (no CUDA graphs)")
    ap.add_argument("--no-rounds", action="store_true", help="skip the full-round (draft loop) timing")
    ap.add_argument("--tp-microbatches", type=int, default=2, choices=[1, 2],
                    help="70b-tp: run the batch as two halves on two streams so one half's all-reduces overlap "
                         "the other's kernels (1 = one batch, collectives in line)")
    ap.add_argument("--host-tables", action="store_true",
                    help="grow the page tables on the host every step (a round trip per step) instead of on the device")
    ap.add_argument("--case", default=None, choices=["gemm", "attention", "accept"],
                    help="time a single kernel at the bench shapes (profiling aid)")
    ap.add_argument("--shape", default=None, help="NxK for --case gemm")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    if args.global_batch is not None:
        from cudaforge_b200.shard import split_global_batch
        args.batch = split_global_batch(args.global_batch, int(os.environ.get("WORLD_SIZE", "1")))
    if args.batch is None:
        args.batch = {"8b-tree": 32, "70b-tp": 128}.get(args.config, 64)
    if args.ctx is None:
        args.ctx = {"8b-tree": 4096, "70b-tp": 2048}.get(args.config, 1024)
    if args.config == "70b-tp" and args.k == 5:
        args.k = 4
    if args.case:
        run_case(args)
        return
    if args.config == "tiny" and args.impl == "ours":
        print(json.dumps(run_cfg2(args)), flush=True)
        return
    if args.impl == "reference":
        out = run_reference(args)
        if out is not None:
            print(json.dumps(out), flush=True)
        return
    out = run_ours(args)
    if out is not None:
        if out["n_gpus"] == 1 and not args.no_cpu_baseline and args.config == "8b":
            par = {}
            s, t, desc, parts = cpu_step_sample(args, 1, parity_out=par)
            out["cpu_baseline"] = {"value": round(t / s, 3), "unit": UNIT, "cores": 1, "kind": "port",
                                   "sample": desc, "parts_s": {k: round(v, 3) for k, v in parts.items()}}
            out["parity"] = par
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
