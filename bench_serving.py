"""Serving workloads of bench.py: BASELINE configs 4 and 5 (the headline line of
bench.py stays config 3).

* config 4 -- chunked prefill and multi-turn on one GPU: 32 requests with
  4096-token prompts in 512-token chunks (token budget 8192) into a K/V pool of
  60% of the GPU's memory; 64 greedy decode tokens; then every request returns
  with a second turn (its committed history, the last sampled token and 1024 new
  tokens) that reuses the history from the prefix cache with a copy-on-write of
  its partial last page, and decodes 64 more tokens. Metric: prompt tokens
  computed per second of device time over both turns' prefill steps.
* config 5 -- request-sharded serving: 2048 requests drawn from a seeded prefix
  tree (16 roots of 2048 tokens, branching 4, depth 3, 256-token segments,
  prompts U[512, 8192], decode lengths U[32, 512]); every GPU serves the requests
  whose root the router deals it (one process per GPU, no collective while
  serving). Metric: output tokens per second of the whole job (strong scaling:
  the request set is fixed as the GPU count grows); the time is the maximum over
  ranks of the device time of each rank's forwards.

Both run through the public engine API (tinyinfer_b200.host.Engine over the B200
runner) on seeded synthetic inputs; `e2e` is the same metric timed by CUDA events
around the engine calls (host bookkeeping and transfers included).
"""
from __future__ import annotations

import sys
import time

import numpy as np


def _pool_pages(fraction: float, layers: int, block_tokens: int, device: int) -> int:
    """Pages of K+V (both pools) that fit in `fraction` of the device's memory."""
    import torch

    total = torch.cuda.get_device_properties(device).total_memory
    page_bytes = 2 * layers * block_tokens * 192 * 4
    return int(fraction * total // page_bytes)


def _serve(engine, dev, prompts: dict, max_new: dict):
    """Submit and step until idle. Returns a dict: outputs, steps, device ms of
    steps with prefill work and of pure decode steps, e2e ms, prompt tokens
    computed, decode tokens, summed counters."""
    for rid, p in prompts.items():
        engine.submit(rid, p, max_new[rid])
    r = {"out": {}, "steps": 0, "prefill_ms": 0.0, "decode_ms": 0.0, "prefill": 0, "decode": 0}
    dev.counters(reset=True)
    dev.sync()
    dev.timer_mark()
    last = 0.0
    while not engine.idle():
        engine.step()
        r["steps"] += 1
        st = engine.last_step_stats()
        now = dev.counters()["forward_ms"]
        if st["prefill_tokens"]:
            r["prefill_ms"] += now - last
        else:
            r["decode_ms"] += now - last
        last = now
        r["prefill"] += st["prefill_tokens"]
        r["decode"] += st["decode_tokens"]
        for rid, tok, reason, err in engine.poll_events():
            if reason == 3:
                raise RuntimeError(f"request {rid} failed: {err}")
            if tok is not None:
                r["out"].setdefault(rid, []).append(tok)
    dev.timer_mark()
    r["e2e_ms"] = dev.timer_elapsed()
    r["counters"] = dev.counters(reset=True)
    return r


def _context(args, world, local_rank):
    import torch

    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local_rank))
    torch.cuda.set_device(local_rank)
    return dist


def _line(args, metric, value, unit, world, device_ms, e2e_value, e2e_ms, counters, config, extra=None):
    line = {
        "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": config.get("steps"),
        "warmup": 0, "ms_per_step": device_ms / max(config.get("steps") or 1, 1), "higher_is_better": True,
        "scaling": config.pop("scaling"), "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) weights, seeded token ids)", "config": config,
        "e2e": {"value": e2e_value, "unit": unit, "ms": e2e_ms,
                "h2d_bytes_per_step": counters["h2d_bytes"] / max(counters["forwards"], 1),
                "d2h_bytes_per_step": counters["d2h_bytes"] / max(counters["forwards"], 1)},
        "gpu_launches": int(counters["kernel_launches"]),
    }
    if extra:
        line.update(extra)
    return line


def run_config4(args, rank, world, local_rank):
    """BASELINE config 4 (one GPU per rank; each rank runs the full workload)."""
    from tinyinfer_b200.host import Engine, Runner
    from tinyinfer_b200.synthetic import ModelConfig, random_weights

    dist = _context(args, world, local_rank)
    n, prompt, chunk, budget, new, turn2 = 32, 4096, 512, 8192, 64, 1024
    context = prompt + new + 1 + turn2 + new + 64
    cfg = ModelConfig(layers=args.layers, context=context)
    bt = args.block_tokens
    pool = _pool_pages(0.6, cfg.layers, bt, local_rank)
    weights = random_weights(cfg, seed=0)
    runner = Runner.b200(cfg, weights, context=context, block_tokens=bt, max_blocks=pool,
                         prefix_blocks=n * (context // bt + 1), device=local_rank, max_sequences=2 * n + 8,
                         max_step_tokens=budget, max_step_sequences=2 * n + 8)
    del weights
    engine = Engine(runner, n, budget, chunk, context)
    dev = engine.device()
    rng = np.random.default_rng(4040 + rank)
    p1 = {f"a{i}": [int(t) for t in rng.integers(0, cfg.vocabulary, prompt)] for i in range(n)}
    r1 = _serve(engine, dev, p1, {k: new for k in p1})
    p2 = {}
    for i in range(n):
        hist = p1[f"a{i}"] + r1["out"][f"a{i}"]
        p2[f"b{i}"] = hist + [int(t) for t in rng.integers(0, cfg.vocabulary, turn2)]
    reused0 = engine.runner_stats()["prefix_reused_tokens"]
    cow0 = engine.cost_stats()["cow_pages"]
    r2 = _serve(engine, dev, p2, {k: new for k in p2})
    reused = engine.runner_stats()["prefix_reused_tokens"] - reused0
    cow = engine.cost_stats()["cow_pages"] - cow0
    engine.shutdown()
    engine.close()
    counters = {k: r1["counters"][k] + r2["counters"][k] for k in ("forwards", "kernel_launches", "h2d_bytes", "d2h_bytes")}
    vals = np.array([r1["prefill_ms"] + r2["prefill_ms"], r1["decode_ms"] + r2["decode_ms"],
                     r1["e2e_ms"] + r2["e2e_ms"], r1["prefill"] + r2["prefill"], r1["decode"] + r2["decode"]])
    if dist:
        import torch

        t = torch.tensor(vals, dtype=torch.float64, device="cuda")
        mx = t.clone()
        dist.all_reduce(mx[:3], op=dist.ReduceOp.MAX)
        dist.all_reduce(t[3:], op=dist.ReduceOp.SUM)
        vals = np.concatenate([mx[:3].cpu().numpy(), t[3:].cpu().numpy()])
        dist.destroy_process_group()
    prefill_ms, decode_ms, e2e_ms, prefill, decode = vals.tolist()
    if rank != 0:
        return None
    config = {"workload": "config4: 32 x 4096-token prompts, 512-token chunks (budget 8192), 64 decode tokens, "
                          "second turn of history + 1024 new tokens reusing the history with COW, 64 decode tokens",
              "model": f"SmolLM2-135M shape, {cfg.layers} layers, FP32, tied head", "requests_per_gpu": n,
              "kv_pool_pages": pool, "kv_pool_gb": round(pool * 2 * cfg.layers * bt * 192 * 4 / 1e9, 1),
              "prefill_tokens": int(prefill), "decode_tokens": int(decode), "steps": r1["steps"] + r2["steps"],
              "prefill_step_ms": prefill_ms, "decode_step_ms": decode_ms,
              "decode_tok_s": decode / (decode_ms * 1e-3) if decode_ms else None,
              "turn2_reused_tokens": reused, "turn2_cow_pages": cow, "scaling": "weak",
              "parallelism": f"request-sharded replicas x{world}"}
    # e2e: prompt tokens over the whole serving time (decode steps included) -- a lower bound
    return _line(args, "chunked-prefill prompt tok/s (BASELINE config 4)", prefill / (prefill_ms * 1e-3), "tok/s",
                 world, prefill_ms + decode_ms, prefill / (e2e_ms * 1e-3), e2e_ms, counters, config)


def run_config5(args, rank, world, local_rank):
    """the prefix-tree request set, sharded by root over the ranks."""
    from tinyinfer_b200 import router
    from tinyinfer_b200.host import Engine, Runner
    from tinyinfer_b200.synthetic import ModelConfig, prefix_tree_requests, random_weights

    dist = _context(args, world, local_rank)
    count = args.serve_requests
    reqs = prefix_tree_requests(seed=5, count=count)
    mine = router.by_root([q.root for q in reqs], world, rank)
    batch, budget, chunk = 256, 8192, 2048
    context = 8192 + 512 + 16
    cfg = ModelConfig(layers=args.layers, context=context)
    bt = args.block_tokens
    pool = _pool_pages(0.6, cfg.layers, bt, local_rank)
    weights = random_weights(cfg, seed=0)
    runner = Runner.b200(cfg, weights, context=context, block_tokens=bt, max_blocks=pool,
                         prefix_blocks=pool // 2, device=local_rank, max_sequences=batch + 8,
                         max_step_tokens=budget, max_step_sequences=batch + 8)
    del weights
    engine = Engine(runner, batch, budget, chunk, context)
    dev = engine.device()
    prompts = {f"q{i}": [int(t) for t in reqs[i].prompt] for i in mine}
    max_new = {f"q{i}": reqs[i].max_new_tokens for i in mine}
    if dist:
        dist.barrier()
    r = _serve(engine, dev, prompts, max_new)
    stats = engine.runner_stats()
    engine.shutdown()
    engine.close()
    outputs = sum(len(v) for v in r["out"].values())
    vals = np.array([r["prefill_ms"] + r["decode_ms"], r["e2e_ms"], float(outputs), float(r["prefill"]),
                     float(stats["prefix_reused_tokens"]), float(len(mine))])
    if dist:
        import torch

        t = torch.tensor(vals, dtype=torch.float64, device="cuda")
        mx = t.clone()
        dist.all_reduce(mx[:2], op=dist.ReduceOp.MAX)
        dist.all_reduce(t[2:], op=dist.ReduceOp.SUM)
        vals = np.concatenate([mx[:2].cpu().numpy(), t[2:].cpu().numpy()])
        dist.destroy_process_group()
    device_ms, e2e_ms, outputs, prefill, reused, served = vals.tolist()
    if rank != 0:
        return None
    config = {"workload": f"config5: {count} requests from a seeded prefix tree (16 roots x 2048 tokens, branching 4, "
                          "depth 3, 256-token segments), prompts U[512,8192], decode U[32,512]; max batch 256/GPU, "
                          "token budget 8192, prefill chunk 2048",
              "model": f"SmolLM2-135M shape, {cfg.layers} layers, FP32, tied head", "requests": count,
              "requests_served": int(served), "output_tokens": int(outputs), "prefill_tokens": int(prefill),
              "prefix_reused_tokens": int(reused), "steps": r["steps"], "kv_pool_pages_per_gpu": pool,
              "prefix_cache_blocks_per_gpu": pool // 2,
              "routing": "by prefix-tree root (roots dealt round-robin over GPUs); no collective while serving",
              "scaling": "strong", "parallelism": f"request-sharded replicas x{world}"}
    return _line(args, "served output tok/s (BASELINE config 5)", outputs / (device_ms * 1e-3), "tok/s", world,
                 device_ms, outputs / (e2e_ms * 1e-3), e2e_ms, r["counters"], config)
