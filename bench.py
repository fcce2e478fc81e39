"""Benchmark: batched greedy decode of the 135M-shape FP32 model over paged KV
on N GPUs, one process per GPU, requests sharded by GPU.

Per GPU: 256 requests whose 2048-token prompts share a 1032-token prefix (64 full
pages + 8 tokens of a partial page that every follower reuses and copies on
write), page size 16. A seed request is prefilled first so that the prefix is
published; the followers then prefill their 1016-token suffixes. A "step" is one
Engine.step() in which all 256 requests decode one token. W untimed warm-up steps,
then exactly K timed steps.

  value  = decode tokens / device time of the K steps' forwards (inputs resident:
           CUDA events around the kernels of each forward on the context stream)
  e2e    = decode tokens / time of the K Engine.step() calls through the C ABI,
           CUDA events on the context stream bracketing them (host bookkeeping,
           H2D of tokens/tables/work lists, forward, D2H of tokens included)
  roofline: the paged-attention kernel (CUDA events around each launch), bytes =
           each decode row's K/V tokens x 1536 B + q/out rows + table entries.

--impl reference times the reference's own CPU engine (oracle/_ref, built from the
reference sources) on the host cores instead. Synthetic seeded data throughout.
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")
METRIC = "decode tok/s, 135M FP32 paged-KV, batch 256/GPU, ctx 2k (shared 1032-token prefix, COW)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=128)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--requests", type=int, default=256)
    p.add_argument("--prompt", type=int, default=2048)
    p.add_argument("--shared", type=int, default=1032)
    p.add_argument("--block-tokens", type=int, default=16)
    p.add_argument("--prefix-blocks", type=int, default=66)
    p.add_argument("--layers", type=int, default=30)
    p.add_argument("--prefill-budget", type=int, default=8192)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-workers", type=int, default=0)
    p.add_argument("--operator", nargs="?", const="decode", choices=["decode", "prefill"], default=None,
                   help="time an attention operator alone: decode on BASELINE config 2, or prefill on config 4's "
                        "last chunk (16 sequences x 512 rows at position 3584)")
    p.add_argument("--workload", choices=["config3", "config4", "config5"], default="config3",
                   help="config3: the headline decode benchmark; config4 / config5: the serving workloads "
                        "of bench_serving.py")
    p.add_argument("--serve-requests", type=int, default=2048, help="config 5 request count")
    p.add_argument("--shared-prefix-kernel", action="store_true",
                   help="serve shared prefix pages with the tensor-core shared-prefix kernel (off by default)")
    return p.parse_args()


def peaks():
    try:
        with open(PEAKS) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def fp16_peak():
    """Dense 16-bit tensor-core throughput of this pool's B200s (the GEMMs' MMA kind,
    kind::f16; FP16 runs at the BF16 rate): MEASURED_PEAKS.json's bf16 burst figure
    (cuBLAS 8192^3, best of 10), the denominator of the GEMM roofline."""
    try:
        with open(PEAKS) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    except Exception:
        return 1590.0, "fallback"


def tf32_peak(device_index):
    """Dense TF32 tensor-core throughput of this GPU, measured here: torch.matmul
    (cuBLAS) on 8192^3 FP32 operands with TF32 enabled, best of 10 launches timed
    with CUDA events (2 N^3 FLOP each). The denominator of the tensor-core prefill
    attention roofline (its MMAs are kind::tf32)."""
    import torch

    dev = torch.device("cuda", device_index)
    n = 8192
    g = torch.Generator(device=dev).manual_seed(1)
    a = torch.randn(n, n, device=dev, generator=g)
    b = torch.randn(n, n, device=dev, generator=g)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        for _ in range(3):
            c = torch.matmul(a, b)
        best = None
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            c = torch.matmul(a, b)
            e1.record()
            e1.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b, c
    torch.cuda.empty_cache()
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12


# ----------------------------------------------------------------------------- workload
# Decode steps run after the timed ones with CUDA events around every attention
# launch and the LM head: the per-kernel breakdown of the roofline lines. They are
# not timed into `value`: an event recorded between two kernels ends programmatic
# dependent launch at that boundary (about 6% of a config-3 step with 61 of them).
PROFILED_STEPS = 3


def max_new_tokens(args):
    """Enough new tokens that no request finishes before the profiled steps end: the
    followers that start decoding first run ahead by up to the prefill steps."""
    prefill_steps = -(-args.requests * (args.prompt - args.shared) // args.prefill_budget)
    return args.warmup + args.steps + PROFILED_STEPS + prefill_steps + 8


def model_config(args):
    from tinyinfer_b200.synthetic import ModelConfig

    return ModelConfig(layers=args.layers, context=args.prompt + max_new_tokens(args) + 32)


def prompts(args, indices):
    """Seeded prompts of the given global requests: one shared prefix, a unique
    suffix per request seeded by its global index (independent of the GPU count)."""
    vocab = 49152
    shared = np.random.default_rng(7).integers(0, vocab, args.shared).astype(np.int32)
    out = []
    for i in indices:
        suffix = np.random.default_rng([20240, i]).integers(0, vocab, args.prompt - args.shared).astype(np.int32)
        out.append(np.concatenate([shared, suffix]))
    return out


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            f = [x.strip() for x in line.split(",")]
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
                for name, v in zip(names, f[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(name)
            except Exception:
                continue
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [s for s in sm if s > 0.5 * (mx or max(sm))] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def logical_decode_bytes(engine, ids):
    """K/V bytes one layer's decode attention would read if every row streamed its
    whole context (no shared-prefix dedup): sum of context lengths x 1536 B."""
    total = 0
    for rid in ids:
        s = engine.sequence(rid)
        if s:
            total += s[0] + 1
    return total * 2 * 192 * 4


def unique_decode_bytes(engine, ids, block_tokens):
    """Bytes of the distinct (page, slot) K/V rows one layer's decode attention reads
    (each shared prefix page once), x 1536 B per token row."""
    seen = {}
    for rid in ids:
        s = engine.sequence(rid)
        if not s:
            continue
        used, blocks = s
        for i, b in enumerate(blocks):
            valid = min(block_tokens, used + 1 - i * block_tokens)
            if valid > 0:
                seen[b] = max(seen.get(b, 0), valid)
    return sum(seen.values()) * 2 * 192 * 4


# ----------------------------------------------------------------------------- CPU baseline
def _cpu_worker(index, layers, prompt, shared, decode_steps, go, results):
    """One single-threaded reference CpuRunner (oracle/_ref) on config 3's request
    `index`: its 2048-token prompt (the shared 1032-token prefix + its own suffix)
    prefilled untimed, then, once `go` is set, `decode_steps` greedy decode tokens
    timed at context 2048+."""
    sys.path.insert(0, ROOT)
    from oracle.oracle import RefLib, RefRunner
    from tinyinfer_b200.synthetic import ModelConfig, random_weights

    try:
        c = ModelConfig(layers=layers, context=len(prompt) + decode_steps + 16)
        w = random_weights(c, seed=0)
        ref = RefLib()
        r = RefRunner.cpu(ref, c, w, c.context, 16, (c.context + 15) // 16 + 1, 0)
        del w
        r.create("s")
        t0 = time.perf_counter()
        logits = r.append("s", prompt)
        prefill_s = time.perf_counter() - t0
        go.wait()
        start = time.perf_counter()
        for _ in range(decode_steps):
            logits = r.append("s", [int(np.argmax(logits))])
        results.put((index, decode_steps, time.perf_counter() - start, prefill_s, None))
    except Exception as e:  # reported, never silently dropped
        results.put((index, 0, 0.0, 0.0, f"{type(e).__name__}: {e}"))


class CpuBaseline:
    """The reference CPU engine at BASELINE config 3's context, on the host cores:
    P single-threaded reference CpuRunner processes (spawned), one per core, each
    holding one of config 3's requests (2048-token prompt: 1032 shared + 1016 own
    tokens). The prefills (minutes of CPU) run untimed and may overlap the GPU arm;
    start() launches them, measure() releases the timed decode steps and returns
    the aggregate decode tok/s at context 2048."""

    def __init__(self, args, workers=None, decode_steps=16):
        self.args = args
        self.n = workers or args.cpu_workers or max(1, min((os.cpu_count() or 1) - 2, 16))
        self.decode_steps = decode_steps
        self.procs = []

    def start(self):
        from oracle import oracle as orc

        self.available = os.path.exists(orc.REF_SO)
        if not self.available:
            return self
        ctx = mp.get_context("spawn")
        self.go = ctx.Event()
        self.results = ctx.Queue()
        self.t0 = time.perf_counter()
        for i, p in enumerate(prompts(self.args, range(self.n))):
            proc = ctx.Process(target=_cpu_worker, args=(i, self.args.layers, [int(t) for t in p], self.args.shared,
                                                          self.decode_steps, self.go, self.results), daemon=True)
            proc.start()
            self.procs.append(proc)
        return self

    def measure(self):
        if not self.available:
            return {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference", "same_config": True,
                    "sample": "oracle/_ref/libmpref.so not present on this host"}
        self.go.set()
        got = [self.results.get(timeout=3600) for _ in self.procs]
        for proc in self.procs:
            proc.join(timeout=60)
        errors = [g[4] for g in got if g[4]]
        if errors:
            return {"value": None, "unit": "tok/s", "cores": self.n, "kind": "reference", "same_config": True,
                    "sample": f"reference CPU workers failed: {errors[0]}"}
        steps = sum(g[1] for g in got)
        elapsed = max(g[2] for g in got)
        prefill = max(g[3] for g in got)
        cpu = "unknown CPU"
        try:
            with open("/proc/cpuinfo") as f:
                cpu = next(l.split(":", 1)[1].strip() for l in f if l.startswith("model name"))
        except Exception:
            pass
        return {"value": steps / elapsed, "unit": "tok/s", "cores": self.n, "kind": "reference",
                "same_config": True, "cpu_model": cpu, "host_cpus": os.cpu_count(),
                "per_core_tok_s": steps / elapsed / self.n,
                "sample": (f"{self.n} single-threaded reference CpuRunner processes (oracle/_ref, AVX2+FMA) on "
                           f"{cpu}, each holding one config-3 request (2048-token prompt = the 1032-token shared "
                           f"prefix + 1016 own tokens, prefilled untimed in {prefill:.0f} s) and greedy-decoding "
                           f"{self.decode_steps} tokens at context 2048-{2048 + self.decode_steps} "
                           f"({steps} tokens in {elapsed:.1f} s)")}


def replay_parity(record, cow=True):
    """CPU-baseline leg, after the timed steps: the run's emitted tokens replayed
    through the UNMODIFIED reference engine over its scripted runner
    (oracle/replay.py). Every step's events (request, token, finish reason) must be
    identical; so must the step stats, KV stats and copy-on-write / reuse counters
    after every untimed step and at the end, and the final page table of every
    request (bit-exact page ids). The token values themselves are checked against
    the C oracle's logits by tests/test_gpu_config3.py at this geometry."""
    from oracle.replay import COUNT_FIELDS, KV_FIELDS, Mismatch, Step, Trace, replay

    t0 = time.perf_counter()
    trace = Trace()
    trace.ids = list(record["ids"])
    for op in record["ops"]:
        if op[0] == "submit":
            trace.ops.append(("submit", op[1], [int(x) for x in op[2]], int(op[3]), None))
        elif op[0] == "step":
            _, evs, ss, rs, cs = op
            trace.ops.append(("step", Step(list(evs), ss, {k: rs[k] for k in KV_FIELDS},
                                           {k: cs[k] for k in COUNT_FIELDS})))
        else:
            req, tok, rea = op[1]
            trace.ops.append(("step", Step([(trace.ids[int(r)], None if int(x) < 0 else int(x),
                                             None if int(y) < 0 else int(y)) for r, x, y in zip(req, tok, rea)])))
    final, last = record["final"], trace.ops[-1][1]
    last.step_stats = final["step_stats"]
    last.kv = {k: final["runner_stats"][k] for k in KV_FIELDS}
    last.costs = {k: final["costs"][k] for k in COUNT_FIELDS}
    last.sequences = {rid: seq for rid, seq in final["sequences"].items() if seq is not None}
    out = {"checked_by": "reference Engine + scripted runner (oracle/_ref) fed this run's emitted tokens"}
    try:
        out["compared"] = replay(trace, cow=cow, **record["geometry"])
        out["bookkeeping"] = "identical"
    except Mismatch as e:
        out["bookkeeping"] = "MISMATCH"
        out["detail"] = str(e)
    except Exception as e:  # reference library missing or failing: say so, do not guess
        out["bookkeeping"] = None
        out["detail"] = f"replay not run: {type(e).__name__}: {e}"
    out["seconds"] = round(time.perf_counter() - t0, 1)
    return out


# ----------------------------------------------------------------------------- B200 arm
def run_b200(args, rank, world, local_rank):
    import torch

    from tinyinfer_b200 import router
    from tinyinfer_b200.host import Engine, Runner
    from tinyinfer_b200.synthetic import random_weights

    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
    torch.cuda.set_device(local_rank)

    cfg = model_config(args)
    weights = random_weights(cfg, seed=0)
    bt = args.block_tokens
    n = args.requests
    max_new = max_new_tokens(args)
    pages_per_request = -(-(args.prompt + max_new - 1) // bt)
    max_blocks = (n + 1) * pages_per_request + 64
    runner = Runner.b200(cfg, weights, context=cfg.context, block_tokens=bt, max_blocks=max_blocks,
                         prefix_blocks=args.prefix_blocks, device=local_rank, max_sequences=n + 8,
                         max_step_tokens=args.prefill_budget, max_step_sequences=n + 8)
    del weights
    engine = Engine(runner, n, args.prefill_budget, args.prompt, cfg.context)
    dev = engine.device()
    if args.shared_prefix_kernel:
        dev.shared_prefix(8, 128)
    # this GPU's shard of the world's requests (round-robin, no collective)
    mine = router.round_robin(n * world, world, rank)
    ps = prompts(args, mine)
    ids = [f"r{i}" for i in mine]

    # The run is recorded (submits, every step's events; stats and page tables
    # outside the timed steps) so that the CPU-baseline leg can replay it through
    # the reference engine: plain lists here, nothing from oracle/.
    record = {"ops": [], "ids": ids}

    def setup_step():
        engine.step()
        evs = engine.poll_events()
        rs, cs = engine.runner_stats(), engine.cost_stats()
        record["ops"].append(("step", [(e[0], e[1], e[2]) for e in evs], engine.last_step_stats(), rs, cs))
        return evs

    def submit(i):
        engine.submit(ids[i], ps[i], max_new)
        record["ops"].append(("submit", ids[i], ps[i], max_new))

    # Seed: prefill to completion so the shared prefix is published.
    t_setup = time.perf_counter()
    submit(0)
    while not any(e[1] is not None for e in setup_step()):
        pass
    for i in range(1, n):
        submit(i)
    started = {ids[0]}
    while len(started) < n:
        for rid, tok, reason, err in setup_step():
            if reason == 3:
                raise RuntimeError(f"request {rid} failed: {err}")
            if tok is not None:
                started.add(rid)
    setup_s = time.perf_counter() - t_setup
    reused = engine.runner_stats()["prefix_reused_tokens"]
    cow = engine.cost_stats()["cow_pages"]

    def decode_step():
        engine.step()
        evs = engine.poll_compact()
        record["ops"].append(("compact", evs))
        return len(evs[0])

    for _ in range(args.warmup):
        decode_step()
    uniq = unique_decode_bytes(engine, ids, bt)
    logical = logical_decode_bytes(engine, ids)
    before = dev.counters(reset=True)
    # kernels launched before the timed steps (for `ncu -s` on this command)
    print(f"launches_before_timed={before['kernel_launches']}", file=sys.stderr, flush=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    dev.sync()
    tokens = 0
    with ClockSampler(local_rank) as clocks:
        # profiler range = the timed steps (`ncu --profile-from-start off` captures
        # exactly these launches; a no-op without a profiler)
        torch.cuda.cudart().cudaProfilerStart()
        dev.timer_mark()
        for _ in range(args.steps):
            tokens += decode_step()
        dev.timer_mark()
        e2e_ms = dev.timer_elapsed()
        dev.sync()
        torch.cuda.cudart().cudaProfilerStop()
    dev.sync()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    counters = dev.counters(reset=True)
    # per-kernel breakdown: a few more decode steps with events around the kernels
    dev.profile_read()
    dev.profile_read_gemm()
    dev.profile(True)
    for _ in range(PROFILED_STEPS):
        decode_step()
    dev.sync()
    dev.profile(False)
    attn_ms, attn_launches, attn_bytes = dev.profile_read()
    gemm_ms, gemm_intervals, head_ms, heads = dev.profile_read_gemm()
    record["final"] = {"step_stats": engine.last_step_stats(), "runner_stats": engine.runner_stats(),
                       "costs": engine.cost_stats(), "sequences": {rid: engine.sequence(rid) for rid in ids}}
    record["geometry"] = dict(vocabulary=cfg.vocabulary, context=cfg.context, layers=cfg.layers, width=cfg.kv_width,
                              block_tokens=bt, max_blocks=max_blocks, prefix_blocks=args.prefix_blocks, max_batch=n,
                              token_budget=args.prefill_budget, prefill_chunk=args.prompt)
    if dist:
        dist.barrier()

    device_ms = counters["forward_ms"]
    stats = torch.tensor([e2e_ms, device_ms, float(tokens)], dtype=torch.float64, device="cuda")
    if dist:
        mx = stats.clone()
        dist.all_reduce(mx[:2], op=dist.ReduceOp.MAX)
        tot = stats.clone()
        dist.all_reduce(tot[2:], op=dist.ReduceOp.SUM)
        e2e_ms, device_ms, tokens_all = float(mx[0]), float(mx[1]), float(tot[2])
    else:
        tokens_all = float(tokens)
    if rank != 0:
        if dist:
            dist.destroy_process_group()
        return None

    hbm, peak_kind = peaks()
    launch_ms = attn_ms / max(attn_launches, 1)
    # DRAM-level algorithmic bytes of one layer's decode attention: every distinct
    # K/V row once (the shared prefix pages are read by all rows but come from
    # DRAM once, then L2), plus each row's query and output
    bytes_per_launch = uniq + n * 2 * 576 * 4
    achieved = bytes_per_launch / (launch_ms * 1e-3) / 1e9 if launch_ms > 0 else None
    traffic, traffic_source = None, None
    # DRAM bytes per launch from the committed ncu capture of the same kernel on the
    # same rows, scaled to this run's algorithmic bytes per launch
    tpath = os.path.join(ROOT, "profiles", "paged_attention_decode_config3_traffic.json")
    if os.path.exists(tpath):
        try:
            with open(tpath) as f:
                t = json.load(f)
            traffic = t["dram_bytes_per_launch"] * bytes_per_launch / t["algorithmic_bytes_per_launch"]
            traffic_source = t.get("source")
        except Exception:
            traffic = None
    line = {
        "metric": METRIC,
        "value": tokens_all / (device_ms * 1e-3),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": device_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) weights, uniform random token ids)",
        "config": {"workload": "config3: batched greedy decode, 256 requests/GPU at ctx 2048, 1032-token shared "
                               "prefix reused with COW of its partial page",
                   "model": "SmolLM2-135M shape, 30 layers, FP32, tied head", "requests_per_gpu": args.requests,
                   "prompt_tokens": args.prompt, "shared_prefix_tokens": args.shared, "block_tokens": bt,
                   "shared_prefix_path": "tensor-core shared-prefix kernel" if args.shared_prefix_kernel else
                                         "every row reads its whole context (shared pages from L2)",
                   "prefix_cache_blocks": args.prefix_blocks, "parallelism": f"request-sharded replicas x{world}",
                   "routing": "round-robin by global request index; each GPU its own weights, KV pool, "
                              "prefix cache and engine; no collective in a step",
                   "l2": "inputs larger than L2 (>= 24 GB of K/V read per step)",
                   "setup_seconds": round(setup_s, 1), "prefix_reused_tokens": reused, "cow_pages": cow},
        "e2e": {"value": tokens_all / (e2e_ms * 1e-3), "unit": "tok/s",
                "h2d_bytes_per_step": counters["h2d_bytes"] / max(counters["forwards"], 1),
                "d2h_bytes_per_step": counters["d2h_bytes"] / max(counters["forwards"], 1),
                "ms_per_step": e2e_ms / args.steps,
                # host wall time per step inside the C ABI (rank 0); the rest of
                # e2e - device is engine bookkeeping (schedule, KV manager, publish)
                "host_ms_per_step": {k: counters[f"host_{k}_ms"] / args.steps for k in ("prepare", "launch", "wait")}},
        "gpu_launches": int(counters["kernel_launches"]),
        "roofline": {"bound": "hbm",
                     "kernel": "paged_attention_kernel: split-K decode attention of every row over its whole "
                               "context; the shared prefix pages are read by all rows, from DRAM once and then L2",
                     "timing": f"CUDA events around each attention launch on the context stream, over "
                               f"{PROFILED_STEPS} decode steps run right after the timed ones (events between "
                               f"kernels end programmatic dependent launch there, so these durations are upper "
                               f"bounds of the timed steps' launches)",
                     "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm if achieved else None, "traffic": traffic,
                     "traffic_source": traffic_source,
                     "peak_kind": peak_kind, "launch_ms": launch_ms, "launches": attn_launches,
                     "algorithmic_bytes_per_launch": bytes_per_launch,
                     "logical_bytes_per_launch": logical,
                     "logical_achieved": logical / (launch_ms * 1e-3) / 1e9 if launch_ms > 0 else None,
                     "attention_share_of_forward": (attn_ms / PROFILED_STEPS) / (device_ms / args.steps)
                     if device_ms else None},
        "gemm_roofline": gemm_roofline(cfg, n, gemm_ms, gemm_intervals, head_ms, heads),
        "clocks": clocks.summary(),
        "_record": record,
    }
    engine.shutdown()
    engine.close()
    if dist:
        dist.destroy_process_group()
    return line


def gemm_roofline(cfg, rows, gemm_ms, intervals, head_ms, heads):
    """The projection GEMMs of one decode step at M = rows, against the measured
    16-bit tensor peak. Useful FLOP 2 M N K (the kernels issue 3x that: the split
    FP16 products A_hi.B_hi, A_hi.B_lo, A_lo.B_hi): per layer QKV 576x960, O
    576x576, gate/up 576x3072, down 1536x576; the tied LM head 576x49152. Times
    from CUDA events on the context stream: each interval between two layers'
    attention launches holds one layer's four GEMMs."""
    H, I, V = cfg.hidden, cfg.intermediate, cfg.vocabulary
    kvw = cfg.kv_width
    layer_flop = 2.0 * rows * (H * (H + 2 * kvw) + H * H + H * 2 * I + I * H)
    head_flop = 2.0 * rows * H * V
    peak, kind = fp16_peak()
    out = {"bound": "tensor", "unit": "TFLOP/s", "peak": peak, "peak_kind": kind, "mma_kind": "f16 (split FP32)",
           "useful_flop_per_layer": layer_flop, "issued_flop_per_layer": 3 * layer_flop,
           "useful_flop_head": head_flop}
    if intervals:
        us = 1000.0 * gemm_ms / intervals
        ach = layer_flop / (us * 1e-6) / 1e12
        out.update({"layer_gemm_us": us, "achieved": ach, "frac": ach / peak, "issued_frac": 3 * ach / peak})
    if heads:
        us = 1000.0 * head_ms / heads
        ach = head_flop / (us * 1e-6) / 1e12
        out.update({"head_us": us, "head_achieved": ach, "head_frac": ach / peak, "head_issued_frac": 3 * ach / peak})
    return out


# ----------------------------------------------------------------------------- operator (config 2)
def config2(seed=2, count=64, max_len=4096, block_tokens=16, pool=32768):
    """64 sequences, lengths U[1, 4096], page 16, tables a random
    permutation of a 32768-page one-layer pool, Q/K/V ~ N(0, 1)."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(1, max_len + 1, size=count).astype(np.int32)
    pages = (lengths + block_tokens - 1) // block_tokens
    perm = rng.permutation(pool).astype(np.int32)
    tables = np.zeros((count, int(pages.max())), dtype=np.int32)
    at = 0
    for i, p in enumerate(pages):
        tables[i, :p] = perm[at:at + p]
        at += p
    return lengths, tables, pool


def run_operator(args, local_rank):
    import torch

    from tinyinfer_b200 import device

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    lengths, tables, pool = config2()
    bt = 16
    gen = torch.Generator(device=dev).manual_seed(2)
    keys = torch.randn(pool * bt * 192, device=dev, generator=gen)
    values = torch.randn(pool * bt * 192, device=dev, generator=gen)
    q = torch.randn(len(lengths), 576, device=dev, generator=gen)
    out = torch.empty_like(q)
    tt = torch.from_numpy(tables).to(dev)
    stream = torch.cuda.current_stream()
    algorithmic = float(lengths.sum()) * 1536 + len(lengths) * 576 * 4 * 2 + float(((lengths + 15) // 16).sum()) * 4 + \
        len(lengths) * 4

    def launch():
        device.paged_attention_decode(q.data_ptr(), keys.data_ptr(), values.data_ptr(), 1, 0, bt, pool, tt.data_ptr(),
                                      tables.shape[1], lengths, out.data_ptr(), 0, stream.cuda_stream)

    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize()
    times = []
    with ClockSampler(local_rank) as clocks:
        torch.cuda.cudart().cudaProfilerStart()
        for _ in range(args.steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            launch()
            b.record(stream)
            times.append((a, b))
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
    assert device.paged_attention_status(stream.cuda_stream) == 0
    ms = [a.elapsed_time(b) for a, b in times]
    avg = sum(ms) / len(ms)
    hbm, kind = peaks()
    gbs = algorithmic / (avg * 1e-3) / 1e9
    return {"metric": "paged-attention decode HBM GB/s (BASELINE config 2)", "value": gbs, "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": avg, "higher_is_better": True,
            "dtype": "f32", "data": "synthetic (seeded N(0,1) Q/K/V)",
            "config": {"workload": "config2: 64 sequences, lengths U[1,4096], 9q/3kv heads, d 64, page 16, "
                                   "32768-page pool, random-permutation tables",
                       "algorithmic_bytes": algorithmic, "l2": "inputs larger than L2 (201 MB per launch)"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "peak_kind": kind, "min_ms": min(ms), "max_ms": max(ms)},
            "clocks": clocks.summary()}


def run_operator_prefill(args, local_rank):
    """The tensor-core prefill attention operator on BASELINE config 4's geometry:
    16 sequences each appending its last 512-token chunk at positions 3584..4095 of
    a 4096-token prompt (one-layer pool, random-permutation tables, Q/K/V ~ N(0,1)).
    Useful FLOP = 4 x 64 per (row, head, visible key); the kernel issues 3x that
    as 3xTF32 MMAs plus the masked part of each 64-token sub-chunk."""
    import torch

    from tinyinfer_b200 import device

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    seqs, start, count, bt = 16, 3584, 512, 16
    pages = (start + count) // bt
    pool = seqs * pages
    rng = np.random.default_rng(4)
    tables = rng.permutation(pool).astype(np.int32).reshape(seqs, pages)
    gen = torch.Generator(device=dev).manual_seed(4)
    keys = torch.randn(pool * bt * 192, device=dev, generator=gen)
    values = torch.randn(pool * bt * 192, device=dev, generator=gen)
    q = torch.randn(seqs * count, 576, device=dev, generator=gen)
    out = torch.empty_like(q)
    tt = torch.from_numpy(tables).to(dev)
    stream = torch.cuda.current_stream()
    starts, counts = [start] * seqs, [count] * seqs
    visible = seqs * sum(start + r + 1 for r in range(count))  # (row, key) pairs per head
    useful = 4.0 * 64 * 9 * visible

    def launch():
        device.paged_attention_prefill(q.data_ptr(), keys.data_ptr(), values.data_ptr(), 1, 0, bt, pool,
                                       tt.data_ptr(), pages, starts, counts, out.data_ptr(), stream.cuda_stream)

    peak = tf32_peak(local_rank)
    for _ in range(max(args.warmup, 1)):
        launch()
    torch.cuda.synchronize()
    times = []
    with ClockSampler(local_rank) as clocks:
        torch.cuda.cudart().cudaProfilerStart()
        for _ in range(args.steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            launch()
            b.record(stream)
            times.append((a, b))
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
    assert device.paged_attention_status(stream.cuda_stream) == 0
    ms = [a.elapsed_time(b) for a, b in times]
    avg = sum(ms) / len(ms)
    tflops = useful / (avg * 1e-3) / 1e12
    return {"metric": "prefill attention useful TFLOP/s (BASELINE config 4, last 512-token chunk)", "value": tflops,
            "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": avg,
            "higher_is_better": True, "dtype": "f32 (3xTF32 tensor-core products)",
            "data": "synthetic (seeded N(0,1) Q/K/V)",
            "config": {"workload": "config4 prefill attention operator: 16 sequences x 512 rows at positions "
                                   "3584..4095, 9q/3kv heads, d 64, page 16, random-permutation tables",
                       "useful_flop": useful, "prompt_tokens_per_step": seqs * count},
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": tflops / peak, "issued_frac": 3 * tflops / peak,
                         "peak_kind": "measured here: cuBLAS TF32 8192^3, best of 10",
                         "min_ms": min(ms), "max_ms": max(ms)},
            "clocks": clocks.summary()}


# ----------------------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    """The reference arm: the reference's own CPU engine (oracle/_ref, compiled from
    the reference sources) at config 3's context on this host's cores; rank 0 only."""
    if rank != 0:
        return None
    from oracle import oracle as orc

    if not os.path.exists(orc.REF_SO):
        return {"impl": "reference", "unavailable": "oracle/_ref/libmpref.so (reference CPU engine) not built on this host"}
    res = CpuBaseline(args, decode_steps=max(4, min(args.steps, 16))).start().measure()
    value = res["value"]
    return {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": None if not value else 1000.0 * res["cores"] / value,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": "config3 decode at context 2048 on the reference CPU engine (see "
                                   "cpu_baseline.sample)",
                       "model": f"SmolLM2-135M shape, {args.layers} layers, FP32, tied head", "same_config": True},
            "cpu_baseline": res,
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
    elif args.operator:
        run = run_operator_prefill if args.operator == "prefill" else run_operator
        line = run(args, local_rank) if rank == 0 else None
    elif args.workload != "config3":
        import bench_serving

        run = bench_serving.run_config4 if args.workload == "config4" else bench_serving.run_config5
        line = run(args, rank, world, local_rank)
    else:
        # the CPU baseline's untimed prefills start first (spawned processes, no
        # CUDA) and overlap the GPU arm; their timed decode runs after it
        baseline = CpuBaseline(args).start() if world == 1 and not args.no_cpu_baseline else None
        line = run_b200(args, rank, world, local_rank)
        record = line.pop("_record", None) if line is not None else None
        if line is not None and baseline is not None:
            line["parity"] = replay_parity(record)
            line["cpu_baseline"] = baseline.measure()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
