"""Bookkeeping parity of a product Engine run -- TEST INFRASTRUCTURE ONLY.

A run of the batched product Engine (tinyinfer_b200.host.Engine, any runner) is
recorded as a trace of submits and steps. ``replay`` then feeds the same
submits, with each request's tokens as emitted by the product run, through the
UNMODIFIED reference Engine (miniprefix/src/engine/engine.cpp:56-125) over the
reference's scripted runner on a real reference KVManager (oracle/_ref), and
compares after every step: the events (request, token, finish reason), the step
stats, the KV fields of the 25 runner stats, the cost counters that do not
measure time, and, where the trace holds them, every live sequence's page
table. A token stream that the device computed therefore gets the reference's
page ids, copy-on-write decisions, prefix reuse, evictions and finish order
checked bit for bit.

Only tests/ and bench.py's CPU-baseline leg import this module.
"""
from __future__ import annotations

from dataclasses import dataclass, field

from .oracle import KV_STATS_FIELDS, RefEngine, RefLib, RefRunner

# RunnerStats fields a scripted reference runner fills (its KV manager's); the
# rest count device traffic, which a scripted runner has none of.
KV_FIELDS = KV_STATS_FIELDS
# CostStats fields recorded from the product run: the prefix-cache lookups and
# publishes (counted by both KV managers) and the copy-on-write pages and bytes
# (counted by the product runner; the reference's scripted runner counts none,
# so they are compared against the copy-on-write regions it recorded instead).
COUNT_FIELDS = ("lookup_calls", "publish_calls", "cow_pages", "cow_bytes")
KV_COUNT_FIELDS = ("lookup_calls", "publish_calls")


@dataclass
class Step:
    events: list                       # (request id, token or None, finish reason or None)
    step_stats: dict | None = None     # Engine.last_step_stats()
    kv: dict | None = None             # KV_FIELDS of Engine.runner_stats()
    costs: dict | None = None          # COUNT_FIELDS of Engine.cost_stats()
    sequences: dict | None = None      # id -> (used, blocks) of live requests


@dataclass
class Trace:
    """Ops of one product Engine run, in call order."""

    ops: list = field(default_factory=list)
    ids: list = field(default_factory=list)  # submission order (poll_compact request index -> id)

    def submit(self, rid, prompt, max_new_tokens, eos=None):
        self.ops.append(("submit", rid, [int(t) for t in prompt], int(max_new_tokens), eos))
        self.ids.append(rid)

    def step(self, engine, events=None, compact=None, full=True, sequences=None):
        """Record one Engine.step(). Pass the step's events as polled
        (``events``: Engine.poll_events() tuples, or ``compact``: the arrays of
        Engine.poll_compact()); ``full`` also records step stats, KV stats and
        costs; ``sequences`` (ids) records those requests' page tables."""
        if compact is not None:
            req, tok, rea = compact
            evs = [(self.ids[int(r)], None if int(t) < 0 else int(t), None if int(x) < 0 else int(x))
                   for r, t, x in zip(req, tok, rea)]
        else:
            evs = [(e[0], e[1], e[2]) for e in events]
        s = Step(evs)
        if full:
            s.step_stats = engine.last_step_stats()
            rs = engine.runner_stats()
            s.kv = {k: rs[k] for k in KV_FIELDS}
            cs = engine.cost_stats()
            s.costs = {k: cs[k] for k in COUNT_FIELDS}
        if sequences is not None:
            s.sequences = {rid: engine.sequence(rid) for rid in sequences}
        self.ops.append(("step", s))

    def tokens(self):
        """Each request's emitted tokens, in order."""
        out = {rid: [] for rid in self.ids}
        for op in self.ops:
            if op[0] == "step":
                for rid, tok, _ in op[1].events:
                    if tok is not None:
                        out[rid].append(tok)
        return out


class Mismatch(AssertionError):
    pass


def replay(trace: Trace, *, vocabulary, context, layers, width, block_tokens, max_blocks, prefix_blocks, max_batch,
           token_budget, prefill_chunk, ref: RefLib | None = None, cow: bool = True) -> dict:
    """Replays ``trace`` through the reference engine; raises Mismatch at the first
    difference, else returns a summary of what was compared. ``cow``: the product
    runner counts its copy-on-write pages and bytes (a device runner does; a
    scripted one does not), and they must equal the number of copy-on-write
    regions the reference engine produced and their bytes (both pools)."""
    ref = ref or RefLib()
    runner = RefRunner.scripted_runner(ref, vocabulary, context, layers, width, block_tokens, max_blocks,
                                       prefix_blocks)
    engine = RefEngine(runner, max_batch, token_budget, prefill_chunk, context)
    counted = {"steps": 0, "events": 0, "stats_checks": 0, "tables": 0}
    ref_cow = [0, 0]  # copy-on-write regions and bytes so far (each read of the regions drains them)
    try:
        for n, op in enumerate(trace.ops):
            if op[0] == "submit":
                _, rid, prompt, max_new, eos = op
                engine.submit(rid, prompt, max_new, eos)
                continue
            s = op[1]
            # The scripted runner answers every append (prefill chunks included)
            # with its script's next token; a request appends at most once per
            # step, so scripting the token the product emitted for it in this step
            # (cursor back to 0) makes the reference sample the same token. An
            # append whose token the product did not emit is ignored by the engine
            # unless the reference samples where the product did not, which the
            # event comparison reports.
            for rid, tok, _ in s.events:
                if tok is not None:
                    engine.script(rid, [tok])
            engine.step()
            got = [(e[0], e[1], e[2]) for e in engine.poll_events()]
            if got != s.events:
                first = next((i for i, (a, b) in enumerate(zip(got, s.events)) if a != b), min(len(got), len(s.events)))
                raise Mismatch(f"op {n}: events differ at {first}: reference "
                               f"{got[first:first + 3]} vs product {s.events[first:first + 3]}")
            counted["steps"] += 1
            counted["events"] += len(got)
            if s.step_stats is not None:
                if engine.last_step_stats() != s.step_stats:
                    raise Mismatch(f"op {n}: step stats {engine.last_step_stats()} vs {s.step_stats}")
                rs = engine.runner_stats()
                kv = {k: rs[k] for k in KV_FIELDS}
                if kv != s.kv:
                    diff = {k: (kv[k], s.kv[k]) for k in KV_FIELDS if kv[k] != s.kv[k]}
                    raise Mismatch(f"op {n}: KV stats differ (reference, product): {diff}")
                cs = engine.cost_stats()
                for k in KV_COUNT_FIELDS:
                    if cs[k] != s.costs[k]:
                        raise Mismatch(f"op {n}: {k} {cs[k]} (reference) vs {s.costs[k]} (product)")
                if cow:
                    regions = engine.regions()
                    ref_cow[0] += len(regions)
                    ref_cow[1] += sum(2 * r[3] * r[4] * 4 for r in regions)  # K and V pools, width x rows floats
                    if tuple(ref_cow) != (s.costs["cow_pages"], s.costs["cow_bytes"]):
                        raise Mismatch(f"op {n}: copy-on-write pages / bytes {ref_cow[0]} / {ref_cow[1]} (reference "
                                       f"regions) vs {s.costs['cow_pages']} / {s.costs['cow_bytes']} (product)")
                    counted["cow_pages"] = ref_cow[0]
                counted["stats_checks"] += 1
            if s.sequences is not None:
                for rid, seq in s.sequences.items():
                    theirs = engine.sequence(rid)
                    if theirs != seq:
                        raise Mismatch(f"op {n}: page table of {rid} differs")
                    counted["tables"] += 1
    finally:
        engine.close()
        runner.close()
    return counted
