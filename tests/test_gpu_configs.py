"""BASELINE configs 4 and 5 as reduced parity cases on the GPU, against the C oracle.

* config 4 (chunked prefill, multi-turn): long prompts prefilled in chunks over
  several steps, a few greedy decode steps, then a second turn per request whose
  prompt is the first turn's history plus new tokens -- it reuses that history from
  the prefix cache and copies its partial last page on write.
* config 5 (prefix-tree serving): requests drawn from a seeded prefix tree (shared
  roots and branch segments, truncated or extended prompts, varied decode lengths),
  the shard of one rank of the by-root router served by one engine.

Every greedy token of every request must equal the oracle's, which recomputes the
whole history from an empty pool (the north star's token-identity bar).
"""
import numpy as np
import pytest

from oracle.oracle import Oracle
from tinyinfer_b200.synthetic import ModelConfig, random_weights, prefix_tree_requests


def greedy_oracle(cfg, w, bt, context):
    o = Oracle(cfg, w, bt)
    pages = context // bt + 2

    def next_token(seq):
        keys, values = o.new_pools(pages)
        out, ok = o.append(keys, values, list(range(pages)), 0, list(seq))
        assert ok
        return int(np.argmax(out))

    return next_token


def run(engine, prompts, max_new):
    for rid, p in prompts.items():
        engine.submit(rid, p, max_new[rid])
    out = {}
    steps = 0
    while not engine.idle():
        engine.step()
        steps += 1
        for rid, tok, reason, err in engine.poll_events():
            assert reason in (None, 1), err
            if tok is not None:
                out.setdefault(rid, []).append(tok)
    return out, steps


@pytest.mark.gpu
def test_config4_chunked_prefill_multi_turn(built):
    from tinyinfer_b200.host import Engine, Runner

    context, bt = 1536, 16
    cfg = ModelConfig(layers=2, intermediate=128, vocabulary=64, context=context, tied=True)
    w = random_weights(cfg, seed=41)
    oracle = greedy_oracle(cfg, w, bt, context)
    n, prompt_len, chunk, new1, turn2 = 3, 700, 128, 5, 300
    runner = Runner.b200(cfg, w, context=context, block_tokens=bt, max_blocks=n * 4 * (context // bt + 1),
                         prefix_blocks=n * (context // bt + 1), max_sequences=2 * n + 4, max_step_tokens=512,
                         max_step_sequences=2 * n + 4)
    engine = Engine(runner, n, 2 * chunk, chunk, context)
    rng = np.random.default_rng(4)
    prompts = {f"t1-{i}": [int(t) for t in rng.integers(0, 64, prompt_len)] for i in range(n)}
    out1, steps = run(engine, prompts, {k: new1 for k in prompts})
    # 700 tokens in 128-token chunks with 2 chunks of budget per step: prefill spans steps
    assert steps >= prompt_len // (2 * chunk)
    reused_before = engine.runner_stats()["prefix_reused_tokens"]
    cow_before = engine.cost_stats()["cow_pages"]
    # turn 2: history (prompt + sampled tokens) + new tokens, reusing the published history
    prompts2 = {}
    for i in range(n):
        hist = prompts[f"t1-{i}"] + out1[f"t1-{i}"]
        prompts2[f"t2-{i}"] = hist + [int(t) for t in rng.integers(0, 64, turn2)]
    out2, _ = run(engine, prompts2, {k: new1 for k in prompts2})
    assert engine.runner_stats()["prefix_reused_tokens"] - reused_before >= n * prompt_len
    assert engine.cost_stats()["cow_pages"] > cow_before
    for prompts_k, outs in ((prompts, out1), (prompts2, out2)):
        for rid, p in prompts_k.items():
            seq = list(p)
            assert len(outs[rid]) == new1
            for t in outs[rid]:
                assert t == oracle(seq), rid
                seq.append(t)
    engine.shutdown()


@pytest.mark.gpu
def test_config5_prefix_tree_shard(built):
    from tinyinfer_b200 import router
    from tinyinfer_b200.host import Engine, Runner

    context, bt = 512, 16
    cfg = ModelConfig(layers=2, intermediate=128, vocabulary=64, context=context, tied=True)
    w = random_weights(cfg, seed=43)
    oracle = greedy_oracle(cfg, w, bt, context)
    reqs = prefix_tree_requests(seed=6, count=48, roots=4, root_tokens=160, branching=3, depth=2, segment=32,
                                min_len=120, max_len=360, min_new=2, max_new=6, vocabulary=64)
    mine = router.by_root([q.root for q in reqs], 2, 0)  # rank 0's shard of a 2-GPU box
    assert 0 < len(mine) < len(reqs)
    pages = context // bt + 1
    runner = Runner.b200(cfg, w, context=context, block_tokens=bt, max_blocks=len(mine) * pages,
                         prefix_blocks=16 * pages, max_sequences=len(mine) + 4, max_step_tokens=1024,
                         max_step_sequences=len(mine) + 4)
    engine = Engine(runner, 16, 1024, 256, context)
    prompts = {f"q{i}": [int(t) for t in reqs[i].prompt] for i in mine}
    max_new = {f"q{i}": reqs[i].max_new_tokens for i in mine}
    out, _ = run(engine, prompts, max_new)
    assert engine.runner_stats()["prefix_hits"] > 0
    for rid, p in prompts.items():
        seq = list(p)
        assert len(out[rid]) == max_new[rid]
        for t in out[rid]:
            assert t == oracle(seq), rid
            seq.append(t)
    engine.shutdown()
