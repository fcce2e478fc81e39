"""One rank of the request-sharded host path, launched by tests/test_multi_rank.py
as `torch.distributed.run --nproc-per-node 2 ... tests/multi_rank_worker.py OUT`.

Every rank builds the same global workload (small prefix-tree requests), keeps
the requests tinyinfer_b200.router.by_root assigns it, serves them with its own
engine over a device-free scripted runner (its own KV manager and prefix cache),
and writes its events and counters to OUT/rank<r>.json; the summed counters of
all ranks (router.gather_counters over gloo) go to the same file. No collective
runs while requests are served.
"""
import json
import os
import sys
from datetime import timedelta

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch.distributed as dist  # noqa: E402

from tinyinfer_b200 import router  # noqa: E402
from tinyinfer_b200.host import Engine, Runner  # noqa: E402
from tinyinfer_b200.synthetic import prefix_tree_requests  # noqa: E402

WORKLOAD = dict(seed=3, count=40, roots=4, root_tokens=12, branching=2, depth=2, segment=5, min_len=4, max_len=30,
                min_new=1, max_new=6, vocabulary=16)
ENGINE = dict(vocab=16, context=48, block_tokens=4, max_blocks=160, prefix_blocks=24, max_batch=4, token_budget=32,
              prefill_chunk=16)


def serve(indices, requests):
    """Runs one shard to completion; returns (events, runner stats, step count)."""
    p = ENGINE
    r = Runner.scripted(p["vocab"], p["context"], 1, 1, p["block_tokens"], p["max_blocks"], p["prefix_blocks"])
    e = Engine(r, p["max_batch"], p["token_budget"], p["prefill_chunk"], p["context"])
    for i in indices:
        q = requests[i]
        r.script(f"q{i}", [(i * 7 + k) % p["vocab"] for k in range(32)])
        e.submit(f"q{i}", [int(t) for t in q.prompt], q.max_new_tokens)
    steps, events = 0, []
    while not e.idle():
        e.step()
        steps += 1
        events += [list(x) for x in e.poll_events()]
    stats = e.runner_stats()
    e.shutdown()
    return events, stats, steps


def main(out):
    dist.init_process_group("gloo", timeout=timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    requests = prefix_tree_requests(**WORKLOAD)
    mine = router.by_root([q.root for q in requests], world, rank)
    events, stats, steps = serve(mine, requests)
    mine_stats = {k: int(v) for k, v in stats.items()}
    total = router.gather_counters({"forward_tokens": mine_stats["forward_tokens"],
                                    "prefix_hits": mine_stats["prefix_hits"], "requests": len(mine)}, dist)
    with open(os.path.join(out, f"rank{rank}.json"), "w") as f:
        json.dump({"rank": rank, "world": world, "indices": mine, "events": events, "stats": mine_stats,
                   "steps": steps, "total": total}, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
