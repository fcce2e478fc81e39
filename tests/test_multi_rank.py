"""Request sharding across ranks (one process per GPU, no data-path collective).

The routing functions partition every workload exactly once and keep submission
order; a world-size-2 run over gloo (tests/multi_rank_worker.py under
torch.distributed.run, device-free scripted runners) gives each rank exactly the
outcome of serving its shard alone, and the counters gathered after serving are
the sums over the shards.
"""
import json
import os
import socket
import subprocess
import sys

import pytest

from tinyinfer_b200 import router
from tinyinfer_b200.synthetic import prefix_tree_requests

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_round_robin_partitions_in_order(world):
    parts = router.partition(37, world)
    flat = sorted(i for p in parts for i in p)
    assert flat == list(range(37))
    for p in parts:
        assert p == sorted(p)
    assert max(map(len, parts)) - min(map(len, parts)) <= 1


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_by_root_keeps_each_root_on_one_rank(world):
    reqs = prefix_tree_requests(seed=9, count=300, roots=16, root_tokens=32, segment=8, min_len=8, max_len=64,
                                min_new=1, max_new=4, vocabulary=100)
    roots = [q.root for q in reqs]
    parts = router.partition(roots, world, "by_root")
    assert sorted(i for p in parts for i in p) == list(range(len(reqs)))
    seen = {}
    for rank, p in enumerate(parts):
        assert p == sorted(p)
        for i in p:
            assert seen.setdefault(roots[i], rank) == rank
    per_rank = [len({roots[i] for i in p}) for p in parts]
    assert max(per_rank) - min(per_rank) <= 1  # 16 roots: 2 per rank at 8 ranks
    if world == 8:
        assert per_rank == [2] * 8


def test_router_rejects_bad_rank():
    with pytest.raises(ValueError):
        router.round_robin(4, 2, 2)
    with pytest.raises(ValueError):
        router.by_root([0, 1], 0, 0)


def test_prefix_tree_requests_share_node_tokens():
    reqs = prefix_tree_requests(seed=1, count=200, roots=2, root_tokens=20, branching=2, depth=2, segment=6,
                                min_len=30, max_len=40, min_new=1, max_new=2, vocabulary=50)
    by_node = {}
    for q in reqs:
        full = 20 + 6 * len(q.path)
        key = (q.root, q.path)
        prefix = tuple(q.prompt[:min(full, q.prompt.size)])
        if key in by_node:
            a, b = by_node[key], prefix
            n = min(len(a), len(b))
            assert a[:n] == b[:n]
        by_node[key] = prefix
        assert 30 <= q.prompt.size <= 40 and 1 <= q.max_new_tokens <= 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_serve_their_shards(built, tmp_path):
    import multi_rank_worker as w

    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", os.path.join(HERE, "multi_rank_worker.py"),
           str(tmp_path)]
    env = dict(os.environ, OMP_NUM_THREADS="1")
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=240)
    assert proc.returncode == 0, proc.stderr[-3000:]
    outs = [json.load(open(tmp_path / f"rank{r}.json")) for r in range(2)]
    requests = prefix_tree_requests(**w.WORKLOAD)
    assert sorted(outs[0]["indices"] + outs[1]["indices"]) == list(range(len(requests)))
    for o in outs:
        events, stats, steps = w.serve(o["indices"], requests)
        assert o["events"] == json.loads(json.dumps(events))
        assert o["stats"] == {k: int(v) for k, v in stats.items()}
        assert o["steps"] == steps
        finished = {e[0] for e in o["events"] if e[2] is not None}
        assert finished == {f"q{i}" for i in o["indices"]}
    total = outs[0]["total"]
    assert total == outs[1]["total"]
    assert total["forward_tokens"] == sum(o["stats"]["forward_tokens"] for o in outs)
    assert total["prefix_hits"] == sum(o["stats"]["prefix_hits"] for o in outs)
    assert total["requests"] == len(requests)
    assert sum(o["stats"]["prefix_hits"] for o in outs) > 0
