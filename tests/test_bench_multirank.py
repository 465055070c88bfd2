"""The multi-GPU side of bench.py on CPU: two ranks over gloo (127.0.0.1).

`bench.py --gpus N` runs one process per GPU. The packed batches are dealt
to the ranks longest-processing-time first on their forward cost
(`rank_share`), and the timing stats are combined across ranks
(`reduce_timing`: max of the times, sum of the tokens); rank 0 prints the
line. The same helpers run here on CPU tensors with the gloo backend."""
import socket
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# the costs of 11 batches, heaviest first as the longest-first planner leaves them
COSTS = [9.0, 8.0, 7.0, 6.0, 5.0, 4.0, 3.0, 2.5, 2.0, 1.5, 1.0]


def _rank(rank: int, world: int, port: int, out_dir: str) -> None:
    import json
    from datetime import timedelta

    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    import bench

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        got = bench.reduce_timing(10.0 + rank, 20.0 + 3 * rank, 100 * (rank + 1), world, "cpu")
        share = bench.rank_share(list(range(11)), COSTS, rank, world, steps=50, warmup=3)
        spread = bench.rank_share(list(range(101)), [1.0] * 101, rank, world, steps=4, warmup=3)
        (Path(out_dir) / f"rank{rank}.json").write_text(json.dumps({"reduce": got, "share": share,
                                                                   "spread": spread}))
    finally:
        dist.destroy_process_group()


def test_two_ranks_share_batches_and_reduce_timing(tmp_path):
    import json

    import torch.multiprocessing as mp

    world = 2
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    res = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(world)]
    for r in res:
        assert r["reduce"] == [11.0, 23.0, 300.0]  # max, max, sum
    # whole shares (steps >= share): disjoint, together every batch, warm-up from the share
    s0, s1 = res[0]["share"], res[1]["share"]
    assert set(s0).isdisjoint(s1) and set(s0) | set(s1) == set(range(11))
    assert len(s0) == len(s1) == 53 and s0[:3] == s0[3:6]
    # LPT: batch 0 to rank 0, batch 1 to rank 1, then each to the lighter rank;
    # the loads differ by at most the lightest batch
    loads = [sum(COSTS[b] for b in set(r)) for r in (s0, s1)]
    assert abs(loads[0] - loads[1]) <= min(COSTS)
    assert s0[3] == 0 and s1[3] == 1  # each share runs heaviest first
    # spread (steps < share): evenly spaced over the rank's share, first and last included
    sp0, sp1 = res[0]["spread"], res[1]["spread"]
    assert len(sp0) == len(sp1) == 7 and sp0[:3] == sp0[3:6]
    assert set(sp0[3:]).isdisjoint(sp1[3:])


def test_single_rank_needs_no_process_group():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.reduce_timing(5.0, 6.0, 7, 1, "cpu") == (5.0, 6.0, 7.0)
    with pytest.raises(Exception):
        bench.rank_share([], [], 0, 1, 2, 1)  # an empty share has nothing to time
