"""The N > 1 path of bench.py on the CPU: two gloo ranks (processes started with `spawn`, rendezvous on 127.0.0.1)
run the bench's own helpers - the window sharding the encoder, decoder and log-mel objects use (every window on
exactly one rank, longest first to the least-loaded rank, as p2_b200_encode_windows assigns windows to GPUs), the
barrier, and the max-over-ranks timing that turns per-rank times into whole-job throughput. The path has no
collective on the data: the ranks exchange only timings."""
import os
import socket
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import json
    import torch.distributed as dist
    sys.path.insert(0, str(ROOT))
    import __graft_entry__ as ge
    ge.load_package()   # the synthetic workload's window lengths come from phonon2_b200.model
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        frames, _ = bench.encoder_workload("long-audio")
        mine = bench.shard_windows(frames, world)[rank]
        bench.barrier(world)
        # a per-rank "time": the slowest rank decides the whole job's time
        slowest = bench.max_over_ranks(float(sum(frames[w] for w in mine)), world)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump({"mine": mine, "slowest": slowest, "all": gathered, "frames": frames}, f)
    finally:
        dist.destroy_process_group()


def test_shard_windows_partition(pkg):
    import bench
    frames, _ = bench.encoder_workload("long-audio")
    for world in (1, 2, 3, 4, 8):
        shards = bench.shard_windows(frames, world)
        flat = sorted(w for s in shards for w in s)
        assert flat == list(range(len(frames)))   # every window on exactly one rank
        loads = [sum(frames[w] for w in s) for s in shards]
        assert max(loads) - min(loads) <= max(frames)   # longest first to the least loaded: within one window
        assert all(s == sorted(s) for s in shards)    # each rank keeps its windows in their original order


def test_two_gloo_ranks(tmp_path):
    import json
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a gloo rank did not finish")
        assert p.exitcode == 0
    res = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(world)]
    frames = res[0]["frames"]
    union = sorted(w for r in res for w in r["mine"])
    assert union == list(range(len(frames)))
    loads = [sum(frames[w] for w in r["mine"]) for r in res]
    assert all(r["slowest"] == max(loads) for r in res)   # every rank sees the slowest rank's value
    assert res[0]["all"] == res[1]["all"] == [r["mine"] for r in res]


def test_plane_bytes_of_the_model(pkg):
    """The plane stream figure's numerator: the 216 five-value tensors' planes and magnitudes, 229 MB."""
    import bench
    from phonon2_b200 import model as M
    assert bench.plane_bytes(M.SyntheticModel(seed=1)) == 230_031_360
