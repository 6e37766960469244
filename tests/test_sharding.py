"""Multi-process host logic of the utterance-sharded run on CPU: world_size 2
gloo ranks each take their block of utterances, compute per-utterance
results, and the gather / max-over-ranks collectives reassemble exactly the
single-process answer."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from i_whisper_b200.sharding import gather_rows, max_over_ranks, shard_bounds, window_seeds


def test_shard_bounds_cover_every_utterance_once():
    for n in (0, 1, 7, 256, 257, 512):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                a, b = shard_bounds(n, world, r)
                assert 0 <= a <= b <= n
                seen += list(range(a, b))
            assert seen == list(range(n))
    with pytest.raises(ValueError):
        shard_bounds(8, 2, 2)


def test_window_seeds_recycle():
    assert window_seeds(30, 35) == [30, 31, 0, 1, 2]


def _utterance_result(g: int) -> np.ndarray:
    # stand-in for one utterance's decoded tokens: depends on its index only
    rng = np.random.default_rng(1000 + g)
    return rng.integers(0, 51865, 12).astype(np.int64)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, per_rank, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a, b = shard_bounds(per_rank * world, world, rank)
        rows = torch.from_numpy(np.stack([_utterance_result(g) for g in range(a, b)]))
        full = gather_rows(rows)
        t = max_over_ranks(10.0 + rank)
        if rank == 0:
            np.save(os.path.join(out_dir, "full.npy"), full.numpy())
            np.save(os.path.join(out_dir, "t.npy"), np.array([t]))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_reassemble(tmp_path):
    world, per_rank = 2, 5
    mp.start_processes(_rank_main, args=(world, _free_port(), per_rank, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    full = np.load(tmp_path / "full.npy")
    want = np.stack([_utterance_result(g) for g in range(world * per_rank)])
    assert np.array_equal(full, want)
    assert float(np.load(tmp_path / "t.npy")[0]) == 11.0


def test_single_process_passthrough():
    t = torch.arange(6).reshape(3, 2)
    assert gather_rows(t) is t
    assert max_over_ranks(3.5) == 3.5


def test_peer_monitor_in_one_process():
    from i_whisper_b200.sharding import PeerFailure, PeerMonitor
    store = dist.HashStore()
    mons = [PeerMonitor(store, r, 3, timeout_s=0.2) for r in range(3)]
    for m in mons:
        m.wait_peers(0)          # nothing to wait for before the first step
        m.post(0)
    for m in mons:
        m.wait_peers(1)
    mons[0].post(1)
    mons[2].post(1)              # rank 1 never finishes step 1
    with pytest.raises(PeerFailure, match=r"rank\(s\) \[1\] did not finish step 1"):
        mons[0].wait_peers(2)
    with pytest.raises(ValueError):
        PeerMonitor(store, 3, 3)


def _failing_rank_main(rank, world, port, out_dir):
    import datetime
    from i_whisper_b200.sharding import PeerFailure, PeerMonitor, default_store
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    mon = PeerMonitor(default_store(), rank, world, timeout_s=2.0)
    mon.wait_peers(0)
    dist.all_reduce(torch.ones(1))   # step 0, both ranks
    mon.post(0)
    if rank == 1:
        os._exit(0)                  # leaves between steps, nothing in flight
    outcome = {}
    mon.wait_peers(1)                # rank 1 did finish step 0
    mon.post(1)                      # step 1: this rank's own utterances, no collective
    try:
        mon.wait_peers(2)
        outcome["monitor"] = "no error"
    except PeerFailure as e:
        outcome["monitor"] = str(e)
    t0 = __import__("time").monotonic()
    try:
        dist.all_reduce(torch.ones(1))  # the collective the monitor would have skipped
        outcome["collective"] = "no error"
    except Exception as e:  # noqa: BLE001 -- any error class ends the wait
        outcome["collective"] = type(e).__name__
    outcome["collective_s"] = __import__("time").monotonic() - t0
    np.save(os.path.join(out_dir, "outcome.npy"), np.array([repr(outcome)]))
    os._exit(0)


def test_rank_that_leaves_is_detected_on_the_host(tmp_path):
    """Rank 1 exits after step 0. Rank 0 runs its own step 1 (sharded work
    has no collective) and learns from the store before step 2 that rank 1
    never finished step 1 (PeerFailure within the monitor's 2 s); a collective
    attempted anyway ends with an error within the process group's short
    timeout instead of waiting for good."""
    mp.start_processes(_failing_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn",
                       join=True)
    outcome = eval(str(np.load(tmp_path / "outcome.npy")[0]))
    assert "rank(s) [1] did not finish step 1" in outcome["monitor"]
    assert outcome["collective"] != "no error"
    assert outcome["collective_s"] < 30
