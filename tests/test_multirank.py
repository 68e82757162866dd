"""Host logic of the multi-GPU path (adai_b200/parallel.py) on CPU: batch shards cover every
sequence once, two gloo ranks that each decode their shard reproduce the one-process result in
batch order, the max-over-ranks timing, and a rank that fails is reported on every rank.

The per-rank "device" work here is the CPU oracle's greedy decode of the tiny model, so the test
exercises the sharding, gathering and failure paths without a GPU.
"""
import os
import socket

import numpy as np
import pytest

from adai_b200.config import TINY
from adai_b200.parallel import balanced_shards, shard_ranges
from adai_b200.synth import make_sources, make_weights

N_SEQ, STEPS = 7, 4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_ranges_cover_the_batch_once():
    for n in (0, 1, 7, 128, 1024):
        for world in (1, 2, 3, 8):
            rs = shard_ranges(n, world)
            assert len(rs) == world
            seen = [b for lo, hi in rs for b in range(lo, hi)]
            assert seen == list(range(n))
            sizes = [hi - lo for lo, hi in rs]
            assert max(sizes) - min(sizes) <= 1
            for b in range(n):   # sequence b lives on rank floor(b * world / n)
                r = b * world // n
                assert rs[r][0] <= b < rs[r][1]


def test_balanced_shards_even_out_source_lengths():
    lens = make_sources(TINY, 64, (128, 1024), 5)
    lens = [len(s) for s in lens]
    for world in (2, 4, 8):
        sh = balanced_shards(lens, world)
        assert sorted(i for s in sh for i in s) == list(range(64))
        assert max(len(s) for s in sh) <= -(-64 // world)
        loads = [sum(lens[i] for i in s) for s in sh]
        contiguous = [sum(lens[lo:hi]) for lo, hi in shard_ranges(64, world)]
        assert max(loads) - min(loads) <= max(contiguous) - min(contiguous)
        assert max(loads) - min(loads) <= max(lens)
    with pytest.raises(ValueError):
        balanced_shards(lens, 0)


def _rank_main(rank, world, port, result_dir, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    from adai_b200.parallel import max_over_ranks, run_sharded
    from oracle.pyoracle import Port
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        w = make_weights(TINY, 4, affine=True)
        srcs = make_sources(TINY, N_SEQ, (3, 30), 4)
        model = Port().model(TINY, w)

        def decode(idx):
            if rank == fail_rank:
                raise RuntimeError("planted failure")
            return [model.generate(srcs[i], STEPS)[0].tolist() for i in idx]

        shards = balanced_shards([len(s) for s in srcs], world)
        assert max_over_ranks(float(rank + 1)) == float(world)
        try:
            got = run_sharded(decode, shards, N_SEQ)
            status = "ok"
        except RuntimeError as e:
            got, status = None, str(e)
        if rank == 0:
            np.save(os.path.join(result_dir, "ids.npy"),
                    np.asarray(got if got is not None else [], dtype=np.int64))
        with open(os.path.join(result_dir, f"status{rank}.txt"), "w") as f:
            f.write(status)
    finally:
        dist.barrier()
        dist.destroy_process_group()


def _spawn(tmp_path, fail_rank):
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(2, _free_port(), str(tmp_path), fail_rank), nprocs=2, join=True)
    return [open(os.path.join(tmp_path, f"status{r}.txt")).read() for r in range(2)]


def test_two_gloo_ranks_match_one_process(tmp_path, port):
    status = _spawn(tmp_path, fail_rank=-1)
    assert status == ["ok", "ok"]
    got = np.load(os.path.join(tmp_path, "ids.npy"))
    w = make_weights(TINY, 4, affine=True)
    srcs = make_sources(TINY, N_SEQ, (3, 30), 4)
    model = port.model(TINY, w)
    want = np.asarray([model.generate(s, STEPS)[0] for s in srcs])
    np.testing.assert_array_equal(got, want)


def test_a_failing_rank_is_reported_on_every_rank(tmp_path):
    status = _spawn(tmp_path, fail_rank=1)
    for s in status:
        assert "rank 1" in s and "planted failure" in s, s
