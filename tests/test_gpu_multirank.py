"""The batch-sharded multi-GPU path on the device: two spawned ranks (gloo for the host-side
gather; one process and one context per rank, on GPU rank % device count) each encode and
greedily decode the shard that adai_b200/parallel.py::balanced_shards gives them; the gathered
ids must equal a one-process device run of the whole batch id for id (rows are independent in
every kernel, so the batch composition must not change a single token) and the oracle's greedy
decode. On a one-GPU box both ranks share the GPU: their kernels never wait on one another, only
the host-side gather does.
"""
import os
import socket

import numpy as np
import pytest

from adai_b200.config import TINY
from adai_b200.synth import make_sources, make_weights

pytestmark = pytest.mark.gpu

N_SEQ, STEPS, BOS = 11, 6, 2
SRC_LENS = (5, 48)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _decode(device, srcs, idx):
    from adai_b200.api import Context
    with Context(device) as c:
        c.upload(TINY, make_weights(TINY, 6, scheme="reference"))
        kv = c.kv_arena(max(1, len(idx)), STEPS + 1, SRC_LENS[1])
        slots = list(range(len(idx)))
        kv.encode(slots, [srcs[i] for i in idx])
        ids = kv.generate(slots, [BOS] * len(idx), STEPS)
        kv.close()
    return ids


def _rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch
    import torch.distributed as dist

    from adai_b200.parallel import balanced_shards
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        srcs = make_sources(TINY, N_SEQ, SRC_LENS, 9)
        mine = balanced_shards([len(s) for s in srcs], world)[rank]
        ids = _decode(rank % torch.cuda.device_count(), srcs, mine)
        parts = [None] * world
        dist.all_gather_object(parts, (list(mine), ids.tolist()))
        if rank == 0:
            out = np.full((N_SEQ, STEPS), -1, np.int64)
            for idx, rows in parts:
                for i, row in zip(idx, rows):
                    out[i] = row
            np.save(os.path.join(out_dir, "ids.npy"), out)
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_two_device_ranks_match_one_process_and_the_oracle(tmp_path, port):
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    got = np.load(os.path.join(tmp_path, "ids.npy"))
    assert (got >= 0).all()
    srcs = make_sources(TINY, N_SEQ, SRC_LENS, 9)
    whole = _decode(0, srcs, list(range(N_SEQ)))
    np.testing.assert_array_equal(got, whole)
    model = port.model(TINY, make_weights(TINY, 6, scheme="reference"))
    want = np.asarray([model.generate(s, STEPS)[0] for s in srcs])
    np.testing.assert_array_equal(got, want)
    # the ids tell the sequences apart (a shard mix-up would show)
    assert len({tuple(r) for r in got.tolist()}) >= N_SEQ // 2
