"""Lockstep parity helpers shared by the GPU parity tests (test infrastructure).

The method is the reference's own GPU-vs-CPU check (benchmarks/GpuDecodeBenchmark.cpp:347-375):
the reference decodes each sequence greedily on the CPU; the device decodes the same sequences
stacked in one batch and is fed the reference's token at every step, so one near tie cannot
derail the rest of a sequence. Every logit must satisfy |gpu - cpu| <= 1e-5 + 1e-4 |cpu|; a step
whose argmax differs must be a near tie. A near-tie step is one where the reference's top-two gap
is at most twice the largest |gpu - cpu| of that row (the reference counts them the same way,
benchmarks/GpuDecodeBenchmark.cpp:363-366).
"""
from __future__ import annotations

import multiprocessing as mp
import os
from dataclasses import dataclass, field

import numpy as np

BOS = 2


@dataclass
class LockstepReport:
    worst: float = 0.0                      # largest |gpu - cpu| / (1e-5 + 1e-4 |cpu|)
    steps: int = 0                          # (sequence, step) pairs compared
    near_ties: list = field(default_factory=list)    # (seq, step) with gap <= 2 max|diff|
    mismatches: list = field(default_factory=list)   # (seq, step, near_tie) where ids differ
    worst_at: tuple = (-1, -1)

    def summary(self) -> str:
        return (f"{self.steps} steps compared, worst tolerance ratio {self.worst:.4f} at "
                f"{self.worst_at}, {len(self.near_ties)} near-tie steps, "
                f"{len(self.mismatches)} argmax differences")


def compare_row(rep: LockstepReport, i: int, t: int, got_row, want_row, got_id, want_id):
    got = np.asarray(got_row, np.float64)
    want = np.asarray(want_row, np.float64)
    diff = np.abs(got - want)
    ratio = float(np.max(diff / (1e-5 + 1e-4 * np.abs(want))))
    if ratio > rep.worst:
        rep.worst, rep.worst_at = ratio, (i, t)
    top2 = np.partition(want, -2)[-2:]
    tie = bool(top2[1] - top2[0] <= 2.0 * diff.max())
    if tie:
        rep.near_ties.append((i, t))
    if int(got_id) != int(want_id):
        rep.mismatches.append((i, t, tie))
    rep.steps += 1


def gpu_lockstep(kv, slots, srcs, want_ids, want_logits, steps, encode=True) -> LockstepReport:
    """Runs the device in lockstep with the reference. want_ids [n, steps]; want_logits(t) gives
    the reference's logits rows [n, V] of step t."""
    if encode:
        kv.encode(slots, srcs)
    rep = LockstepReport()
    feed = np.full(len(slots), BOS, np.int32)
    for t in range(steps):
        nxt, lg = kv.decode_step(slots, feed, want_logits=True)
        wl = want_logits(t)
        for i in range(len(slots)):
            compare_row(rep, i, t, lg[i], wl[i], nxt[i], want_ids[i][t])
        feed = np.asarray([want_ids[i][t] for i in range(len(slots))], np.int32)
    return rep


def distinct_stream_pairs(ids) -> float:
    """Fraction of sequence pairs whose greedy id streams differ."""
    n = len(ids)
    pairs = [(a, b) for a in range(n) for b in range(a + 1, n)]
    return sum(not np.array_equal(ids[a], ids[b]) for a, b in pairs) / max(len(pairs), 1)


# ---- the reference build in worker processes (spawned: no CUDA state is inherited) ----

def _ref_worker(job):
    cfg_name, seed, scheme, src, steps = job
    from adai_b200 import config
    from adai_b200.synth import make_weights
    from oracle.pyoracle import Ref
    cfg = getattr(config, cfg_name)
    w = make_weights(cfg, seed, affine=True, scheme=scheme)
    return Ref().model(cfg, w).generate(np.asarray(src, np.int32), steps, want_logits=True)


def reference_generate_parallel(cfg_name, seed, scheme, srcs, steps):
    """The reference's greedy decode of every source (ids [n, steps], logits [n, steps, V]), one
    single-threaded worker process per source (the reference decodes sequences one after
    another; the workers only spread them over the host's cores)."""
    n = len(srcs)
    old = os.environ.get("OMP_NUM_THREADS")
    os.environ["OMP_NUM_THREADS"] = "1"
    try:
        with mp.get_context("spawn").Pool(max(1, min(n, os.cpu_count() or 1))) as pool:
            res = pool.map(_ref_worker, [(cfg_name, seed, scheme, s, steps) for s in srcs])
    finally:
        if old is None:
            os.environ.pop("OMP_NUM_THREADS", None)
        else:
            os.environ["OMP_NUM_THREADS"] = old
    return np.stack([r[0] for r in res]), np.stack([r[1] for r in res])
