"""Stream-parallel (stream-DP) host logic on two CPU ranks over gloo: each
rank gets its own disjoint streams whose token ids match the library's
generator (gdn_synth_token, via the oracle's copy of it), the timing
reduction returns the slowest rank's time on every rank, and the job's
throughput counts every rank's tokens over that time. The decode itself has
no collective, so this is the whole cross-rank contract of bench.py."""
from __future__ import annotations

import os
import socket

import pytest
import torch.multiprocessing as mp

from gateddeltanet_b200 import workload as w


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, q) -> None:
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        streams = w.rank_streams(rank, world, per_rank=2)
        toks = {s: w.token_stream(s, 8, w.SHAPE["vocab"]) for s in streams}
        elapsed = 1.0 + rank  # rank 1 is the slow one
        slowest = w.max_over_ranks(elapsed)
        dist.barrier()
        q.put((rank, streams, toks, slowest))
    finally:
        dist.destroy_process_group()


def test_two_rank_stream_dp():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, s0, t0, m0), (r1, s1, t1, m1) = results
    assert (r0, r1) == (0, 1)
    assert s0 == [0, 1] and s1 == [2, 3]                 # disjoint stream blocks
    assert m0 == m1 == 2.0                               # both see the slowest rank's time
    assert w.job_tokens_per_s(world, 100, m0) == 100.0   # 200 tokens over 2 s
    import oracle_lib
    lib = oracle_lib.load()
    for toks in (t0, t1):
        for s, ids in toks.items():
            assert ids == [lib.gdn_oracle_synth_token(w.STREAM_SEED, s, i, w.SHAPE["vocab"]) for i in range(8)]
    assert t0[0] != t1[2]


def test_rank_streams_rejects_bad_layout():
    with pytest.raises(ValueError):
        w.rank_streams(2, 2)
    with pytest.raises(ValueError):
        w.job_tokens_per_s(1, 1, 0.0)
