"""Host logic of tensor-parallel decode, on the CPU.

* owner_rank / unit_owner reproduce the decode kernel's unit partition over
  the global CTAs (c * total // ncta, gdn_decode.cu span_of) for every phase
  of GDN-1.3B at 2..8 GPUs with the grid the library picks (tp_grid), and
  give every rank a share;
* merge_state rebuilds the full recurrent state and conv tails from ranks that
  each hold only their own columns and channels (the rest garbage);
* attach() over two gloo ranks gathers the tokens in rank order, hands each
  run state the same list and its own rank, and ends with a barrier.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from gateddeltanet_b200 import tensor_parallel as tp

FULL = dict(vocab=32000, hidden=2048, layers=24, heads=8, head_dim=256, inter=5632, conv=4)
SMALL = dict(vocab=4096, hidden=512, layers=2, heads=2, head_dim=256, inter=1536, conv=4)


def _kernel_partition(total, ncta):
    return [(c * total // ncta, (c + 1) * total // ncta) for c in range(ncta)]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_owner_matches_the_kernel_partition(world):
    grid = tp.tp_grid(FULL, world, 148)
    assert grid == (88 if world == 8 else 148)  # 704 gate/up tiles bind at 8 GPUs
    ncta = grid * world
    for name, total in tp.phase_units(FULL).items():
        assert total >= ncta, name
        owner = tp.unit_owner(np.arange(total), total, ncta)
        for c, (u0, u1) in enumerate(_kernel_partition(total, ncta)):
            assert (owner[u0:u1] == c).all()
        ranks = tp.owner_rank(np.arange(total), total, grid, world)
        assert set(ranks.tolist()) == set(range(world))
        assert (np.diff(ranks) >= 0).all()


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_image_geometry_matches_the_library_and_its_maps_are_bijections(world):
    """The tensor-parallel weight image's chunk geometry: the library's choice
    (gdn_b200_test_image_geometry, host code only) equals the restatement in
    tensor_parallel.image_geometry, every chunk fits a ring slot, and the
    layout maps the device re-layout gathers through are bijections for that
    geometry and the one-GPU one."""
    import ctypes

    import gateddeltanet_b200 as gdn
    from gateddeltanet_b200 import build
    build.build()
    L = gdn.lib()
    for dims in (FULL, SMALL):
        grid = tp.tp_grid(dims, world, 148)
        ncta = grid * world
        geom = (ctypes.c_uint32 * 4)()
        assert L.gdn_b200_test_image_geometry(dims["hidden"], dims["inter"], dims["vocab"], ncta, geom, 1) == 0, \
            gdn.last_error()
        got = tuple(geom)
        assert got == tp.image_geometry(dims, ncta)
        H = dims["hidden"]
        g_qkvg, g_gu, g_lm, ng = got
        for G in (g_qkvg, g_gu, g_lm):
            assert (H // 64) % G == 0
        assert ng % 8 == 0
        for tiles, tile_rows, G in ((4 * H // 8, 8, g_qkvg), (2 * dims["inter"] // 16, 16, g_gu),
                                    (dims["vocab"] // 16, 16, g_lm)):
            assert min(tp.PASS_TILES, -(-tiles // ncta)) * G * tile_rows * 128 <= tp.SLOT_BYTES
        assert -(-H // ncta) * min(ng, max(H, dims["inter"]) // 64) * 128 <= tp.SLOT_BYTES
    # the one-GPU grid gives the one-GPU image; the measured tensor-parallel grids these
    expect = {1: (4, 2, 2, 16), 2: (8, 4, 2, 32), 4: (16, 8, 4, 64), 8: (16, 16, 4, 80)}
    assert tp.image_geometry(FULL, tp.tp_grid(FULL, world, 148) * world) == expect[world]


def test_image_geometry_rejects_unsupported_sizes():
    import ctypes

    import gateddeltanet_b200 as gdn
    from gateddeltanet_b200 import build
    build.build()
    L = gdn.lib()
    geom = (ctypes.c_uint32 * 4)()
    assert L.gdn_b200_test_image_geometry(2000, 5632, 32000, 296, geom, 0) == -1
    assert "multiples of 512" in gdn.last_error()
    assert L.gdn_b200_test_image_geometry(2048, 5632, 32000, 0, geom, 0) == -1


@pytest.mark.parametrize("world", [2, 3])
def test_merge_state_takes_each_unit_from_its_owner(world):
    dims = SMALL
    grid = tp.tp_grid(dims, world, 148)
    L, nh, dk, H = dims["layers"], dims["heads"], dims["head_dim"], dims["hidden"]
    rng = np.random.default_rng(1)
    rec = rng.standard_normal(L * nh * dk * dk).astype(np.float32)
    conv = rng.standard_normal(L * 3 * 3 * H).astype(np.float32)
    col_rank = tp.owner_rank(np.arange(nh * dk), nh * dk, grid, world).reshape(nh, dk)
    # conv channel of row r: the owner of r's 8-row QKVG tile
    ch_rank = tp.owner_rank(np.arange(3 * H) // 8, 4 * H // 8, grid, world).reshape(3, H)
    parts = []
    for r in range(world):
        pr = np.full((L, nh, dk, dk), np.nan, dtype=np.float32)
        pc = np.full((L, 3, 3, H), np.nan, dtype=np.float32)
        m = np.broadcast_to((col_rank == r)[None, :, None, :], pr.shape)
        pr[m] = rec.reshape(pr.shape)[m]
        mc = np.broadcast_to((ch_rank == r)[None, :, None, :], pc.shape)
        pc[mc] = conv.reshape(pc.shape)[mc]
        parts.append((pr.reshape(-1), pc.reshape(-1), grid, r, world))
    m_rec, m_conv = tp.merge_state(parts, dims)
    assert np.array_equal(m_rec, rec) and np.array_equal(m_conv, conv)
    # the grid travels with the parts; parts from another attachment are refused
    with pytest.raises(ValueError):
        tp.merge_state([(a, b, grid, (r + 1) % world, world) for r, (a, b, *_) in enumerate(parts)], dims)


class _FakeRunState:
    def __init__(self, rank):
        self.rank = rank
        self.calls = []

    def tp_token(self):
        return bytes([self.rank]) * 128

    def tp_attach(self, rank, world, tokens):
        self.calls.append((rank, world, list(tokens)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rs = _FakeRunState(rank)
        got = tp.attach(rs)
        q.put((rank, got, rs.calls))
    finally:
        dist.destroy_process_group()


def test_attach_over_two_gloo_ranks():
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
    tokens = [bytes([0]) * 128, bytes([1]) * 128]
    for rank, (r, got, calls) in enumerate(results):
        assert r == rank and got == (rank, world)
        assert calls == [(rank, world, tokens)]
