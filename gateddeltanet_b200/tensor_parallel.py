"""Host side of tensor-parallel batch-1 decode.

One decode stream runs over `world` GPUs, one process (rank) per GPU. The
decode kernel's unit partitions -- GEMV output rows, recurrent-state columns,
LM-head rows -- run over the global CTAs of all GPUs: global CTA c of
world * grid takes units [c * total // (world * grid), (c + 1) * total //
(world * grid)) of a phase with `total` units, and GPU r holds the global
CTAs r * grid .. r * grid + grid - 1. Every output a CTA computes is stored
into every GPU's exchange region over NVLink (peer stores from inside the
kernel; no NCCL call on the data path), so each GPU reads the whole vector of
a phase from its own memory and the step equals the single-GPU step bit for
bit. The reference splits heads and the MLP instead and all-reduces the
hidden partials after the O and down projections; that
re-orders the reference's bank-chain sums, this does not.

State that stays per rank: recurrent-state column v of head h (unit
h * 256 + v of the state phase, nh * 256 units) and the conv-tail channel of
q/k/v row r (held by the CTA that owns row r's 8-row tile of the QKVG
projection, 4H / 8 tiles) are updated only by the rank that owns the unit.
After a tensor-parallel step the library refuses whole-state reads, prefill
and single-GPU decode on a run state until a full state is uploaded;
RunState.read_state_part() gives each rank's part and merge_state()
reassembles the full state from the parts.
"""
from __future__ import annotations

from typing import Sequence

import numpy as np


def unit_owner(u, total: int, ncta: int):
    """Global CTA whose range holds unit u (the largest c with c * total // ncta <= u)."""
    u = np.asarray(u, dtype=np.int64)
    return ((u + 1) * ncta + total - 1) // total - 1


def owner_rank(u, total: int, grid: int, world: int):
    """Rank holding unit u of a phase with `total` units."""
    return unit_owner(u, total, grid * world) // grid


QKVG_TILE_ROWS = 8  # rows of a QKVG tile (gdn_engine.h kTileRowsQKVG)
GU_TILE_ROWS = 16   # kTileRowsGU
LM_TILE_ROWS = 16   # kTileRowsLM


def phase_units(dims: dict) -> dict:
    """Units of each partitioned phase of the decode kernel: QKVG tiles,
    recurrent-state columns, O and down-projection rows, gate/up tiles,
    LM-head tiles."""
    H, nh, I, V = dims["hidden"], dims["heads"], dims["inter"], dims["vocab"]
    return {"qkvg_tiles": 4 * H // QKVG_TILE_ROWS, "state_cols": nh * dims["head_dim"], "o_rows": H,
            "down_rows": H, "gu_tiles": 2 * I // GU_TILE_ROWS, "lm_tiles": V // LM_TILE_ROWS}


def tp_grid(dims: dict, world: int, grid: int) -> int:
    """CTAs per GPU the library picks when `world` GPUs of `grid` SMs attach
    (gdn_b200_tp_attach): the largest g <= grid whose world * g CTAs all own
    units of every phase."""
    return min(grid, min(phase_units(dims).values()) // world)


SLOT_BYTES = 32768  # one slot of the decode kernel's 4-slot shared-memory ring
PASS_TILES = 7      # tiles of a tiled projection per pass


def image_geometry(dims: dict, ncta: int) -> tuple[int, int, int, int]:
    """Chunk geometry of the weight image gdn_b200_tp_attach builds for
    `ncta` CTAs over all GPUs: (groups of 64 columns per chunk of the QKVG,
    gate/up and LM-head tiles, groups per chunk of the O / DOWN rows). Each
    is the largest whose biggest copy -- a CTA's ceil(units / ncta) tiles
    (at most PASS_TILES a pass) or rows -- still fits a ring slot; the tiled
    counts are powers of two dividing hidden / 64, the row count a multiple
    of 8. At one GPU's 148 CTAs this is the one-GPU image (4, 2, 2, 16)."""
    H, I, V = dims["hidden"], dims["inter"], dims["vocab"]

    def wide(tiles: int, tile_rows: int) -> int:
        n = min(PASS_TILES, -(-tiles // ncta))
        g = 1
        while (H // 64) % (2 * g) == 0 and n * 2 * g * tile_rows * 128 <= SLOT_BYTES:
            g *= 2
        return g
    rows = -(-H // ncta)
    ng = min(SLOT_BYTES // (rows * 128) // 8 * 8, max(H, I) // 64)
    return (wide(4 * H // QKVG_TILE_ROWS, QKVG_TILE_ROWS), wide(2 * I // GU_TILE_ROWS, GU_TILE_ROWS),
            wide(V // LM_TILE_ROWS, LM_TILE_ROWS), ng)


def owner_maps(dims: dict, grid: int, world: int):
    """(col_rank [heads][256], ch_rank [3][hidden]): the rank that updates
    recurrent-state column v of head h, and the conv-tail channel of row d of
    q, k and v (the owner of the row's QKVG tile)."""
    nh, dk, H = dims["heads"], dims["head_dim"], dims["hidden"]
    cols = nh * dk
    col_rank = owner_rank(np.arange(cols), cols, grid, world).reshape(nh, dk)
    tiles = 4 * H // QKVG_TILE_ROWS
    ch_rank = owner_rank(np.arange(3 * H) // QKVG_TILE_ROWS, tiles, grid, world).reshape(3, H)
    return col_rank, ch_rank


def owned_values(rec: np.ndarray, conv: np.ndarray, dims: dict, grid: int, rank: int, world: int) -> bytes:
    """The recurrent-state and conv-tail values rank `rank` owns, in index
    order, as bytes: equal for a rank's part and the full state exactly when
    the part is right."""
    L, nh, dk, H = dims["layers"], dims["heads"], dims["head_dim"], dims["hidden"]
    W = dims["conv"] - 1
    col_rank, ch_rank = owner_maps(dims, grid, world)
    r4 = np.asarray(rec, dtype=np.float32).reshape(L, nh, dk, dk)
    c4 = np.asarray(conv, dtype=np.float32).reshape(L, 3, W, H)
    m = np.broadcast_to((col_rank == rank)[None, :, None, :], r4.shape)
    mc = np.broadcast_to((ch_rank == rank)[None, :, None, :], c4.shape)
    return r4[m].tobytes() + c4[mc].tobytes()


def merge_state(parts: Sequence[tuple], dims: dict, grid: int | None = None):
    """Full (rec, conv) from every rank's part, rank order.

    A part is (rec, conv) with the CTAs per GPU given as `grid`, or the tuple
    RunState.read_state_part() returns (rec, conv, grid, rank, world). rec is
    the host layout [L][h][k][v], conv [L][q,k,v][row][H] (the ABI's
    .gdnstate order)."""
    world = len(parts)
    grids = {int(p[2]) for p in parts if len(p) > 2}
    if grid is None:
        if len(grids) != 1:
            raise ValueError("merge_state: the parts disagree on the grid (or carry none): pass grid=")
        grid = grids.pop()
    for r, p in enumerate(parts):
        if len(p) > 4 and (int(p[3]) != r or int(p[4]) != world):
            raise ValueError(f"merge_state: part {r} is rank {p[3]} of {p[4]}, expected rank {r} of {world}")
    L, nh, dk, H = dims["layers"], dims["heads"], dims["head_dim"], dims["hidden"]
    W = dims["conv"] - 1
    col_rank, ch_rank = owner_maps(dims, grid, world)
    rec = np.empty(L * nh * dk * dk, dtype=np.float32).reshape(L, nh, dk, dk)
    conv = np.empty(L * 3 * W * H, dtype=np.float32).reshape(L, 3, W, H)
    for r, p in enumerate(parts):
        pr = np.asarray(p[0], dtype=np.float32).reshape(L, nh, dk, dk)
        pc = np.asarray(p[1], dtype=np.float32).reshape(L, 3, W, H)
        m = np.broadcast_to((col_rank == r)[None, :, None, :], rec.shape)
        rec[m] = pr[m]
        mc = np.broadcast_to((ch_rank == r)[None, :, None, :], conv.shape)
        conv[mc] = pc[mc]
    return rec.reshape(-1), conv.reshape(-1)


def attach(run_state, group=None) -> tuple[int, int]:
    """Join `run_state` to a tensor-parallel decode over the ranks of the
    torch.distributed process group (one run state per rank, each on its own
    GPU): gather every rank's token in rank order, attach, then a barrier so
    that no rank steps before every rank is attached. Returns (rank, world)."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    tokens: list = [None] * world
    dist.all_gather_object(tokens, run_state.tp_token(), group=group)
    run_state.tp_attach(rank, world, tokens)
    dist.barrier(group=group)
    return rank, world
