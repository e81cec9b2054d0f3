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
h * 256 + v of the state phase) and the conv-tail channel of q/k/v row r
(unit r of the QKVGAB phase, 4H + 2 nh units) are updated only by the rank
that owns the unit. merge_state() reassembles the full state from the ranks'
downloads.
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


def merge_state(parts: Sequence[tuple[np.ndarray, np.ndarray]], dims: dict, grid: int):
    """Full (rec, conv) from every rank's download, rank order.

    rec is the host layout [L][h][k][v], conv [L][q,k,v][row][H] (the ABI's
    .gdnstate order)."""
    world = len(parts)
    L, nh, dk, H = dims["layers"], dims["heads"], dims["head_dim"], dims["hidden"]
    W = dims["conv"] - 1
    cols = nh * dk
    col_rank = owner_rank(np.arange(cols), cols, grid, world).reshape(nh, dk)        # [h][v]
    qkv_total = 4 * H + 2 * nh
    ch_rank = owner_rank(np.arange(3 * H), qkv_total, grid, world).reshape(3, H)     # [kind][d]
    rec = np.empty(L * nh * dk * dk, dtype=np.float32).reshape(L, nh, dk, dk)
    conv = np.empty(L * 3 * W * H, dtype=np.float32).reshape(L, 3, W, H)
    for r, (pr, pc) in enumerate(parts):
        pr = np.asarray(pr, dtype=np.float32).reshape(L, nh, dk, dk)
        pc = np.asarray(pc, dtype=np.float32).reshape(L, 3, W, H)
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
