"""Host-side logic of the stream-parallel decode workload (no GPU needed).

Stream-DP: every rank (one process per GPU) decodes its own independent
batch-1 streams with a full weight replica; there is no data-path collective.
The only cross-rank steps are a barrier around the timed region and the
max-over-ranks of the measured time; the job's throughput is the tokens of
all ranks over that maximum (weak scaling: fixed work per GPU).

Token streams are the seeded uniform ids of gateddeltanet_b200/csrc/
gdn_synth.h (gdn_synth_token), re-stated here so drivers need no library
call to build them.
"""
from __future__ import annotations

# GDN-1.3B (BASELINE config[0] header) and the seeds of the benchmark workload.
SHAPE = dict(vocab=32000, hidden=2048, layers=24, heads=8, head_dim=256, inter=5632, conv=4)
SEED = 1234
STREAM_SEED = 99
PROMPT_OFFSET = 1 << 20  # prompt ids come from the same stream, far from the teacher ids

MASK = (1 << 64) - 1
_GOLDEN = 0x9E3779B97F4A7C15
STREAM_TOKENS = 0x70000000  # GDN_SYNTH_STREAM_TOKENS


def _mix64(z: int) -> int:
    z = (z + _GOLDEN) & MASK
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK
    return z ^ (z >> 31)


def _key(seed: int, stream: int) -> int:
    return _mix64(seed ^ _mix64((stream * 0xD1B54A32D192ED03 + 0x1234567) & MASK))


def token_stream(stream: int, n: int, vocab: int, offset: int = 0, seed: int = STREAM_SEED) -> list[int]:
    """Ids offset .. offset + n - 1 of seeded stream `stream` (gdn_synth_token)."""
    key = _key(seed, STREAM_TOKENS + stream)
    out = []
    for i in range(offset, offset + n):
        r = _mix64((key + (i + 1) * _GOLDEN) & MASK)
        out.append(((r >> 32) * vocab) >> 32)
    return out


def rank_streams(rank: int, world: int, per_rank: int = 1) -> list[int]:
    """Stream ids decoded by `rank`: a disjoint block of `per_rank` streams."""
    if not 0 <= rank < world or per_rank < 1:
        raise ValueError("bad rank/world/per_rank")
    return list(range(rank * per_rank, (rank + 1) * per_rank))


def max_over_ranks(x: float, device=None) -> float:
    """Maximum of x over all ranks (identity without a process group)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_tokens_per_s(world: int, tokens_per_rank: int, max_seconds: float) -> float:
    """Whole-job throughput: every rank's tokens over the slowest rank's time."""
    if max_seconds <= 0:
        raise ValueError("non-positive time")
    return world * tokens_per_rank / max_seconds
