"""One rank of a tensor-parallel decode check (launched by tests/test_gpu_tp.py
under torch.distributed.run, one process per GPU).

Every rank loads the same seeded model and initial state, attaches its run
state to the others (gateddeltanet_b200.tensor_parallel.attach) and decodes a
teacher-forced stream, then a greedy continuation. Rank 0 then decodes the
same tokens on one GPU with a run state of its own and compares: tokens,
logits and the merged recurrent state and conv tails must be identical bit
for bit. Each rank also records that the library refuses whole-state reads,
saves, prefill and (after detaching) single-GPU decode of its partial state.
With --failure, rank 1 then sits out one step: rank 0's step must fail with
the exchange-wait timeout, and after every rank attaches again the decode
must again equal the single-GPU decode. The verdict goes to --out as JSON.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import gateddeltanet_b200 as gdn  # noqa: E402
from gateddeltanet_b200 import tensor_parallel as tp  # noqa: E402

DIMS = {
    "full": dict(vocab=32000, hidden=2048, layers=24, heads=8, head_dim=256, inter=5632, conv=4, eps=1e-6),
    "small": dict(vocab=4096, hidden=512, layers=2, heads=2, head_dim=256, inter=1536, conv=4, eps=1e-6),
}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--dims", choices=sorted(DIMS), default="small")
    ap.add_argument("--steps", type=int, default=12)
    ap.add_argument("--greedy", type=int, default=6)
    ap.add_argument("--out", required=True)
    ap.add_argument("--failure", action="store_true", help="also run the failure-path check")
    args = ap.parse_args()
    dims = DIMS[args.dims]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    L = gdn.lib()
    gdn.check(L.gdn_b200_set_device(local), "gdn_b200_set_device")
    hdr = gdn.make_header(vocab=dims["vocab"], hidden=dims["hidden"], layers=dims["layers"], heads=dims["heads"],
                          head_dim=dims["head_dim"], inter=dims["inter"], conv=dims["conv"], eps=dims["eps"])
    model = gdn.Model(header=hdr, seed=20261202)
    rng = np.random.default_rng(5)
    rs = gdn.RunState(model)
    rec0 = (rng.standard_normal(rs.rec_floats) * 0.05).astype(np.float32)
    conv0 = (rng.standard_normal(rs.conv_floats) * 0.5).astype(np.float32)
    teacher = rng.integers(0, dims["vocab"], size=args.steps).astype(np.int32)

    def run(state, together):
        state.load_state(rec0, conv0)
        if together:
            dist.barrier()  # every rank's state is in place before any rank steps
        out, ms = state.decode(teacher)
        logits, _ = state.outputs()
        greedy, _ = state.decode([int(out[-1])] * args.greedy, greedy=True)
        return out, ms, logits, greedy

    def refused(fn) -> bool:
        try:
            fn()
        except RuntimeError as e:
            return "tensor-parallel state" in str(e)
        return False

    tp.attach(rs)
    out, ms, logits, greedy = run(rs, True)
    # while attached, the state is this rank's part only: whole-state reads,
    # .gdnstate saves and prefill are refused
    guards = {"download_refused": refused(rs.read_state),
              "save_refused": refused(lambda: rs.save_state(os.devnull)),
              "prefill_refused": refused(lambda: rs.prefill([1, 2, 3]))}
    part = rs.read_state_part()
    parts = [None] * world if rank == 0 else None
    dist.gather_object(part, parts, dst=0)
    seen = [None] * world
    dist.all_gather_object(seen, (out.tolist(), greedy.tolist(), logits.tobytes()))
    rs.tp_detach()
    guards["single_gpu_decode_refused"] = refused(lambda: rs.step(int(teacher[0])))
    dist.barrier()
    res = {}
    if rank == 0:
        ref = gdn.RunState(model)
        r_out, r_ms, r_logits, r_greedy = run(ref, False)
        r_rec, r_conv = ref.read_state()
        m_rec, m_conv = tp.merge_state(parts, dims)
        res = {
            "world": world, "grid": part[2], "dims": args.dims,
            "tokens_equal": bool(np.array_equal(out, r_out)),
            "greedy_equal": bool(np.array_equal(greedy, r_greedy)),
            "logits_bitwise_equal": bool(np.array_equal(logits.view(np.uint32), r_logits.view(np.uint32))),
            "ranks_agree": all(s[0] == seen[0][0] and s[1] == seen[0][1] and s[2] == seen[0][2] for s in seen),
            "rec_bitwise_equal": bool(np.array_equal(m_rec.view(np.uint32), r_rec.view(np.uint32))),
            "conv_bitwise_equal": bool(np.array_equal(m_conv.view(np.uint32), r_conv.view(np.uint32))),
            "tp_ms_per_token": ms / args.steps, "one_gpu_ms_per_token": r_ms / args.steps,
            "tokens": out.tolist(), "greedy": greedy.tolist(),
        }
        ref.free()
    # every rank's guards, gathered on rank 0
    all_guards = [None] * world if rank == 0 else None
    dist.gather_object(guards, all_guards, dst=0)
    if rank == 0:
        res["guards"] = all_guards
    if args.failure:
        # failure path: rank 1 sits out one step between steps (no kernel of
        # its own in flight); rank 0's bounded exchange waits run out and its
        # step returns -1. Then every rank attaches again, reloads the state
        # and the decode equals the single-GPU decode bit for bit.
        tp.attach(rs)
        rs.load_state(rec0, conv0)
        dist.barrier()
        err = ""
        if rank == 0:
            try:
                rs.step(int(teacher[0]))
            except RuntimeError as e:
                err = str(e)
        dist.barrier()  # rank 0's failed step has ended before anyone re-attaches
        tp.attach(rs)
        out2, _, logits2, greedy2 = run(rs, True)
        if rank == 0:
            res["failure"] = {
                "step_error": err,
                "timed_out": "exchange wait timeout" in err,
                "tokens_equal_after_reattach": bool(np.array_equal(out2, out)),
                "logits_bitwise_equal_after_reattach": bool(np.array_equal(logits2.view(np.uint32),
                                                                           logits.view(np.uint32))),
                "greedy_equal_after_reattach": bool(np.array_equal(greedy2, greedy)),
            }
        rs.tp_detach()
        dist.barrier()
    if rank == 0:
        with open(args.out, "w") as f:
            json.dump(res, f)
    dist.barrier()
    rs.free()
    model.free()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
