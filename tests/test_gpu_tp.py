"""Tensor-parallel decode on two GPUs: the step is the
single-GPU step with its row and column partitions spread over both GPUs'
CTAs and every output stored into both GPUs' exchange regions over NVLink, so
tokens, logits and the (merged) recurrent state must equal a single-GPU run
bit for bit. The library refuses whole-state reads, saves, prefill and
single-GPU decode of a rank's partial state; a rank that sits out a step
makes the other's step fail on its bounded waits, and attaching again
recovers. Runs tests/tp_rank.py as two processes under torch.distributed.run;
skipped with fewer than two GPUs."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="tensor-parallel decode needs two GPUs")
@pytest.mark.parametrize("dims,steps,failure", [("small", 12, True), ("full", 6, False)])
def test_two_gpu_decode_is_the_one_gpu_decode(tmp_path, dims, steps, failure):
    from gateddeltanet_b200 import build
    build.build()
    out = str(tmp_path / "tp.json")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "60", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(REPO, "tests", "tp_rank.py"), "--dims", dims, "--steps", str(steps), "--out", out] + (["--failure"] if failure else [])
    run = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=720)
    assert run.returncode == 0, run.stdout[-2000:] + run.stderr[-4000:]
    res = json.loads(open(out).read())
    assert res["world"] == 2
    for key in ("tokens_equal", "greedy_equal", "logits_bitwise_equal", "ranks_agree", "rec_bitwise_equal",
                "conv_bitwise_equal"):
        assert res[key], (key, res)
    # each rank's partial state is refused where a whole state is needed
    for g in res["guards"]:
        assert all(g.values()), g
    if failure:
        # a rank that sits out a step: the other's bounded waits run out and
        # its step fails; attaching again recovers the bit-exact decode
        f = res["failure"]
        assert f["timed_out"], f
        assert f["tokens_equal_after_reattach"] and f["logits_bitwise_equal_after_reattach"], f
        assert f["greedy_equal_after_reattach"], f
