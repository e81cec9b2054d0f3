"""Tensor-parallel decode on two GPUs: the step is the
single-GPU step with its row and column partitions spread over both GPUs'
CTAs and every output stored into both GPUs' exchange regions over NVLink, so
tokens, logits and the (merged) recurrent state must equal a single-GPU run
bit for bit. Runs tests/tp_rank.py as two processes under
torch.distributed.run; skipped with fewer than two GPUs."""
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
@pytest.mark.parametrize("dims,steps", [("small", 12), ("full", 6)])
def test_two_gpu_decode_is_the_one_gpu_decode(tmp_path, dims, steps):
    from gateddeltanet_b200 import build
    build.build()
    out = str(tmp_path / "tp.json")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "60", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(REPO, "tests", "tp_rank.py"), "--dims", dims, "--steps", str(steps), "--out", out]
    run = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=720)
    assert run.returncode == 0, run.stdout[-2000:] + run.stderr[-4000:]
    res = json.loads(open(out).read())
    assert res["world"] == 2
    for key in ("tokens_equal", "greedy_equal", "logits_bitwise_equal", "ranks_agree", "rec_bitwise_equal",
                "conv_bitwise_equal"):
        assert res[key], (key, res)
