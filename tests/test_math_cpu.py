"""Host check of the decode kernel's scalar math (gateddeltanet_b200/csrc/
gdn_math.h) against the host libm the reference is built with: exp by the
table-driven method and the branch-free sigmoid must agree with glibc expf
and the reference's sigmoid (c_impl/gdn_model.cpp:1307-1316) on all but a
tiny fraction of inputs, and never by more than one ulp. The GPU side of
the same functions is pinned by the bit-exact engine-vs-oracle parity
tests."""
from __future__ import annotations

import json
import os
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def math_check(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("math") / "math_check")
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off",
                    "-I", os.path.join(REPO, "gateddeltanet_b200", "csrc"),
                    os.path.join(REPO, "tests", "native", "math_check.cpp"), "-o", exe], check=True)
    return exe


def test_exp_and_sigmoid_track_libm(math_check):
    out = subprocess.run([math_check, "61"], check=True, capture_output=True, text=True).stdout
    r = json.loads(out)
    assert r["n"] > 30_000_000
    assert r["exp_far"] == 0                      # never more than one ulp from glibc expf
    assert r["exp_mismatch"] / r["n"] < 3e-4      # measured 1.6e-4
    assert r["sigmoid_mismatch"] / r["n"] < 2e-4  # measured 8.5e-5
