"""The CPU oracle (oracle/gdn_oracle.c) against golden vectors produced by the
reference itself (tests/golden/reference_goldens.json, written by
tests/golden/make_golden.py from the reference's c_impl compiled natively).

Pins, bit for bit:
  * BF16 RNE (c_impl/gdn_model.cpp:314-325) over 65536 spread bit patterns
    and every high half with the five interesting low halves;
  * the native BF16 product (c_impl/gdn_model.cpp:392-466) of every BF16
    weight with 32 edge-case activations (zeros, subnormals, the flush
    boundary, Inf, NaN, ...);
  * full GDN-1.3B decode (seeded weights, zero and seeded states) in the
    reference contract: tokens, argmax, FP32 logits, hidden vector, recurrent
    state and conv tails.
CPU only; the decode cases take about a minute on 8 cores.
"""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np
import pytest

import oracle_lib

GOLD = json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                                   "reference_goldens.json")))

# The 32 activations of the reference product grid (oracle/ref_driver.cpp).
GRID_ACTIVATIONS = [
    0x0000, 0x8000, 0x0001, 0x807F, 0x0080, 0x8080, 0x3F80, 0xBF80, 0x7F80, 0xFF80, 0x7FC0,
    0x7F81, 0x7F7F, 0xFF7F, 0x3F81, 0x4000, 0x00FF, 0x3E4C, 0xC2F7, 0x1F00, 0x2000, 0x2080,
    0x5F00, 0x6000, 0x0100, 0x3C00, 0x3B80, 0x1C3F, 0x23A1, 0x9E77, 0x4B19, 0xD0E3]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def lib():
    return oracle_lib.load()


def rne_inputs() -> np.ndarray:
    a = (np.arange(65536, dtype=np.uint64) * 65521) & 0xFFFFFFFF
    lows = np.array([0x0000, 0x7FFF, 0x8000, 0x8001, 0xFFFF], dtype=np.uint64)
    b = ((np.arange(65536, dtype=np.uint64)[:, None] << 16) | lows[None, :]).reshape(-1)
    return np.concatenate([a, b]).astype(np.uint32)


def test_bf16_rne_matches_reference(lib):
    x = rne_inputs()
    out = np.empty(len(x), dtype=np.uint16)
    lib.gdn_oracle_bf16_rne_batch(x.ctypes.data_as(oracle_lib.ctypes.c_void_p), len(x),
                                  out.ctypes.data_as(oracle_lib.ctypes.c_void_p))
    g = GOLD["primitives"]
    idx = np.array(g["rne_sample"]["index"])
    np.testing.assert_array_equal(out[idx], np.array(g["rne_sample"]["bits"], dtype=np.uint16))
    assert sha(out[:65536]) == g["rne_set_a_sha256"]
    assert sha(out[65536:]) == g["rne_set_b_sha256"]


def test_native_product_matches_reference(lib):
    w = np.arange(65536, dtype=np.uint16)
    a = np.array(GRID_ACTIVATIONS, dtype=np.uint16)
    out = np.empty(len(w) * len(a), dtype=np.uint32)
    lib.gdn_oracle_native_product_grid(w.ctypes.data_as(oracle_lib.ctypes.c_void_p), len(w),
                                       a.ctypes.data_as(oracle_lib.ctypes.c_void_p), len(a),
                                       out.ctypes.data_as(oracle_lib.ctypes.c_void_p))
    g = GOLD["primitives"]
    idx = np.array(g["product_sample"]["index"])
    np.testing.assert_array_equal(out[idx], np.array(g["product_sample"]["bits"], dtype=np.uint32))
    assert sha(out) == g["product_grid_sha256"]


@pytest.fixture(scope="module")
def full_oracle():
    return oracle_lib.Oracle(oracle_lib.FULL_DIMS, seed=GOLD["decode"][0]["seed"])


@pytest.mark.parametrize("case", GOLD["decode"], ids=[c["name"] for c in GOLD["decode"]])
def test_decode_matches_reference(full_oracle, case):
    o = full_oracle
    assert case["seed"] == GOLD["decode"][0]["seed"]
    o.reset_state(case["state_seed"])
    for i, ref in enumerate(case["steps_out"]):
        tok = o.token(case["stream_seed"], case["stream"], i)
        assert tok == ref["token"]
        out = o.step(tok, oracle_lib.REFERENCE_MODE)
        assert out.argmax == ref["argmax"], f"step {i}"
        assert sha(out.logits) == ref["logits_sha256"], f"step {i} logits"
        assert sha(out.hidden) == ref["hidden_sha256"], f"step {i} hidden"
        top = np.argsort(-out.logits, kind="stable")[:5]
        assert top.tolist() == ref["top5_index"]
    assert sha(o.rec) == case["rec_sha256"]
    assert sha(o.conv) == case["conv_sha256"]


def test_config0_trajectory_starts_as_the_zero_state_goldens():
    """The 256-step config[0] digests (tests/golden/reference_config0_256.json,
    checked against the GPU in tests/test_gpu_config0.py) come from the same
    reference build, seed and token stream as the zero-state trajectory here:
    their first steps must agree digest for digest, and the stream's tokens are
    the seeded stream's."""
    c0 = json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_config0_256.json")))
    zero = next(c for c in GOLD["decode"] if c["name"] == "zero_state")
    assert (c0["seed"], c0["stream_seed"], c0["stream"], c0["state_seed"]) == \
        (zero["seed"], zero["stream_seed"], zero["stream"], zero["state_seed"])
    assert c0["steps"] == len(c0["steps_out"]) == 256
    for i, ref in enumerate(zero["steps_out"]):
        got = c0["steps_out"][i]
        for key in ("token", "argmax", "logits_sha256", "hidden_sha256", "top5_index"):
            assert got[key] == ref[key], (i, key)
    from gateddeltanet_b200.workload import token_stream
    assert [s["token"] for s in c0["steps_out"]] == token_stream(c0["stream"], 256, 32000, seed=c0["stream_seed"])
