"""GPU prefill (gdn_b200_prefill) against token-by-token decoding in the CPU
oracle's FP32 control (tests/oracle_lib.py), through the C ABI.

Prefill runs the prompt's projections as tensor-core GEMMs over the tokens and
the recurrence in token order, in FP32; the gates are the north star's FP32
rows: recurrent state and conv tails rel-L2 <= 1e-3 (state) after the prompt,
and logits rel-L2 <= 1e-4 for the FP32-control decode steps that follow.
"""
import numpy as np
import pytest

import gateddeltanet_b200 as gdn
import oracle_lib as ol
import parity

pytestmark = pytest.mark.gpu

SEED = 20261201
STREAM_SEED = 555


def header_for(dims):
    return gdn.make_header(vocab=dims["vocab"], hidden=dims["hidden"], layers=dims["layers"], heads=dims["heads"],
                           head_dim=dims["head_dim"], inter=dims["inter"], conv=dims["conv"], eps=dims["eps"])


@pytest.fixture(scope="module")
def lib():
    from gateddeltanet_b200 import build
    build.build()
    L = gdn.lib()
    assert L.gdn_b200_set_device(0) == 0, gdn.last_error()
    return L


@pytest.fixture(scope="module")
def small(lib):
    return gdn.Model(header=header_for(ol.SMALL_DIMS), seed=SEED), ol.Oracle(ol.SMALL_DIMS, seed=SEED)


def check_prefill(model, oracle, n, state_seed=0, follow=3, stream=0):
    oracle.reset_state(state_seed)
    rs = gdn.RunState(model)
    rs.set_numerics(False, False, False)  # FP32 control for the decode steps that follow
    if state_seed:
        rs.load_state(oracle.rec, oracle.conv)
    toks = [oracle.token(STREAM_SEED, stream, i) for i in range(n + follow)]
    ms = rs.prefill(toks[:n])
    for t in toks[:n]:
        oracle.step(t, ol.FP32_CONTROL)
    rec, conv = rs.read_state()
    e_rec = parity.rel_l2(rec, oracle.rec)
    e_conv = parity.rel_l2(conv, oracle.conv)
    assert e_rec <= parity.STATE, e_rec
    assert e_conv <= parity.STATE, e_conv
    worst = 0.0
    for t in toks[n:]:
        rs.step(t)
        logits, _ = rs.outputs()
        ref = oracle.step(t, ol.FP32_CONTROL)
        e = parity.rel_l2(logits, ref.logits)
        worst = max(worst, e)
        assert e <= parity.LOGITS_FP32, e
    rs.free()
    return e_rec, e_conv, worst, ms


@pytest.mark.parametrize("n", [1, 2, 5, 37, 500])
def test_prefill_small_from_zero(small, n):
    model, oracle = small
    e_rec, e_conv, worst, ms = check_prefill(model, oracle, n)
    print(f"prefill {n} tokens: state {e_rec:.2e}, tails {e_conv:.2e}, next logits {worst:.2e}, {ms:.2f} ms")


def test_prefill_small_from_seeded_state(small):
    model, oracle = small
    check_prefill(model, oracle, 53, state_seed=7, stream=1)


def test_prefill_rejects_bad_token(small):
    model, _ = small
    rs = gdn.RunState(model)
    with pytest.raises(RuntimeError):
        rs.prefill([1, 2, model.config.vocab_size])
    assert rs.prefill([]) == 0.0
    rs.free()


def test_prefill_full_model(lib):
    model = gdn.Model(header=header_for(ol.FULL_DIMS), seed=SEED)
    oracle = ol.Oracle(ol.FULL_DIMS, seed=SEED)
    e_rec, e_conv, worst, ms = check_prefill(model, oracle, 24, follow=2)
    print(f"GDN-1.3B prefill 24 tokens: state {e_rec:.2e}, tails {e_conv:.2e}, next logits {worst:.2e}, {ms:.2f} ms")
