"""Teacher-forced scoring (gdn_b200_score_window) against the CPU oracle, through
the C ABI: the reference's score_window_hw (c_impl/host.cpp:1954-1994) restated
over the oracle's logits in float64. The scoring itself adds nothing (a window
equals the same sums over the step logits read back from the host); the
engine's logits match the oracle's bit for bit on most trajectories, and where a
1-ulp exp difference flips a BF16 rounding they stay within the north star's
1e-2 logits gate, so a window agrees within 1e-3 relative. With the FP32
prefill the FP32 control is the comparison.
"""
import numpy as np
import pytest

import gateddeltanet_b200 as gdn
import oracle_lib as ol

pytestmark = pytest.mark.gpu

SEED = 20261201
STREAM_SEED = 808


def header_for(dims):
    return gdn.make_header(vocab=dims["vocab"], hidden=dims["hidden"], layers=dims["layers"], heads=dims["heads"],
                           head_dim=dims["head_dim"], inter=dims["inter"], conv=dims["conv"], eps=dims["eps"])


@pytest.fixture(scope="module")
def small():
    from gateddeltanet_b200 import build
    build.build()
    assert gdn.lib().gdn_b200_set_device(0) == 0, gdn.last_error()
    return gdn.Model(header=header_for(ol.SMALL_DIMS), seed=SEED), ol.Oracle(ol.SMALL_DIMS, seed=SEED)


def oracle_window(oracle, ctx, cont, mode):
    """score_window_hw over the oracle's logits (float64 log-softmax, max-shifted)."""
    oracle.reset_state(0)
    toks = list(ctx) + list(cont)
    lp, n = 0.0, 0
    for i in range(len(toks) - 1):
        lg = oracle.step(toks[i], mode).logits.astype(np.float64)
        if i + 1 < len(ctx):
            continue
        m = lg.max()
        lp += (lg[toks[i + 1]] - m) - np.log(np.exp(lg - m).sum())
        n += 1
    return lp, n


@pytest.mark.parametrize("numerics,mode", [((True, False, False), ol.ENGINE_MODE),
                                           ((True, True, True), ol.REFERENCE_MODE)])
def test_score_window_matches_oracle(small, numerics, mode):
    model, oracle = small
    rs = gdn.RunState(model)
    rs.set_numerics(*numerics)
    for w, (lc, lk) in enumerate([(1, 1), (5, 7), (12, 3)]):
        toks = [oracle.token(STREAM_SEED, w, i) for i in range(lc + lk)]
        lp, n = rs.score_window(toks[:lc], toks[lc:])
        ref, rn = oracle_window(oracle, toks[:lc], toks[lc:], mode)
        assert n == rn == lk
        assert abs(lp - ref) <= 1e-3 * max(1.0, abs(ref)), (lp, ref)
    rs.free()


def test_score_window_with_prefill(small):
    model, oracle = small
    rs = gdn.RunState(model)
    rs.set_numerics(False, False, False)
    toks = [oracle.token(STREAM_SEED, 9, i) for i in range(40)]
    lp, n = rs.score_window(toks[:30], toks[30:], use_prefill=True)
    ref, rn = oracle_window(oracle, toks[:30], toks[30:], ol.FP32_CONTROL)
    assert n == rn == 10
    assert abs(lp - ref) <= 1e-4 * abs(ref), (lp, ref)
    rs.free()


def test_score_window_rejects_bad_windows(small):
    model, _ = small
    rs = gdn.RunState(model)
    with pytest.raises(RuntimeError):
        rs.score_window([1, 2], [])
    with pytest.raises(RuntimeError):
        rs.score_window([], [1])
    with pytest.raises(RuntimeError):
        rs.score_window([1], [model.config.vocab_size])
    rs.free()
