"""Parity of the B200 engine (libgdn_b200.so, through its C ABI) with the CPU
oracle (oracle/gdn_oracle.c, itself pinned bit-exact to the reference's
c_impl/gdn_model.cpp decode by tests/test_oracle_golden.py).

Contracts compared (see tests/oracle_lib.py):
  c_impl (default) the reference's own arithmetic (BF16-rounded products, BF16
                   state, BF16 boundaries) vs oracle REFERENCE_MODE: logits,
                   final hidden vector, recurrent state and conv tails equal
                   bit for bit (the fast packed-BF16 product and the exact
                   emulation both)
  engine           exact BF16 products, FP32 state, BF16 boundaries vs oracle
                   ENGINE_MODE: bit for bit
  FP32 control     FP32 boundaries vs oracle FP32_CONTROL: logits rel-L2 <=
                   1e-4, state <= 1e-4
The gates of tests/parity.py (logits rel-L2 1e-2, state 1e-3, argmax wherever
the oracle's top-2 margin exceeds 4x the logit error) are asserted as well.
"""
import numpy as np
import pytest

import gateddeltanet_b200 as gdn
import oracle_lib as ol
import parity

pytestmark = pytest.mark.gpu

SEED = 20261201
STREAM_SEED = 77


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
    model = gdn.Model(header=header_for(ol.SMALL_DIMS), seed=SEED)
    oracle = ol.Oracle(ol.SMALL_DIMS, seed=SEED)
    np.testing.assert_array_equal(
        np.ctypeslib.as_array(model.m.weight_data, shape=(oracle.blob.size,)).view(np.uint32),
        oracle.blob.view(np.uint32))
    return model, oracle


@pytest.fixture(scope="module")
def full(lib):
    model = gdn.Model(header=header_for(ol.FULL_DIMS), seed=SEED)
    oracle = ol.Oracle(ol.FULL_DIMS, seed=SEED)
    return model, oracle


ENGINE = (True, False, False)      # exact products, FP32 state (gdn_b200_set_numerics)
CIMPL = (True, True, True)         # the c_impl's own arithmetic (the default)
FP32 = (False, False, False)       # FP32 control


def run_parity(model, oracle, steps, mode, numerics, state_seed, tol_logits, tol_state, use_loop=False,
               bitexact=False, exact_products=False):
    oracle.reset_state(state_seed)
    rs = gdn.RunState(model)
    rs.set_numerics(*numerics)
    if exact_products:
        rs.force_exact_products(True)
    if state_seed:
        rs.load_state(oracle.rec, oracle.conv)
    tokens = [oracle.token(STREAM_SEED, 0, i) for i in range(steps)]
    worst = 0.0
    for i, tok in enumerate(tokens):
        if use_loop:
            picks, _ = rs.decode([tok])
            pick = int(picks[0])
        else:
            pick = rs.step(tok)
        logits, hidden = rs.outputs()
        ref = oracle.step(tok, mode)
        err = parity.rel_l2(logits, ref.logits)
        worst = max(worst, err)
        assert err <= tol_logits, f"step {i}: logits rel-L2 {err:.3e} > {tol_logits}"
        if bitexact:
            np.testing.assert_array_equal(logits.view(np.uint32), ref.logits.view(np.uint32), err_msg=f"step {i} logits")
            np.testing.assert_array_equal(hidden.view(np.uint32), ref.hidden.view(np.uint32), err_msg=f"step {i} hidden")
            assert pick == ref.argmax
        assert pick == parity.argmax_first(logits), "kernel argmax != argmax of its own logits"
        assert parity.argmax_agrees(logits, ref.logits, pick), f"step {i}: argmax {pick} vs oracle {ref.argmax}"
    rec, conv = rs.read_state()
    s_err = parity.rel_l2(rec, oracle.rec)
    c_err = parity.rel_l2(conv, oracle.conv)
    assert s_err <= tol_state, f"recurrent state rel-L2 {s_err:.3e} > {tol_state}"
    assert c_err <= tol_logits, f"conv tails rel-L2 {c_err:.3e}"
    if bitexact:
        np.testing.assert_array_equal(rec.view(np.uint32), oracle.rec.view(np.uint32))
        np.testing.assert_array_equal(conv.view(np.uint32), oracle.conv.view(np.uint32))
    rs.free()
    return worst, s_err


@pytest.mark.parametrize("state_seed", [0, 7])
def test_small_engine_mode(small, state_seed):
    model, oracle = small
    run_parity(model, oracle, 8, ol.ENGINE_MODE, ENGINE, state_seed, parity.LOGITS_BF16, parity.STATE, bitexact=True)


@pytest.mark.parametrize("state_seed", [0, 7])
def test_small_fp32_control(small, state_seed):
    model, oracle = small
    run_parity(model, oracle, 6, ol.FP32_CONTROL, FP32, state_seed, parity.LOGITS_FP32, parity.LOGITS_FP32)


@pytest.mark.parametrize("state_seed", [0, 7])
def test_small_reference_mode(small, state_seed):
    model, oracle = small
    run_parity(model, oracle, 8, ol.REFERENCE_MODE, CIMPL, state_seed, parity.LOGITS_BF16, parity.STATE, bitexact=True)


def test_small_reference_mode_exact_products(small):
    """The exact emulation of the reference's BF16 product (special values,
    DAZ, FTZ), which phases use when an input could produce a product below
    the normal range, gives the same bits as the packed BF16 multiply."""
    model, oracle = small
    run_parity(model, oracle, 4, ol.REFERENCE_MODE, CIMPL, 7, parity.LOGITS_BF16, parity.STATE, bitexact=True,
               exact_products=True)


def test_default_is_reference_contract(small):
    """A run state decodes in the reference's own arithmetic unless told
    otherwise (gdn_decode_step_host as a drop-in returns the reference's
    results)."""
    model, oracle = small
    oracle.reset_state(0)
    rs = gdn.RunState(model)
    tok = oracle.token(STREAM_SEED, 4, 0)
    pick = rs.step(tok)
    logits, _ = rs.outputs()
    ref = oracle.step(tok, ol.REFERENCE_MODE)
    np.testing.assert_array_equal(logits.view(np.uint32), ref.logits.view(np.uint32))
    assert pick == ref.argmax
    with pytest.raises(RuntimeError, match="not a contract"):
        rs.set_numerics(True, True, False)
    rs.free()


def test_small_device_loop_matches_host_steps(small):
    """gdn_b200_decode_tokens (device-resident loop) and gdn_decode_step_host
    compute bit-identical logits and state; the kernel is deterministic."""
    model, oracle = small
    tokens = [oracle.token(STREAM_SEED, 1, i) for i in range(5)]
    a = gdn.RunState(model)
    b = gdn.RunState(model)
    picks_a = [a.step(t) for t in tokens]
    la, _ = a.outputs()
    picks_b, ms = b.decode(tokens)
    lb, _ = b.outputs()
    assert list(picks_b) == picks_a
    np.testing.assert_array_equal(la.view(np.uint32), lb.view(np.uint32))
    ra, ca = a.read_state()
    rb, cb = b.read_state()
    np.testing.assert_array_equal(ra.view(np.uint32), rb.view(np.uint32))
    np.testing.assert_array_equal(ca.view(np.uint32), cb.view(np.uint32))
    assert ms > 0.0


def test_small_greedy_loop(small):
    """Device greedy loop == host-driven greedy loop (c_impl/gdn_eval.cpp:336-440)."""
    model, oracle = small
    a = gdn.RunState(model)
    seed_tok = oracle.token(STREAM_SEED, 2, 0)
    traj = [seed_tok]
    for _ in range(6):
        traj.append(a.step(traj[-1]))
    b = gdn.RunState(model)
    picks, _ = b.decode([seed_tok] + [0] * 5, greedy=True)
    assert list(picks) == traj[1:]


def test_debug_buffers_and_token_line(small, lib):
    model, oracle = small
    c = model.config
    hid = np.zeros(c.hidden_size, dtype=np.float32)
    log = np.zeros(c.vocab_size, dtype=np.float32)
    fp = gdn._FP
    lib.gdn_set_native_debug_buffers(hid.ctypes.data_as(fp), log.ctypes.data_as(fp))
    try:
        rs = gdn.RunState(model)
        pick = rs.step(oracle.token(STREAM_SEED, 3, 0))
    finally:
        lib.gdn_set_native_debug_buffers(None, None)
    logits, hidden = rs.outputs()
    np.testing.assert_array_equal(log, logits)
    np.testing.assert_array_equal(hid, hidden)
    line = rs.workspace(gdn.GDN_WS_OFF_X_NORM, 16)
    assert line[0] == float(pick) and not line[1:].any()
    # gdn_compute_logits (independent scalar LM head with BF16 product rounding)
    scalar = model.compute_logits(hidden)
    assert parity.rel_l2(scalar, logits) < 1e-2


def test_out_of_range_token_rejected(small):
    model, _ = small
    rs = gdn.RunState(model)
    with pytest.raises(RuntimeError, match="out of range"):
        rs.step(model.config.vocab_size)
    with pytest.raises(RuntimeError, match="out of range"):
        rs.step(-1)
    with pytest.raises(RuntimeError, match="out of range"):
        rs.decode([0, model.config.vocab_size])
    rs.step(0)  # stream still usable


def test_state_roundtrip_and_gdnstate_file(small, tmp_path):
    model, oracle = small
    oracle.reset_state(11)
    rs = gdn.RunState(model)
    rs.load_state(oracle.rec, oracle.conv)
    rec, conv = rs.read_state()
    np.testing.assert_array_equal(rec, oracle.rec)
    np.testing.assert_array_equal(conv, oracle.conv)
    rs.step(5)
    path = str(tmp_path / "s.gdnstate")
    assert model.lib.gdn_b200_state_save_file(rs.s, path.encode(), 123) == 0
    rs2 = gdn.RunState(model)
    seed = gdn.ctypes.c_int32(0)
    assert model.lib.gdn_b200_state_load_file(rs2.s, path.encode(), gdn.ctypes.byref(seed)) == 0
    assert seed.value == 123
    r1, c1 = rs.read_state()
    r2, c2 = rs2.read_state()
    np.testing.assert_array_equal(r1, r2)
    np.testing.assert_array_equal(c1, c2)
    # truncated / trailing files are rejected (c_impl/host.cpp:675-735)
    data = open(path, "rb").read()
    open(path, "wb").write(data[:-4])
    assert model.lib.gdn_b200_state_load_file(rs2.s, path.encode(), None) != 0
    open(path, "wb").write(data + b"\0")
    assert model.lib.gdn_b200_state_load_file(rs2.s, path.encode(), None) != 0


def test_full_engine_and_reference_modes(full):
    """GDN-1.3B shape: 3 teacher-forced steps from a
    seeded state in the engine contract, then in the reference's own
    arithmetic (BF16 products, BF16 state), both bit for bit."""
    model, oracle = full
    run_parity(model, oracle, 3, ol.ENGINE_MODE, ENGINE, 7, parity.LOGITS_BF16, parity.STATE, bitexact=True)
    run_parity(model, oracle, 3, ol.REFERENCE_MODE, CIMPL, 7, parity.LOGITS_BF16, parity.STATE, use_loop=True,
               bitexact=True)


def test_full_fp32_control(full):
    model, oracle = full
    run_parity(model, oracle, 2, ol.FP32_CONTROL, FP32, 0, parity.LOGITS_FP32, parity.LOGITS_FP32)
