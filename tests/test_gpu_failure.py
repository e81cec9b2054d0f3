"""The decode kernel's failure path, exercised without faulting the GPU: a
test hook (gdn_b200_test_drop_outputs) makes one CTA leave out its outputs
of one phase, the CTAs waiting for them give up after their bounded wait,
every CTA stops, and the step returns -1 carrying the kernel's report. The
run state stays usable: with the hook off and the recurrent state reloaded,
the next steps match an untouched run state bit for bit."""
import ctypes

import numpy as np
import pytest

import gateddeltanet_b200 as gdn
import oracle_lib as ol

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    from gateddeltanet_b200 import build
    build.build()
    L = gdn.lib()
    assert L.gdn_b200_set_device(0) == 0, gdn.last_error()
    d = ol.SMALL_DIMS
    m = gdn.Model(header=gdn.make_header(vocab=d["vocab"], hidden=d["hidden"], layers=d["layers"], heads=d["heads"],
                                         head_dim=d["head_dim"], inter=d["inter"], conv=d["conv"], eps=d["eps"]),
                  seed=99)
    yield m
    m.free()


def test_dropped_outputs_time_out_and_recover(model):
    L = gdn.lib()
    toks = [5, 17, 300, 4000, 9, 1234]
    good, bad = gdn.RunState(model), gdn.RunState(model)
    try:
        ref_picks, _ = good.decode(toks)
        ref_rec, ref_conv = good.read_state()
        # layer 1, phase A (QKVGAB): CTA 0's rows never arrive
        assert L.gdn_b200_test_drop_outputs(ctypes.byref(bad.s), 0, 5) == 0
        with pytest.raises(RuntimeError, match="exchange wait timeout"):
            bad.step(toks[0])
        # off again; a phase that is not a GEMV phase is rejected
        assert L.gdn_b200_test_drop_outputs(ctypes.byref(bad.s), 0, 6) != 0
        assert L.gdn_b200_test_drop_outputs(ctypes.byref(bad.s), -1, -1) == 0
        rec, conv = bad.read_state()
        bad.load_state(np.zeros_like(rec), np.zeros_like(conv))
        picks, _ = bad.decode(toks)
        np.testing.assert_array_equal(picks, ref_picks)
        rec, conv = bad.read_state()
        np.testing.assert_array_equal(rec.view(np.uint32), ref_rec.view(np.uint32))
        np.testing.assert_array_equal(conv.view(np.uint32), ref_conv.view(np.uint32))
    finally:
        good.free()
        bad.free()


def test_exchange_tags_wrap_and_refills_restart_them(model):
    """16-bit exchange tags (BF16-boundary contracts): a launch whose tags run
    past 0xffff after earlier launches wrote every word decodes exactly; after
    a refill of the exchange buffers with 0xff (tp_detach, or a change of the
    boundary contract) the next launch starts from tag 0, never from a range
    that holds 0xffff -- the tag an unwritten word carries."""
    L = gdn.lib()
    toks = [5, 17, 300, 4000, 9, 1234, 77, 3]
    stride = 5 * ol.SMALL_DIMS["layers"] + 1
    near = 0x10000 - stride // 2  # the launch's tags straddle 0xffff
    ref, a, b, c = (gdn.RunState(model) for _ in range(4))
    try:
        ref_picks, _ = ref.decode(toks)
        ref_lg, _ = ref.outputs()
        ref_rec, ref_conv = ref.read_state()
        # a: words already written by two launches, then tags through 0xffff
        a.decode(toks[:2])
        assert L.gdn_b200_test_set_epoch(ctypes.byref(a.s), near) == 0
        pa, _ = a.decode(toks[2:])
        # b: the epoch near the wrap, then a refill (detach): it restarts at 0
        assert L.gdn_b200_test_set_epoch(ctypes.byref(b.s), near) == 0
        b.tp_detach()
        pb, _ = b.decode(toks)
        # c: the same through a change of contract and back
        assert L.gdn_b200_test_set_epoch(ctypes.byref(c.s), near) == 0
        c.set_numerics(*gdn.RunState.FP32)
        c.set_numerics(*gdn.RunState.CIMPL)
        pc, _ = c.decode(toks)
        for name, rs, picks in (("wrap", a, np.concatenate([ref_picks[:2], pa])), ("detach", b, pb),
                                ("numerics", c, pc)):
            np.testing.assert_array_equal(picks, ref_picks, err_msg=name)
            lg, _ = rs.outputs()
            np.testing.assert_array_equal(lg.view(np.uint32), ref_lg.view(np.uint32), err_msg=name)
            rec, conv = rs.read_state()
            np.testing.assert_array_equal(rec.view(np.uint32), ref_rec.view(np.uint32), err_msg=name)
            np.testing.assert_array_equal(conv.view(np.uint32), ref_conv.view(np.uint32), err_msg=name)
    finally:
        for rs in (ref, a, b, c):
            rs.free()
