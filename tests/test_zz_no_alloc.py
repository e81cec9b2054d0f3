"""gdn_b200_decode_tokens_noalloc (include/gdn_b200.h) against
gdn_b200_decode_tokens: two run states of one model decode the same two
calls in a row (a teacher-forced call, then a greedy one), one through each
entry point; every step's argmax, the token line and the recurrent state and
conv tails must agree bit for bit after each call. Also: a call longer than
the 4096-token scratch is rejected with an error naming the limit, and a
call on a fresh run state, longer than any call before it, leaves the
device's free memory unchanged (the property the entry point exists for).
The file is named so that it is collected last."""
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
                  seed=4242)
    yield m
    m.free()


def test_noalloc_matches_decode_tokens(model):
    rng = np.random.default_rng(5)
    first = rng.integers(0, model.m.config.vocab_size, size=37).tolist()
    second = rng.integers(0, model.m.config.vocab_size, size=23).tolist()
    a, b = gdn.RunState(model), gdn.RunState(model)
    try:
        for tokens, greedy in ((first, False), (second, True)):
            pa, _ = a.decode(tokens, greedy=greedy)
            pb, _ = b.decode_noalloc(tokens, greedy=greedy)
            np.testing.assert_array_equal(pa, pb)
            assert a.workspace(gdn.GDN_WS_OFF_X_NORM, 1)[0] == b.workspace(gdn.GDN_WS_OFF_X_NORM, 1)[0]
            ra, ca = a.read_state()
            rb, cb = b.read_state()
            np.testing.assert_array_equal(ra.view(np.uint32), rb.view(np.uint32))
            np.testing.assert_array_equal(ca.view(np.uint32), cb.view(np.uint32))
    finally:
        a.free()
        b.free()


def test_noalloc_rejects_oversized_call(model):
    s = gdn.RunState(model)
    try:
        with pytest.raises(RuntimeError, match="at most 4096 tokens"):
            s.decode_noalloc([1] * 4097)
    finally:
        s.free()


def test_noalloc_allocates_nothing(model):
    import ctypes
    free_b, total_b = ctypes.c_size_t(0), ctypes.c_size_t(0)
    cudart = None
    for name in ("libcudart.so.12", "libcudart.so"):
        try:
            cudart = ctypes.CDLL(name)
            break
        except OSError:
            continue
    if cudart is None:
        import torch
        mem_get_info = lambda: torch.cuda.mem_get_info(0)[0]  # noqa: E731
    else:
        def mem_get_info():
            assert cudart.cudaMemGetInfo(ctypes.byref(free_b), ctypes.byref(total_b)) == 0
            return free_b.value
    warm = gdn.RunState(model)
    s = gdn.RunState(model)
    try:
        warm.decode_noalloc([1, 2, 3])  # the scratch's address is looked up once per device
        before = mem_get_info()
        s.decode_noalloc(list(range(100, 100 + 1500)))
        after = mem_get_info()
        assert after == before, f"free device memory changed by {before - after} bytes"
    finally:
        warm.free()
        s.free()
