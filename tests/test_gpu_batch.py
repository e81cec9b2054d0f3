"""Multi-stream decode (gdn_b200_batch_*, BASELINE config[3]) against the CPU
oracle, through the C ABI.

The batch engine's projections run on the tensor cores (tcgen05, FP32
accumulation), so it follows the FP32-boundary contract: activations and
state FP32, BF16 weights, exact products, a different summation order than
the reference's bank chains. It is compared with the oracle's FP32_CONTROL
mode per stream: logits rel-L2 <= 1e-4, recurrent state rel-L2 <= 1e-3,
argmax identical wherever the oracle's top-2 margin exceeds 4x the logit
error (tests/parity.py). The tile GEMM alone is compared with a float64
product.
"""
import numpy as np
import pytest

import gateddeltanet_b200 as gdn
import oracle_lib as ol
import parity

pytestmark = pytest.mark.gpu

SEED = 20261201
STREAM_SEED = 4242


def bf16_exact(a: np.ndarray) -> np.ndarray:
    """Round float32 to BF16 (nearest even) and widen back."""
    b = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return b.astype(np.uint32).view(np.float32)


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


@pytest.mark.parametrize("m,k,n", [(128, 64, 16), (200, 128, 3), (8208, 2048, 16), (2048, 5632, 64),
                                   (1024, 512, 80), (4096, 2048, 1)])
def test_tile_gemm_matches_float64(lib, m, k, n):
    rng = np.random.default_rng(m * 131 + k * 7 + n)
    w = bf16_exact(rng.normal(0.0, 0.02, size=(m, k)).astype(np.float32))
    x = rng.normal(0.0, 1.0, size=(n, k)).astype(np.float32)
    y = gdn.tile_gemm(w, x)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    # FP32 accumulation of exact products: error well below 1e-5 of the row scale
    scale = np.abs(x).astype(np.float64) @ np.abs(w).astype(np.float64).T
    err = np.abs(y - ref)
    assert np.all(np.isfinite(y))
    assert float(np.max(err / np.maximum(scale, 1e-30))) < 1e-5, float(np.max(err / np.maximum(scale, 1e-30)))
    assert parity.rel_l2(y, ref) < 1e-5  # measured <= 2.8e-6 at K = 2048


@pytest.fixture(scope="module")
def small(lib):
    model = gdn.Model(header=header_for(ol.SMALL_DIMS), seed=SEED)
    oracle = ol.Oracle(ol.SMALL_DIMS, seed=SEED)
    return model, oracle


def run_against_oracle(model, oracle, streams, steps, seeded_streams=(), check_state=True):
    """Advance `streams` streams for `steps` steps on the GPU and in the oracle
    (FP32 control), stream s from zero state or, for s in seeded_streams, from
    the oracle's seeded state 1000 + s. Returns the worst logits rel-L2."""
    batch = gdn.Batch(model, streams)
    init = {}
    for s in range(streams):
        oracle.reset_state(1000 + s if s in seeded_streams else 0)
        init[s] = (oracle.rec.copy(), oracle.conv.copy())
        if s in seeded_streams:
            batch.load_state(s, *init[s])
    toks = np.array([[oracle.token(STREAM_SEED, s, i) for s in range(streams)] for i in range(steps)],
                    dtype=np.int32)
    gpu_logits, gpu_tokens = [], []
    for i in range(steps):
        am, lg = batch.step(toks[i], with_logits=True)
        gpu_logits.append(lg)
        gpu_tokens.append(am)
    worst = 0.0
    for s in range(streams):
        oracle.rec[:], oracle.conv[:] = init[s]
        for i in range(steps):
            ref = oracle.step(int(toks[i, s]), ol.FP32_CONTROL)
            e = parity.rel_l2(gpu_logits[i][s], ref.logits)
            worst = max(worst, e)
            assert e <= parity.LOGITS_FP32, (s, i, e)
            assert parity.argmax_agrees(gpu_logits[i][s], ref.logits, gpu_tokens[i][s]), (s, i)
        if check_state:
            rec, conv = batch.read_state(s)
            assert parity.rel_l2(rec, oracle.rec) <= parity.STATE
            assert parity.rel_l2(conv, oracle.conv) <= parity.LOGITS_FP32
    batch.free()
    return worst


def test_batch_small_matches_oracle(small):
    model, oracle = small
    worst = run_against_oracle(model, oracle, streams=3, steps=6, seeded_streams=(1,))
    print(f"small model, 3 streams x 6 steps: worst logits rel-L2 {worst:.3e}")


def test_batch_two_passes(small):
    """More than 80 streams: two GEMM passes per projection (80 + 50). Streams
    0, 79, 80 and 129 are checked against the oracle; the rest ride along."""
    model, oracle = small
    streams, steps = 130, 3
    batch = gdn.Batch(model, streams)
    toks = np.array([[oracle.token(STREAM_SEED, s, i) for s in range(streams)] for i in range(steps)],
                    dtype=np.int32)
    logits = []
    for i in range(steps):
        _, lg = batch.step(toks[i], with_logits=True)
        logits.append(lg)
    for s in (0, 79, 80, 129):
        oracle.reset_state(0)
        for i in range(steps):
            ref = oracle.step(int(toks[i, s]), ol.FP32_CONTROL)
            assert parity.rel_l2(logits[i][s], ref.logits) <= parity.LOGITS_FP32, (s, i)
    batch.free()


def test_batch_streams_are_independent(small):
    """Streams fed the same tokens from the same state produce the same
    logits whatever their position in the batch."""
    model, oracle = small
    batch = gdn.Batch(model, 5)
    for i in range(3):
        tok = oracle.token(STREAM_SEED, 0, i)
        _, lg = batch.step([tok] * 5, with_logits=True)
        for s in range(1, 5):
            assert parity.rel_l2(lg[s], lg[0]) <= 1e-6
    batch.free()


def test_batch_device_loop_matches_host_steps(small):
    """gdn_b200_batch_decode_tokens (tokens on the device, teacher-forced and
    greedy) gives the tokens of the same steps taken one by one from the host."""
    model, oracle = small
    streams, steps = 4, 5
    toks = np.array([[oracle.token(STREAM_SEED, s, i) for s in range(streams)] for i in range(steps)],
                    dtype=np.int32)
    a = gdn.Batch(model, streams)
    host = np.stack([a.step(toks[i]) for i in range(steps)])
    a.reset()
    dev, ms = a.decode(toks)
    np.testing.assert_array_equal(dev, host)
    assert ms > 0.0
    # greedy: each stream feeds its own argmax back
    a.reset()
    g, _ = a.decode(toks[:1].repeat(steps, axis=0), greedy=True)
    a.reset()
    cur = toks[0].copy()
    for i in range(steps):
        cur = a.step(cur)
        np.testing.assert_array_equal(g[i], cur)
    a.free()


def test_batch_rejects_bad_tokens(small):
    model, _ = small
    b = gdn.Batch(model, 2)
    with pytest.raises(RuntimeError):
        b.step([0, model.config.vocab_size])
    b.step([0, 1])  # still usable
    b.free()


def test_batch_small_long_trajectory(small):
    """64 steps: the reordered FP32 sums must not drift toward the gate."""
    model, oracle = small
    worst = run_against_oracle(model, oracle, streams=2, steps=64, seeded_streams=(0,))
    print(f"small model, 2 streams x 64 steps: worst logits rel-L2 {worst:.3e}")


def test_batch_full_model_matches_oracle(lib):
    model = gdn.Model(header=header_for(ol.FULL_DIMS), seed=SEED)
    oracle = ol.Oracle(ol.FULL_DIMS, seed=SEED)
    worst = run_against_oracle(model, oracle, streams=2, steps=8, seeded_streams=(1,))
    print(f"GDN-1.3B, 2 streams x 8 steps: worst logits rel-L2 {worst:.3e}")
