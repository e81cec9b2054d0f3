"""The reference's own native evaluator, unmodified, on this library.

oracle/_ref/gdn_eval_b200 is c_impl/gdn_eval.cpp compiled from the
reference's sources and linked against libgdn_b200.so instead of the
reference's gdn_model.o (`make -C oracle eval-b200`). With
GDN_B200_ABI_COMPAT=1 it loads a .gdnw, validates the packed weight shards,
loads a .gdnstate through gdn_scatter_recurrent_state /
gdn_pack_conv_tails_bf16 and decodes greedily from the state's seed token --
every step on the GPU -- while checking, itself:
  * the kernel's logits against the independent scalar LM head (gdn_compute_logits),
  * the on-chip argmax against its own scan of the logits,
  * the logits bit for bit against a reference dump (--logits-reference),
which here is the CPU oracle in the reference's arithmetic (pinned to the
reference by tests/test_oracle_golden.py). Its state dump (--dump-state)
reads the BF16 state stripes, which the library keeps in step.
"""
import json
import os
import struct
import subprocess

import numpy as np
import pytest

import gateddeltanet_b200 as gdn
import oracle_lib as ol
import parity

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EVAL = os.path.join(REPO, "oracle", "_ref", "gdn_eval_b200")
SEED = 20261201


def write_gdnstate(path, dims, rec, conv, seed_token):
    with open(path, "wb") as f:
        f.write(b"GDNSTAT1")
        f.write(struct.pack("<9I", 1, dims["layers"], dims["heads"], dims["head_dim"], dims["head_dim"],
                            dims["hidden"], dims["conv"], 0, seed_token & 0xFFFFFFFF))
        f.write(np.ascontiguousarray(rec, dtype=np.float32).tobytes())
        f.write(np.ascontiguousarray(conv, dtype=np.float32).tobytes())


def write_fixture(path, ctx, cont):
    with open(path, "wb") as f:
        f.write(b"GDNREQ1\0")
        f.write(struct.pack("<3I", 1, 2, 1))  # version, kind LL, one example
        f.write(struct.pack("<2I", len(ctx), len(cont)))
        f.write(np.asarray(ctx, dtype=np.int32).tobytes())
        f.write(np.asarray(cont, dtype=np.int32).tobytes())


@pytest.mark.skipif(not os.path.exists(EVAL), reason="oracle/_ref/gdn_eval_b200 not built (make -C oracle eval-b200)")
def test_reference_gdn_eval_decodes_on_the_gpu(tmp_path):
    from gateddeltanet_b200 import build
    build.build()
    dims = ol.FULL_DIMS
    hdr = gdn.make_header(vocab=dims["vocab"], hidden=dims["hidden"], layers=dims["layers"], heads=dims["heads"],
                          head_dim=dims["head_dim"], inter=dims["inter"], conv=dims["conv"], eps=dims["eps"])
    model = gdn.Model(header=hdr, seed=SEED)
    weights = str(tmp_path / "model.gdnw")
    model.save(weights)
    model.free()

    oracle = ol.Oracle(dims, seed=SEED)
    oracle.reset_state(7)
    rec0, conv0 = oracle.rec.copy(), oracle.conv.copy()
    seed_token = oracle.token(31, 0, 0)
    n = 6
    traj, ref_logits = [seed_token], []
    for step in range(1, n):
        out = oracle.step(traj[-1], ol.REFERENCE_MODE)
        ref_logits.append(out.logits.astype(np.float32))
        traj.append(parity.argmax_first(out.logits))
    state = str(tmp_path / "prompt.gdnstate")
    write_gdnstate(state, dims, rec0, conv0, seed_token)
    fixture = str(tmp_path / "decode.gdnreq")
    write_fixture(fixture, [seed_token], traj[1:])
    logref = str(tmp_path / "ref.gdnlog")
    with open(logref, "wb") as f:
        f.write(b"GDNLOG1\0" + struct.pack("<3I", 1, dims["vocab"], n - 1))
        for lg in ref_logits:
            f.write(lg.tobytes())
    out_json = str(tmp_path / "decode.json")
    dump = str(tmp_path / "state.gdnsdmp")
    env = dict(os.environ, GDN_B200_ABI_COMPAT="1")
    run = subprocess.run([EVAL, weights, fixture, out_json, "--decode", "--decode-from-state", state, "--decode-len",
                          str(n), "--logits-reference", logref, "--dump-state", dump],
                         env=env, capture_output=True, text=True, timeout=900)
    assert run.returncode == 0, run.stderr[-3000:]
    res = json.loads(open(out_json).read())
    ex = res["examples"][0]
    assert ex["gen_traj"] == traj
    lp = res["logits_parity"]
    assert lp["checked_steps"] == n - 1
    assert lp["exact_reference_mismatches"] == 0 and lp["argmax_mismatches"] == 0
    assert lp["cpu_tolerance_failures"] == 0
    # the state dump reads the library's BF16 stripes: the oracle's state after
    # the same steps, within the state gate
    data = open(dump, "rb").read()
    assert data[:8] == b"GDNSDMP1"
    stripe_beats, ports, head_beats, _ = struct.unpack("<4I", data[8:24])
    L = gdn.lib()
    stripes = [np.frombuffer(data, dtype=np.uint8, count=64 * stripe_beats, offset=24 + p * 64 * stripe_beats).copy()
               for p in range(ports)]
    expect = [np.zeros(64 * stripe_beats, dtype=np.uint8) for _ in range(ports)]
    import ctypes
    ptrs = (ctypes.c_void_p * ports)(*[e.ctypes.data for e in expect])
    rec = np.ascontiguousarray(oracle.rec, dtype=np.float32)
    assert L.gdn_scatter_recurrent_state(ptrs, rec.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), rec.size) == 0
    got = np.concatenate([s.view(np.uint16) for s in stripes]).astype(np.uint32) << 16
    ref = np.concatenate([e.view(np.uint16) for e in expect]).astype(np.uint32) << 16
    assert parity.rel_l2(got.view(np.float32), ref.view(np.float32)) <= parity.STATE
