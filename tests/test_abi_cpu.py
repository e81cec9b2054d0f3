"""CPU tests of the C-ABI library (no GPU needed): symbol coverage of
include/*.h, the .gdnw loader's validation (c_impl/gdn_model.cpp:1082-1229),
the seeded weight generator, and the host-side reference helpers
(gdn_native_bf16_mul_to_fp32, gdn_compute_logits) against the oracle."""
import ctypes
import os
import re
import struct

import numpy as np
import pytest

import gateddeltanet_b200 as gdn
import oracle_lib as ol

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SMALL = ol.SMALL_DIMS


@pytest.fixture(scope="module")
def lib():
    from gateddeltanet_b200 import build
    build.build()
    return gdn.lib()


def small_header(**kw):
    d = dict(SMALL)
    d.update(kw)
    return gdn.make_header(vocab=d["vocab"], hidden=d["hidden"], layers=d["layers"], heads=d["heads"],
                           head_dim=d["head_dim"], inter=d["inter"], conv=d["conv"], eps=d["eps"])


def declared_functions():
    names = set()
    for h in ("gdn_model.h", "gdn_b200.h"):
        src = open(os.path.join(REPO, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(gdn_[a-z0-9_]+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"
    assert {n for n, _, _ in gdn.EXPORTS} == names


def test_synth_matches_oracle_generator(lib):
    model = gdn.Model(header=small_header(), seed=42)
    o = ol.Oracle(SMALL, seed=42, threads=4)
    blob = np.ctypeslib.as_array(model.m.weight_data, shape=(o.blob.size,))
    np.testing.assert_array_equal(blob.view(np.uint32), o.blob.view(np.uint32))
    assert (blob.view(np.uint32) & 0xFFFF).max() == 0  # BF16-exact words
    # norm weights are 1.0, linear weights have std ~0.02
    emb = blob[:SMALL["vocab"] * SMALL["hidden"]]
    assert abs(float(emb.std()) - 0.02) < 0.001
    model.free()


def test_gdnw_roundtrip_and_rejections(lib, tmp_path):
    model = gdn.Model(header=small_header(), seed=3)
    path = str(tmp_path / "m.gdnw")
    model.save(path)
    m2 = gdn.Model(path=path)
    n = os.path.getsize(path) // 4 - 15
    a = np.ctypeslib.as_array(model.m.weight_data, shape=(n,))
    b = np.ctypeslib.as_array(m2.m.weight_data, shape=(n,))
    np.testing.assert_array_equal(a, b)
    # views follow the blob order (c_impl/gdn_model.cpp:1102-1159)
    H, nh = SMALL["hidden"], SMALL["heads"]
    base = ctypes.addressof(m2.m.weight_data.contents)
    l0 = m2.m.layers[0]
    assert ctypes.addressof(l0.attn_norm.contents) - base == 4 * SMALL["vocab"] * H
    assert ctypes.addressof(l0.q_proj.contents) - ctypes.addressof(l0.attn_norm.contents) == 4 * (H + 2 * nh)
    m2.free()
    raw = bytearray(open(path, "rb").read())

    def reject(mutated, what):
        p = str(tmp_path / f"bad_{what}.gdnw")
        open(p, "wb").write(bytes(mutated))
        m = gdn.GDNModel()
        assert lib.gdn_model_load(ctypes.byref(m), p.encode()) == -1, what
        assert not m.weight_data

    bad = bytearray(raw); bad[0:6] = b"XXXXXX"; reject(bad, "magic")
    bad = bytearray(raw); bad[8:12] = struct.pack("<I", 2); reject(bad, "version")
    bad = bytearray(raw); bad[24:28] = struct.pack("<I", 3); reject(bad, "v_heads")
    bad = bytearray(raw); bad[28:32] = struct.pack("<I", 128); reject(bad, "head_dim")
    bad = bytearray(raw); bad[60 + 4 * 1000] ^= 0x01; reject(bad, "not_bf16_exact")
    reject(raw[:-4], "truncated")
    model.free()


def test_run_state_rejects_max_tokens(lib):
    model = gdn.Model(header=small_header(), seed=3)
    st = gdn.GDNRunState()
    assert lib.gdn_run_state_init(ctypes.byref(st), ctypes.byref(model.m), 0) == -1
    assert lib.gdn_run_state_init(ctypes.byref(st), ctypes.byref(model.m), model.config.max_seq_len + 1) == -1
    model.free()


def test_native_product_matches_oracle(lib):
    o = ol.load()
    rng = np.random.default_rng(5)
    w = rng.integers(0, 65536, 20000, dtype=np.uint32)
    a = rng.integers(0, 65536, 20000, dtype=np.uint32)
    specials = [0x0000, 0x8000, 0x0001, 0x7f80, 0xff80, 0x7fc0, 0x0080, 0x00ff, 0x3f80, 0x7f7f]
    w = np.concatenate([w, np.repeat(specials, len(specials))])
    a = np.concatenate([a, np.tile(specials, len(specials))])
    for x, y in zip(w.tolist(), a.tolist()):
        got = struct.unpack("<I", struct.pack("<f", lib.gdn_native_bf16_mul_to_fp32(x, y)))[0]
        exp = o.gdn_oracle_native_product_bits(x, y)
        assert got == exp, (hex(x), hex(y), hex(got), hex(exp))


def test_compute_logits_matches_oracle(lib):
    """gdn_compute_logits (the reference's independent scalar LM head) is
    restated bit-exactly by the oracle."""
    model = gdn.Model(header=small_header(), seed=9)
    o = ol.load()
    o.gdn_oracle_compute_logits.argtypes = [ctypes.POINTER(ol.Dims), ol._fp, ol._fp, ol._fp, ctypes.c_int]
    d = ol.Dims(**SMALL)
    n = o.gdn_oracle_weight_floats(ctypes.byref(d))
    blob = np.ctypeslib.as_array(model.m.weight_data, shape=(n,))
    hidden = np.random.default_rng(1).standard_normal(SMALL["hidden"]).astype(np.float32)
    got = model.compute_logits(hidden)
    exp = np.empty(SMALL["vocab"], dtype=np.float32)
    o.gdn_oracle_compute_logits(ctypes.byref(d), ol.ptr(blob), ol.ptr(hidden), ol.ptr(exp), 4)
    np.testing.assert_array_equal(got.view(np.uint32), exp.view(np.uint32))
    model.free()
