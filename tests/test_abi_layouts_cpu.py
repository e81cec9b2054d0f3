"""The reference's host image helpers as exported by libgdn_b200.so
(gateddeltanet_b200/csrc/gdn_abi_host.cpp), against digests of the reference's
own implementation (c_impl/gdn_model.cpp:595-1080, run natively by
oracle/ref_driver.cpp --layouts; tests/golden/reference_goldens.json). Pure
host code: no GPU is touched.
"""
import ctypes
import hashlib
import json
import os

import numpy as np
import pytest

import gateddeltanet_b200 as gdn
import oracle_lib as ol

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = json.load(open(os.path.join(HERE, "golden", "reference_goldens.json")))
LAY = GOLD["layouts"]
FP = ctypes.POINTER(ctypes.c_float)
VP = ctypes.c_void_p


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def lib():
    from gateddeltanet_b200 import build
    build.build()
    L = gdn.lib()
    return L


@pytest.fixture(scope="module")
def small(lib):
    m = LAY["model"]
    dims = dict(vocab=m["vocab"], hidden=m["hidden"], layers=m["layers"], heads=m["heads"], head_dim=m["head_dim"],
                inter=m["inter"], conv=m["conv"], eps=1e-6)
    o = ol.Oracle(dims, seed=m["seed"], threads=os.cpu_count() or 1)
    hdr = gdn.make_header(**dims)
    return o, hdr, dims


def test_weight_shards_match_reference(lib, small):
    o, hdr, _ = small
    sb = lib.gdn_weight_shard_beats(ctypes.byref(hdr))
    assert sb == LAY["shard_beats"]
    assert lib.gdn_weight_shard_bytes(ctypes.byref(hdr)) == 64 * sb
    shards = np.zeros((32, sb * 64), dtype=np.uint8)
    ptrs = (VP * 32)(*[shards[c].ctypes.data for c in range(32)])
    blob = o.blob.ctypes.data_as(FP)
    lib.gdn_build_weight_shards(blob, ctypes.byref(hdr), ptrs)
    assert [sha(shards[c]) for c in range(32)] == LAY["shard_sha256"]
    assert lib.gdn_validate_weight_shards(blob, ctypes.byref(hdr), ptrs) == 0
    shards[5, 1000] ^= 1  # a corrupted lane is caught
    assert lib.gdn_validate_weight_shards(blob, ctypes.byref(hdr), ptrs) == -1
    assert lib.gdn_validate_bf16_exact_weights(blob, ctypes.byref(hdr)) == 0


def test_aux_image_matches_reference(lib, small):
    o, hdr, _ = small
    n = lib.gdn_aux_image_beats(ctypes.byref(hdr))
    assert n == LAY["aux_beats"]
    aux = np.zeros(n * 64, dtype=np.uint8)
    blob = o.blob.ctypes.data_as(FP)
    lib.gdn_build_aux_image(blob, ctypes.byref(hdr), aux.ctypes.data_as(VP))
    assert sha(aux) == LAY["aux_sha256"]
    assert lib.gdn_validate_aux_image(aux.ctypes.data_as(VP), blob, ctypes.byref(hdr)) == 0
    aux[64 * 3 + 7] ^= 0x10
    assert lib.gdn_validate_aux_image(aux.ctypes.data_as(VP), blob, ctypes.byref(hdr)) == -1


def test_state_stripes_and_conv_packing_match_reference(lib, small):
    o, _, dims = small
    o.reset_state(LAY["state_seed"])
    rec = o.rec.copy()
    stb = LAY["stripe_beats"]
    stripes = np.zeros((4, stb * 64), dtype=np.uint8)
    ptrs = (VP * 4)(*[stripes[p].ctypes.data for p in range(4)])
    assert lib.gdn_scatter_recurrent_state(ptrs, rec.ctypes.data_as(FP), ctypes.c_size_t(rec.size)) == 0
    assert sha(stripes) == LAY["stripes_sha256"]
    rec[3] = np.float32(1.0 + 2 ** -10)  # not BF16-exact
    assert lib.gdn_scatter_recurrent_state(ptrs, rec.ctypes.data_as(FP), ctypes.c_size_t(rec.size)) == -1
    # conv tails of the full shape (GDN_WSF_HEADBUF floats) from the same generator
    d = ol.Dims(**ol.FULL_DIMS)
    conv = np.zeros(o.lib.gdn_oracle_conv_floats(ctypes.byref(d)), dtype=np.float32)
    big_rec = np.zeros(o.lib.gdn_oracle_rec_floats(ctypes.byref(d)), dtype=np.float32)
    o.lib.gdn_oracle_synth_state(ctypes.byref(d), LAY["conv_seed_full_dims"], big_rec.ctypes.data_as(FP),
                                 conv.ctypes.data_as(FP))
    head = np.zeros(LAY["conv_head_beats"] * 64, dtype=np.uint8)
    assert lib.gdn_pack_conv_tails_bf16(head.ctypes.data_as(VP), conv.ctypes.data_as(FP),
                                        ctypes.c_size_t(conv.size)) == 0
    assert sha(head) == LAY["conv_head_sha256"]
    assert lib.gdn_pack_conv_tails_bf16(head.ctypes.data_as(VP), conv.ctypes.data_as(FP),
                                        ctypes.c_size_t(conv.size - 1)) == -1


def test_lane_helpers_match_reference_primitives(lib):
    prim = GOLD["primitives"]
    xs = (np.arange(65536, dtype=np.uint64) * 65521) & 0xFFFFFFFF
    rne = np.array([lib.gdn_test_fp32_to_bf16_rne_bits(int(x)) for x in xs], dtype=np.uint16)
    assert sha(rne) == prim["rne_set_a_sha256"]
    beat = (ctypes.c_uint8 * 64)()
    lib.gdn_test_set_bf16_lane_bits(ctypes.byref(beat), 31, 0xBEEF)
    lib.gdn_test_set_fp32_lane_bits(ctypes.byref(beat), 0, 0x12345678)
    assert bytes(beat)[62:64] == b"\xef\xbe" and bytes(beat)[0:4] == b"\x78\x56\x34\x12"
    assert lib.gdn_test_get_bf16_lane_bits(ctypes.byref(beat), 31) == 0xBEEF
    assert lib.gdn_test_get_fp32_lane_bits(ctypes.byref(beat), 0) == 0x12345678
    assert lib.gdn_test_bf16_to_fp32_bits(0x3F80) == 0x3F800000
