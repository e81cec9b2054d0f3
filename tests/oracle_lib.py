"""ctypes wrapper of the CPU oracle (oracle/libgdn_oracle.so) for the tests.

Test infrastructure only: the oracle is the checker the B200 engine is
compared against. It restates c_impl/gdn_model.cpp's decode step; its own pin
against the reference is tests/test_oracle_golden.py.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_SO = os.path.join(REPO, "oracle", "libgdn_oracle.so")
REF_DRIVER = os.path.join(REPO, "oracle", "_ref", "gdn_ref_driver")


class Dims(ctypes.Structure):
    _fields_ = [
        ("vocab", ctypes.c_uint32),
        ("hidden", ctypes.c_uint32),
        ("layers", ctypes.c_uint32),
        ("heads", ctypes.c_uint32),
        ("head_dim", ctypes.c_uint32),
        ("inter", ctypes.c_uint32),
        ("conv", ctypes.c_uint32),
        ("eps", ctypes.c_float),
    ]


class Mode(ctypes.Structure):
    _fields_ = [("native_product", ctypes.c_int), ("bf16_state", ctypes.c_int), ("bf16_boundary", ctypes.c_int)]


REFERENCE_MODE = (1, 1, 1)   # native products, BF16 state, BF16 boundaries
ENGINE_MODE = (0, 0, 1)      # exact products, FP32 state, BF16 boundaries
FP32_CONTROL = (0, 0, 0)     # exact products, FP32 state, FP32 boundaries

FULL_DIMS = dict(vocab=32000, hidden=2048, layers=24, heads=8, head_dim=256, inter=5632, conv=4, eps=1e-6)
SMALL_DIMS = dict(vocab=4096, hidden=512, layers=2, heads=2, head_dim=256, inter=1536, conv=4, eps=1e-6)

_fp = ctypes.POINTER(ctypes.c_float)


def build_oracle() -> None:
    subprocess.run(["make", "-s", "-C", os.path.join(REPO, "oracle"), "oracle"], check=True)


def load() -> ctypes.CDLL:
    if not os.path.exists(ORACLE_SO):
        build_oracle()
    lib = ctypes.CDLL(ORACLE_SO)
    lib.gdn_oracle_weight_floats.restype = ctypes.c_size_t
    lib.gdn_oracle_weight_floats.argtypes = [ctypes.POINTER(Dims)]
    lib.gdn_oracle_rec_floats.restype = ctypes.c_size_t
    lib.gdn_oracle_rec_floats.argtypes = [ctypes.POINTER(Dims)]
    lib.gdn_oracle_conv_floats.restype = ctypes.c_size_t
    lib.gdn_oracle_conv_floats.argtypes = [ctypes.POINTER(Dims)]
    lib.gdn_oracle_synth_weights.restype = None
    lib.gdn_oracle_synth_weights.argtypes = [ctypes.POINTER(Dims), ctypes.c_uint64, _fp, ctypes.c_int]
    lib.gdn_oracle_synth_token.restype = ctypes.c_int32
    lib.gdn_oracle_synth_token.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32]
    lib.gdn_oracle_synth_state.restype = None
    lib.gdn_oracle_synth_state.argtypes = [ctypes.POINTER(Dims), ctypes.c_uint64, _fp, _fp]
    lib.gdn_oracle_step.restype = ctypes.c_int
    lib.gdn_oracle_step.argtypes = [ctypes.POINTER(Dims), _fp, Mode, _fp, _fp, ctypes.c_int32,
                                    _fp, _fp, ctypes.POINTER(ctypes.c_int32), ctypes.c_int]
    lib.gdn_oracle_bf16_rne_bits.restype = ctypes.c_uint16
    lib.gdn_oracle_bf16_rne_bits.argtypes = [ctypes.c_uint32]
    lib.gdn_oracle_native_product_bits.restype = ctypes.c_uint32
    lib.gdn_oracle_native_product_bits.argtypes = [ctypes.c_uint16, ctypes.c_uint16]
    lib.gdn_oracle_row_dot.restype = ctypes.c_float
    lib.gdn_oracle_row_dot.argtypes = [_fp, _fp, ctypes.c_uint32, ctypes.c_int]
    lib.gdn_oracle_delta_rule_head.restype = None
    lib.gdn_oracle_delta_rule_head.argtypes = [_fp, _fp, _fp, _fp, ctypes.c_float, ctypes.c_float,
                                               ctypes.c_int, _fp]
    return lib


def ptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_fp)


@dataclass
class StepOut:
    logits: np.ndarray
    hidden: np.ndarray
    argmax: int


class Oracle:
    """A model instance of the oracle: seeded weights plus a decode state."""

    def __init__(self, dims: dict, seed: int, state_seed: int = 0, threads: int | None = None,
                 lib: ctypes.CDLL | None = None):
        self.lib = lib or load()
        self.dims = Dims(**dims)
        self.threads = threads or max(1, os.cpu_count() or 1)
        n = self.lib.gdn_oracle_weight_floats(ctypes.byref(self.dims))
        self.blob = np.empty(n, dtype=np.float32)
        self.lib.gdn_oracle_synth_weights(ctypes.byref(self.dims), seed, ptr(self.blob), self.threads)
        self.rec = np.zeros(self.lib.gdn_oracle_rec_floats(ctypes.byref(self.dims)), dtype=np.float32)
        self.conv = np.zeros(self.lib.gdn_oracle_conv_floats(ctypes.byref(self.dims)), dtype=np.float32)
        if state_seed:
            self.lib.gdn_oracle_synth_state(ctypes.byref(self.dims), state_seed, ptr(self.rec), ptr(self.conv))

    def reset_state(self, state_seed: int = 0) -> None:
        """Zero state, or the seeded BF16-exact initial state."""
        self.rec[:] = 0.0
        self.conv[:] = 0.0
        if state_seed:
            self.lib.gdn_oracle_synth_state(ctypes.byref(self.dims), state_seed, ptr(self.rec), ptr(self.conv))

    def token(self, stream_seed: int, stream: int, i: int) -> int:
        return int(self.lib.gdn_oracle_synth_token(stream_seed, stream, i, self.dims.vocab))

    def step(self, token: int, mode=ENGINE_MODE) -> StepOut:
        logits = np.empty(self.dims.vocab, dtype=np.float32)
        hidden = np.empty(self.dims.hidden, dtype=np.float32)
        am = ctypes.c_int32(-1)
        rc = self.lib.gdn_oracle_step(ctypes.byref(self.dims), ptr(self.blob), Mode(*mode), ptr(self.rec),
                                      ptr(self.conv), int(token), ptr(logits), ptr(hidden), ctypes.byref(am),
                                      self.threads)
        if rc != 0:
            raise ValueError(f"oracle step rejected token {token}")
        return StepOut(logits, hidden, int(am.value))


def read_ref_dump(path: str):
    """Parse the binary written by oracle/_ref/gdn_ref_driver --out."""
    with open(path, "rb") as f:
        data = f.read()
    assert data[:8] == b"GDNREF01"
    steps, vocab, hidden, _ = np.frombuffer(data[8:24], dtype=np.uint32)
    off = 24
    out = []
    for _ in range(int(steps)):
        tok, pick = np.frombuffer(data[off:off + 8], dtype=np.int32)
        ms = float(np.frombuffer(data[off + 8:off + 16], dtype=np.float64)[0])
        off += 16
        logits = np.frombuffer(data[off:off + 4 * vocab], dtype=np.float32).copy()
        off += 4 * int(vocab)
        hid = np.frombuffer(data[off:off + 4 * hidden], dtype=np.float32).copy()
        off += 4 * int(hidden)
        out.append(dict(token=int(tok), argmax=int(pick), ms=ms, logits=logits, hidden=hid))
    rest = np.frombuffer(data[off:], dtype=np.float32)
    return out, rest
