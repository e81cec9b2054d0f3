"""gateddeltanet_b200 -- B200-native GatedDeltaNet-1.3B decode engine.

The product is libgdn_b200.so (built in-tree by gateddeltanet_b200.build): a
C-ABI library exporting the reference's decode interface (c_impl/gdn_model.h:
gdn_model_load, gdn_run_state_init, gdn_decode_step_host, gdn_compute_logits,
...) over hand-written sm_100a CUDA. This module is a thin ctypes host layer
over that ABI for Python callers (tests, bench.py); it performs no
computation of its own and raises if the native library is missing.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import numpy as np

__all__ = [
    "GDNWeightHeader", "GDNLayerWeights", "GDNModel", "GDNRunState", "lib", "make_header",
    "Model", "RunState", "GDN_WS_OFF_X", "GDN_WS_OFF_X_NORM", "GDN_WS_OFF_LOGITS", "GDN_WS_FLOATS",
]

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgdn_b200.so")

# Workspace float offsets, c_impl/gdn_model.h:54-75 (same values as include/gdn_model.h).
GDN_WSF_HID, GDN_WSF_HEAD, GDN_WSF_MLP = 2048, 16, 5632
GDN_WSF_STATE, GDN_WSF_HEADBUF, GDN_WSF_LOGITS = 12582912, 442368, 32000
GDN_WS_OFF_X = 0
GDN_WS_OFF_X_NORM = GDN_WS_OFF_X + GDN_WSF_HID
GDN_WS_OFF_Q = GDN_WS_OFF_X_NORM + GDN_WSF_HID
GDN_WS_OFF_K = GDN_WS_OFF_Q + GDN_WSF_HID
GDN_WS_OFF_V = GDN_WS_OFF_K + GDN_WSF_HID
GDN_WS_OFF_A = GDN_WS_OFF_V + GDN_WSF_HID
GDN_WS_OFF_B = GDN_WS_OFF_A + GDN_WSF_HEAD
GDN_WS_OFF_GATE = GDN_WS_OFF_B + GDN_WSF_HEAD
GDN_WS_OFF_ATTN = GDN_WS_OFF_GATE + GDN_WSF_HID
GDN_WS_OFF_TMP_HIDDEN = GDN_WS_OFF_ATTN + GDN_WSF_HID
GDN_WS_OFF_MLP_GATE = GDN_WS_OFF_TMP_HIDDEN + GDN_WSF_HID
GDN_WS_OFF_MLP_UP = GDN_WS_OFF_MLP_GATE + GDN_WSF_MLP
GDN_WS_OFF_REC_STATE = GDN_WS_OFF_MLP_UP + GDN_WSF_MLP
GDN_WS_OFF_HEAD_BUF = GDN_WS_OFF_REC_STATE + GDN_WSF_STATE
GDN_WS_OFF_LOGITS = GDN_WS_OFF_HEAD_BUF + GDN_WSF_HEADBUF
GDN_WS_FLOATS = GDN_WS_OFF_LOGITS + GDN_WSF_LOGITS


class GDNWeightHeader(ctypes.Structure):
    """c_impl/gdn_model.h:30-45 (60 bytes)."""
    _fields_ = [
        ("magic", ctypes.c_char * 8), ("version", ctypes.c_uint32), ("vocab_size", ctypes.c_uint32),
        ("hidden_size", ctypes.c_uint32), ("num_layers", ctypes.c_uint32), ("num_heads", ctypes.c_uint32),
        ("num_v_heads", ctypes.c_uint32), ("head_dim", ctypes.c_uint32), ("intermediate_size", ctypes.c_uint32),
        ("conv_size", ctypes.c_uint32), ("max_seq_len", ctypes.c_uint32), ("bos_token_id", ctypes.c_int32),
        ("eos_token_id", ctypes.c_int32), ("norm_eps", ctypes.c_float),
    ]


_FP = ctypes.POINTER(ctypes.c_float)


class GDNLayerWeights(ctypes.Structure):
    """c_impl/gdn_model.h:123-142."""
    _fields_ = [(n, _FP) for n in (
        "attn_norm", "a_log", "dt_bias", "q_proj", "k_proj", "v_proj", "a_proj", "b_proj", "q_conv", "k_conv",
        "v_conv", "g_proj", "o_norm", "o_proj", "mlp_norm", "mlp_gate_proj", "mlp_up_proj", "mlp_down_proj")]


class GDNModel(ctypes.Structure):
    """c_impl/gdn_model.h:144-151."""
    _fields_ = [("config", GDNWeightHeader), ("weight_data", _FP), ("layers", ctypes.POINTER(GDNLayerWeights)),
                ("embeddings", _FP), ("final_norm", _FP), ("lm_head", _FP)]


class GDNRunState(ctypes.Structure):
    """c_impl/gdn_model.h:153-160."""
    _fields_ = [("workspace", ctypes.c_void_p), ("x", _FP), ("recurrent_state", _FP), ("head_buffer", _FP),
                ("weight_shards", ctypes.c_void_p * 32), ("aux_weights", ctypes.c_void_p)]


assert ctypes.sizeof(GDNWeightHeader) == 60

_LIB: Optional[ctypes.CDLL] = None

# (name, restype, argtypes) of every entry point declared in include/gdn_model.h and include/gdn_b200.h
EXPORTS = [
    ("gdn_model_load", ctypes.c_int, [ctypes.POINTER(GDNModel), ctypes.c_char_p]),
    ("gdn_model_free", None, [ctypes.POINTER(GDNModel)]),
    ("gdn_run_state_init", ctypes.c_int, [ctypes.POINTER(GDNRunState), ctypes.POINTER(GDNModel), ctypes.c_uint32]),
    ("gdn_run_state_free", None, [ctypes.POINTER(GDNRunState)]),
    ("gdn_decode_step_host", ctypes.c_int,
     [ctypes.POINTER(GDNModel), ctypes.POINTER(GDNRunState), ctypes.POINTER(ctypes.c_int32)]),
    ("gdn_compute_logits", None, [ctypes.POINTER(GDNModel), _FP, _FP]),
    ("gdn_native_bf16_mul_to_fp32", ctypes.c_float, [ctypes.c_uint16, ctypes.c_uint16]),
    ("gdn_set_native_debug_buffers", None, [_FP, _FP]),
    ("gdn_reset_mixed_mul_stats", None, []),
    ("gdn_get_mixed_mul_stats", None, None),  # returns a struct; argtypes set below
    ("gdn_decode_step_host_partitioned", ctypes.c_int,
     [ctypes.POINTER(GDNModel), ctypes.POINTER(GDNRunState), ctypes.POINTER(ctypes.c_int32)]),
    ("gdn_forward", ctypes.c_int, [ctypes.c_void_p] * 34),
    ("gdn_weight_shard_beats", ctypes.c_size_t, [ctypes.POINTER(GDNWeightHeader)]),
    ("gdn_weight_shard_bytes", ctypes.c_size_t, [ctypes.POINTER(GDNWeightHeader)]),
    ("gdn_validate_bf16_exact_weights", ctypes.c_int, [_FP, ctypes.POINTER(GDNWeightHeader)]),
    ("gdn_build_weight_shards", None, [_FP, ctypes.POINTER(GDNWeightHeader), ctypes.c_void_p]),
    ("gdn_validate_weight_shards", ctypes.c_int, [_FP, ctypes.POINTER(GDNWeightHeader), ctypes.c_void_p]),
    ("gdn_aux_image_beats", ctypes.c_size_t, [ctypes.POINTER(GDNWeightHeader)]),
    ("gdn_build_aux_image", None, [_FP, ctypes.POINTER(GDNWeightHeader), ctypes.c_void_p]),
    ("gdn_validate_aux_image", ctypes.c_int, [ctypes.c_void_p, _FP, ctypes.POINTER(GDNWeightHeader)]),
    ("gdn_scatter_recurrent_state", ctypes.c_int, [ctypes.c_void_p, _FP, ctypes.c_size_t]),
    ("gdn_pack_conv_tails_bf16", ctypes.c_int, [ctypes.c_void_p, _FP, ctypes.c_size_t]),
    ("gdn_test_fp32_to_bf16_rne_bits", ctypes.c_uint16, [ctypes.c_uint32]),
    ("gdn_test_bf16_to_fp32_bits", ctypes.c_uint32, [ctypes.c_uint16]),
    ("gdn_test_set_fp32_lane_bits", None, [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32]),
    ("gdn_test_get_fp32_lane_bits", ctypes.c_uint32, [ctypes.c_void_p, ctypes.c_uint32]),
    ("gdn_test_set_bf16_lane_bits", None, [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint16]),
    ("gdn_test_get_bf16_lane_bits", ctypes.c_uint16, [ctypes.c_void_p, ctypes.c_uint32]),
    ("gdn_b200_set_abi_compat", ctypes.c_int, [ctypes.c_int]),
    ("gdn_b200_set_device", ctypes.c_int, [ctypes.c_int]),
    ("gdn_b200_last_error", ctypes.c_char_p, []),
    ("gdn_b200_model_synth", ctypes.c_int, [ctypes.POINTER(GDNModel), ctypes.POINTER(GDNWeightHeader), ctypes.c_uint64]),
    ("gdn_b200_model_save", ctypes.c_int, [ctypes.POINTER(GDNModel), ctypes.c_char_p]),
    ("gdn_b200_set_numerics", ctypes.c_int, [ctypes.POINTER(GDNRunState), ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    ("gdn_b200_state_upload", ctypes.c_int, [ctypes.POINTER(GDNRunState), _FP, ctypes.c_size_t, _FP, ctypes.c_size_t]),
    ("gdn_b200_state_download", ctypes.c_int, [ctypes.POINTER(GDNRunState), _FP, ctypes.c_size_t, _FP, ctypes.c_size_t]),
    ("gdn_b200_state_load_file", ctypes.c_int, [ctypes.POINTER(GDNRunState), ctypes.c_char_p, ctypes.POINTER(ctypes.c_int32)]),
    ("gdn_b200_state_save_file", ctypes.c_int, [ctypes.POINTER(GDNRunState), ctypes.c_char_p, ctypes.c_int32]),
    ("gdn_b200_fetch_outputs", ctypes.c_int, [ctypes.POINTER(GDNRunState), _FP, _FP]),
    ("gdn_b200_decode_tokens", ctypes.c_int,
     [ctypes.POINTER(GDNModel), ctypes.POINTER(GDNRunState), ctypes.POINTER(ctypes.c_int32), ctypes.c_uint32,
      ctypes.c_int, ctypes.POINTER(ctypes.c_int32), _FP]),
    ("gdn_b200_decode_tokens_noalloc", ctypes.c_int,
     [ctypes.POINTER(GDNModel), ctypes.POINTER(GDNRunState), ctypes.POINTER(ctypes.c_int32), ctypes.c_uint32,
      ctypes.c_int, ctypes.POINTER(ctypes.c_int32), _FP]),
    ("gdn_b200_trace_step", ctypes.c_int,
     [ctypes.POINTER(GDNModel), ctypes.POINTER(GDNRunState), ctypes.c_int32, ctypes.POINTER(ctypes.c_uint64),
      ctypes.c_size_t]),
    ("gdn_b200_delta_rule_step", ctypes.c_int,
     [ctypes.c_uint32, _FP, _FP, _FP, _FP, _FP, _FP, _FP, ctypes.c_uint32, _FP]),
    ("gdn_b200_test_drop_outputs", ctypes.c_int, [ctypes.POINTER(GDNRunState), ctypes.c_int, ctypes.c_int]),
    ("gdn_b200_test_force_exact_products", ctypes.c_int, [ctypes.POINTER(GDNRunState), ctypes.c_int]),
    ("gdn_b200_test_set_epoch", ctypes.c_int, [ctypes.POINTER(GDNRunState), ctypes.c_uint32]),
    ("gdn_b200_test_image_geometry", ctypes.c_int, [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                                     ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]),
    ("gdn_b200_grid_size", ctypes.c_int, []),
    ("gdn_b200_batch_create", ctypes.c_void_p, [ctypes.POINTER(GDNModel), ctypes.c_uint32]),
    ("gdn_b200_batch_free", None, [ctypes.c_void_p]),
    ("gdn_b200_batch_launches_per_step", ctypes.c_uint32, [ctypes.c_void_p]),
    ("gdn_b200_batch_reset", ctypes.c_int, [ctypes.c_void_p]),
    ("gdn_b200_batch_state_upload", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_uint32, _FP, ctypes.c_size_t, _FP, ctypes.c_size_t]),
    ("gdn_b200_batch_state_download", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_uint32, _FP, ctypes.c_size_t, _FP, ctypes.c_size_t]),
    ("gdn_b200_batch_step_host", ctypes.c_int,
     [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32), _FP]),
    ("gdn_b200_batch_decode_tokens", ctypes.c_int,
     [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32), ctypes.c_uint32, ctypes.c_int,
      ctypes.POINTER(ctypes.c_int32), _FP]),
    ("gdn_b200_batch_fetch_logits", ctypes.c_int, [ctypes.c_void_p, _FP]),
    ("gdn_b200_score_window", ctypes.c_int,
     [ctypes.POINTER(GDNModel), ctypes.POINTER(GDNRunState), ctypes.POINTER(ctypes.c_int32), ctypes.c_uint32,
      ctypes.POINTER(ctypes.c_int32), ctypes.c_uint32, ctypes.c_int, ctypes.POINTER(ctypes.c_double),
      ctypes.POINTER(ctypes.c_uint64)]),
    ("gdn_b200_prefill", ctypes.c_int,
     [ctypes.POINTER(GDNModel), ctypes.POINTER(GDNRunState), ctypes.POINTER(ctypes.c_int32), ctypes.c_uint32, _FP]),
    ("gdn_b200_test_tile_gemm", ctypes.c_int,
     [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, _FP, _FP, _FP]),
    ("gdn_b200_tp_token", ctypes.c_int, [ctypes.POINTER(GDNRunState), ctypes.c_void_p]),
    ("gdn_b200_tp_attach", ctypes.c_int, [ctypes.POINTER(GDNRunState), ctypes.c_int, ctypes.c_int, ctypes.c_char_p]),
    ("gdn_b200_tp_detach", ctypes.c_int, [ctypes.POINTER(GDNRunState)]),
    ("gdn_b200_tp_state_download_part", ctypes.c_int,
     [ctypes.POINTER(GDNRunState), ctypes.POINTER(ctypes.c_float), ctypes.c_size_t, ctypes.POINTER(ctypes.c_float),
      ctypes.c_size_t, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32),
      ctypes.POINTER(ctypes.c_int32)]),
]

GDN_B200_TP_TOKEN_BYTES = 128


class GDNMixedMulStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in ("calls", "special_inputs", "flushed_inputs", "flushed_outputs", "overflows")]


def lib(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libgdn_b200.so; raises if it has not been built (no fallback)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise RuntimeError(f"libgdn_b200.so not found at {path}: run `python -m gateddeltanet_b200.build`")
    L = ctypes.CDLL(path)
    for name, res, args in EXPORTS:
        fn = getattr(L, name)
        if name == "gdn_get_mixed_mul_stats":
            fn.restype, fn.argtypes = GDNMixedMulStats, []
            continue
        fn.restype = res
        fn.argtypes = args
    _LIB = L
    return L


def last_error() -> str:
    return lib().gdn_b200_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed: {last_error()}")


def make_header(vocab=32000, hidden=2048, layers=24, heads=8, head_dim=256, inter=5632, conv=4,
                max_seq_len=2048, eps=1e-6, bos=1, eos=2) -> GDNWeightHeader:
    """A .gdnw header (the 1.3B shape by default, c_impl/artifacts/gdn-1.3b-bf16w.json)."""
    return GDNWeightHeader(b"GDNWv1\0\0", 1, vocab, hidden, layers, heads, heads, head_dim, inter, conv,
                           max_seq_len, bos, eos, eps)


def _fptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_FP)


class Model:
    """A loaded (or seeded synthetic) model: GDNModel plus its device image."""

    def __init__(self, path: Optional[str] = None, header: Optional[GDNWeightHeader] = None, seed: int = 1234):
        self.lib = lib()
        self.m = GDNModel()
        if path is not None:
            check(self.lib.gdn_model_load(ctypes.byref(self.m), path.encode()), "gdn_model_load")
        else:
            hdr = header if header is not None else make_header()
            check(self.lib.gdn_b200_model_synth(ctypes.byref(self.m), ctypes.byref(hdr), seed), "gdn_b200_model_synth")

    @property
    def config(self) -> GDNWeightHeader:
        return self.m.config

    def save(self, path: str) -> None:
        check(self.lib.gdn_b200_model_save(ctypes.byref(self.m), path.encode()), "gdn_b200_model_save")

    def compute_logits(self, hidden: np.ndarray) -> np.ndarray:
        out = np.empty(self.config.vocab_size, dtype=np.float32)
        h = np.ascontiguousarray(hidden, dtype=np.float32)
        self.lib.gdn_compute_logits(ctypes.byref(self.m), _fptr(h), _fptr(out))
        return out

    def free(self) -> None:
        if self.m.weight_data:
            self.lib.gdn_model_free(ctypes.byref(self.m))

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class RunState:
    """One decode stream (GDNRunState) of a Model."""

    def __init__(self, model: Model, max_tokens: Optional[int] = None):
        self.model = model
        self.lib = model.lib
        self.s = GDNRunState()
        mt = model.config.max_seq_len if max_tokens is None else max_tokens
        check(self.lib.gdn_run_state_init(ctypes.byref(self.s), ctypes.byref(model.m), mt), "gdn_run_state_init")
        c = model.config
        self.rec_floats = c.num_layers * c.num_heads * c.head_dim * c.head_dim
        self.conv_floats = c.num_layers * 3 * (c.conv_size - 1) * c.hidden_size
        # per-step call objects, built once (step() is on the timed e2e path)
        self._tok = ctypes.c_int32(0)
        self._mref, self._sref, self._tref = ctypes.byref(model.m), ctypes.byref(self.s), ctypes.byref(self._tok)
        self._step = self.lib.gdn_decode_step_host
        self._ws = ctypes.cast(self.s.workspace, _FP)

    def workspace(self, offset: int, count: int) -> np.ndarray:
        ptr = ctypes.cast(self.s.workspace, _FP)
        return np.ctypeslib.as_array(ptr, shape=(GDN_WS_FLOATS,))[offset:offset + count]

    def step(self, token: int) -> int:
        """gdn_decode_step_host; returns the kernel's greedy token (workspace[X_NORM] lane 0)."""
        t = self._tok
        t.value = int(token)
        if self._step(self._mref, self._sref, self._tref) != 0:
            raise RuntimeError(f"gdn_decode_step_host failed: {last_error()}")
        return int(self._ws[GDN_WS_OFF_X_NORM])

    def decode(self, tokens: Sequence[int], greedy: bool = False):
        """Device-resident loop; returns (argmax per step, device ms for all steps)."""
        tok = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        n = len(tok)
        out = np.empty(n, dtype=np.int32)
        ms = ctypes.c_float(0.0)
        check(self.lib.gdn_b200_decode_tokens(ctypes.byref(self.model.m), ctypes.byref(self.s),
                                              tok.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), n, int(greedy),
                                              out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), ctypes.byref(ms)),
              "gdn_b200_decode_tokens")
        return out, float(ms.value)

    def decode_noalloc(self, tokens: Sequence[int], greedy: bool = False):
        """decode() through gdn_b200_decode_tokens_noalloc (no device allocation,
        at most 4096 tokens per call)."""
        tok = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        n = len(tok)
        out = np.empty(n, dtype=np.int32)
        ms = ctypes.c_float(0.0)
        check(self.lib.gdn_b200_decode_tokens_noalloc(ctypes.byref(self.model.m), ctypes.byref(self.s),
                                                      tok.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), n,
                                                      int(greedy), out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                                      ctypes.byref(ms)),
              "gdn_b200_decode_tokens_noalloc")
        return out, float(ms.value)

    def prefill(self, tokens: Sequence[int]) -> float:
        """gdn_b200_prefill: advance by the tokens at once (no logits); returns device ms."""
        tok = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        ms = ctypes.c_float(0.0)
        check(self.lib.gdn_b200_prefill(ctypes.byref(self.model.m), ctypes.byref(self.s),
                                        tok.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), len(tok),
                                        ctypes.byref(ms)), "gdn_b200_prefill")
        return float(ms.value)

    def score_window(self, ctx: Sequence[int], cont: Sequence[int], use_prefill: bool = False):
        """gdn_b200_score_window: (log-probability of cont given ctx, scored tokens); resets the state."""
        a = np.ascontiguousarray(np.asarray(ctx, dtype=np.int32))
        b = np.ascontiguousarray(np.asarray(cont, dtype=np.int32))
        lp = ctypes.c_double(0.0)
        n = ctypes.c_uint64(0)
        P = ctypes.POINTER(ctypes.c_int32)
        check(self.lib.gdn_b200_score_window(ctypes.byref(self.model.m), ctypes.byref(self.s), a.ctypes.data_as(P),
                                             len(a), b.ctypes.data_as(P), len(b), int(bool(use_prefill)),
                                             ctypes.byref(lp), ctypes.byref(n)), "gdn_b200_score_window")
        return float(lp.value), int(n.value)

    def trace(self, token: int) -> np.ndarray:
        """One traced step: array [cta, phase, 8] of %globaltimer ns stamps
        (see gdn_b200_trace_step in include/gdn_b200.h)."""
        c = self.model.config
        grid = self.lib.gdn_b200_grid_size()
        phases = c.num_layers * 5 + 1
        buf = np.zeros(grid * phases * 8, dtype=np.uint64)
        n = self.lib.gdn_b200_trace_step(ctypes.byref(self.model.m), ctypes.byref(self.s), int(token),
                                         buf.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), buf.size)
        if n < 0:
            raise RuntimeError(f"gdn_b200_trace_step failed: {last_error()}")
        return buf.reshape(grid, phases, 8)

    def outputs(self):
        c = self.model.config
        logits = np.empty(c.vocab_size, dtype=np.float32)
        hidden = np.empty(c.hidden_size, dtype=np.float32)
        check(self.lib.gdn_b200_fetch_outputs(ctypes.byref(self.s), _fptr(logits), _fptr(hidden)),
              "gdn_b200_fetch_outputs")
        return logits, hidden

    # the supported numeric contracts (gdn_b200_set_numerics)
    CIMPL = (True, True, True)
    ENGINE = (True, False, False)
    FP32 = (False, False, False)

    def set_numerics(self, bf16_boundary: bool = True, bf16_products: bool = True, bf16_state: bool = True) -> None:
        """The c_impl contract (True, True, True) is the default; (True, False,
        False) exact products with FP32 state; (False, False, False) the FP32
        control."""
        check(self.lib.gdn_b200_set_numerics(ctypes.byref(self.s), int(bool(bf16_boundary)), int(bool(bf16_products)),
                                             int(bool(bf16_state))), "gdn_b200_set_numerics")

    def force_exact_products(self, on: bool = True) -> None:
        """Test hook: the exact emulation of the BF16 product in every phase."""
        check(self.lib.gdn_b200_test_force_exact_products(ctypes.byref(self.s), int(bool(on))),
              "gdn_b200_test_force_exact_products")

    def load_state(self, rec: np.ndarray, conv: np.ndarray) -> None:
        rec = np.ascontiguousarray(rec, dtype=np.float32)
        conv = np.ascontiguousarray(conv, dtype=np.float32)
        check(self.lib.gdn_b200_state_upload(ctypes.byref(self.s), _fptr(rec), rec.size, _fptr(conv), conv.size),
              "gdn_b200_state_upload")

    def read_state(self):
        rec = np.empty(self.rec_floats, dtype=np.float32)
        conv = np.empty(self.conv_floats, dtype=np.float32)
        check(self.lib.gdn_b200_state_download(ctypes.byref(self.s), _fptr(rec), rec.size, _fptr(conv), conv.size),
              "gdn_b200_state_download")
        return rec, conv

    def save_state(self, path: str, seed_token: int = 0) -> None:
        """gdn_b200_state_save_file: the state as a .gdnstate file."""
        check(self.lib.gdn_b200_state_save_file(ctypes.byref(self.s), os.fsencode(path), int(seed_token)),
              "gdn_b200_state_save_file")

    def load_state_file(self, path: str) -> int:
        """gdn_b200_state_load_file; returns the file's seed token."""
        tok = ctypes.c_int32()
        check(self.lib.gdn_b200_state_load_file(ctypes.byref(self.s), os.fsencode(path), ctypes.byref(tok)),
              "gdn_b200_state_load_file")
        return tok.value

    def read_state_part(self):
        """gdn_b200_tp_state_download_part: this rank's part of a
        tensor-parallel state and the attachment it came from, as
        (rec, conv, grid, rank, world) for tensor_parallel.merge_state."""
        rec = np.empty(self.rec_floats, dtype=np.float32)
        conv = np.empty(self.conv_floats, dtype=np.float32)
        g, r, w = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        check(self.lib.gdn_b200_tp_state_download_part(ctypes.byref(self.s), _fptr(rec), rec.size, _fptr(conv),
                                                       conv.size, ctypes.byref(g), ctypes.byref(r),
                                                       ctypes.byref(w)), "gdn_b200_tp_state_download_part")
        return rec, conv, g.value, r.value, w.value

    def tp_token(self) -> bytes:
        """gdn_b200_tp_token: what the peers of a tensor-parallel decode need to map this run state."""
        buf = ctypes.create_string_buffer(GDN_B200_TP_TOKEN_BYTES)
        check(self.lib.gdn_b200_tp_token(ctypes.byref(self.s), buf), "gdn_b200_tp_token")
        return buf.raw

    def tp_attach(self, rank: int, world: int, tokens: Sequence[bytes]) -> None:
        """gdn_b200_tp_attach with every rank's token, in rank order."""
        blob = b"".join(tokens)
        if len(tokens) != world or len(blob) != world * GDN_B200_TP_TOKEN_BYTES:
            raise ValueError("tp_attach: one token of GDN_B200_TP_TOKEN_BYTES per rank expected")
        check(self.lib.gdn_b200_tp_attach(ctypes.byref(self.s), int(rank), int(world), blob), "gdn_b200_tp_attach")

    def tp_detach(self) -> None:
        check(self.lib.gdn_b200_tp_detach(ctypes.byref(self.s)), "gdn_b200_tp_detach")

    def free(self) -> None:
        if self.s.workspace:
            self.lib.gdn_run_state_free(ctypes.byref(self.s))

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Batch:
    """Several decode streams of a Model advanced together (gdn_b200_batch_*):
    each step reads every weight byte once for all streams; projections on
    the tensor cores, FP32-boundary numerics."""

    def __init__(self, model: Model, streams: int):
        self.model = model
        self.lib = model.lib
        self.streams = int(streams)
        self.b = self.lib.gdn_b200_batch_create(ctypes.byref(model.m), self.streams)
        if not self.b:
            raise RuntimeError(f"gdn_b200_batch_create failed: {last_error()}")
        c = model.config
        self.rec_floats = c.num_layers * c.num_heads * c.head_dim * c.head_dim
        self.conv_floats = c.num_layers * 3 * (c.conv_size - 1) * c.hidden_size

    @property
    def launches_per_step(self) -> int:
        return int(self.lib.gdn_b200_batch_launches_per_step(self.b))

    def reset(self) -> None:
        check(self.lib.gdn_b200_batch_reset(self.b), "gdn_b200_batch_reset")

    def step(self, tokens: Sequence[int], with_logits: bool = False):
        """One step from host memory; returns argmax [streams] (and logits [streams, vocab])."""
        tok = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        assert tok.size == self.streams
        am = np.empty(self.streams, dtype=np.int32)
        lg = np.empty((self.streams, self.model.config.vocab_size), dtype=np.float32) if with_logits else None
        check(self.lib.gdn_b200_batch_step_host(self.b, tok.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                                am.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                                _fptr(lg) if lg is not None else None), "gdn_b200_batch_step_host")
        return (am, lg) if with_logits else am

    def decode(self, tokens: np.ndarray, greedy: bool = False):
        """tokens [n, streams] (greedy: row 0 only is read); returns (argmax [n, streams], device ms)."""
        tok = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        n = tok.shape[0]
        out = np.empty((n, self.streams), dtype=np.int32)
        ms = ctypes.c_float(0.0)
        check(self.lib.gdn_b200_batch_decode_tokens(self.b, tok.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), n,
                                                    int(greedy), out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                                    ctypes.byref(ms)), "gdn_b200_batch_decode_tokens")
        return out, float(ms.value)

    def logits(self) -> np.ndarray:
        lg = np.empty((self.streams, self.model.config.vocab_size), dtype=np.float32)
        check(self.lib.gdn_b200_batch_fetch_logits(self.b, _fptr(lg)), "gdn_b200_batch_fetch_logits")
        return lg

    def load_state(self, stream: int, rec: np.ndarray, conv: np.ndarray) -> None:
        rec = np.ascontiguousarray(rec, dtype=np.float32)
        conv = np.ascontiguousarray(conv, dtype=np.float32)
        check(self.lib.gdn_b200_batch_state_upload(self.b, int(stream), _fptr(rec), rec.size, _fptr(conv), conv.size),
              "gdn_b200_batch_state_upload")

    def read_state(self, stream: int):
        rec = np.empty(self.rec_floats, dtype=np.float32)
        conv = np.empty(self.conv_floats, dtype=np.float32)
        check(self.lib.gdn_b200_batch_state_download(self.b, int(stream), _fptr(rec), rec.size, _fptr(conv),
                                                     conv.size), "gdn_b200_batch_state_download")
        return rec, conv

    def free(self) -> None:
        if self.b:
            self.lib.gdn_b200_batch_free(self.b)
            self.b = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def tile_gemm(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    """gdn_b200_test_tile_gemm: y [n, m] = x [n, k] . w [m, k]^T through one
    tensor-core tile-GEMM launch (w BF16-exact float32)."""
    L = lib()
    w = np.ascontiguousarray(w, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = w.shape
    n = x.shape[0]
    y = np.empty((n, m), dtype=np.float32)
    check(L.gdn_b200_test_tile_gemm(m, k, n, _fptr(w), _fptr(x), _fptr(y)), "gdn_b200_test_tile_gemm")
    return y


def delta_rule_step(S: np.ndarray, q: np.ndarray, k: np.ndarray, v: np.ndarray, decay: np.ndarray,
                    beta: np.ndarray, steps: int = 1):
    """gdn_b200_delta_rule_step on host arrays: S [slices, 256, 256] (v, k),
    q/k/v [slices, 256], decay/beta [slices], all float32. Returns
    (S after `steps` steps, o of the last step, mean device ms per step)."""
    L = lib()
    S = np.ascontiguousarray(S, dtype=np.float32).copy()
    slices = S.shape[0]
    arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v, decay, beta)]
    o = np.empty((slices, 256), dtype=np.float32)
    ms = ctypes.c_float(0.0)
    check(L.gdn_b200_delta_rule_step(slices, _fptr(S), *[_fptr(a) for a in arrs], _fptr(o), int(steps),
                                     ctypes.byref(ms)), "gdn_b200_delta_rule_step")
    return S, o, float(ms.value)

