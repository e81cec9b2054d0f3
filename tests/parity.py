"""Parity metrics shared by the GPU tests (test infrastructure).

Tolerances are the north-star gates: logits relative-L2 1e-2 with BF16
boundaries and 1e-4 in the FP32 control; recurrent state relative-L2 1e-3;
argmax identical wherever the oracle's top-2 margin exceeds the observed
logit error (4x max |delta|).
"""
import numpy as np

LOGITS_BF16 = 1e-2
LOGITS_FP32 = 1e-4
STATE = 1e-3


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def argmax_first(x) -> int:
    """Maximum value, lowest index on ties (the reference's rule)."""
    return int(np.argmax(x))


def argmax_agrees(engine_logits, oracle_logits, engine_token) -> bool:
    """True unless the oracle's top-2 margin exceeds 4x the logit error and
    the engine picked a different token."""
    o = np.asarray(oracle_logits, dtype=np.float64)
    e = np.asarray(engine_logits, dtype=np.float64)
    top2 = np.partition(o, -2)[-2:]
    margin = float(top2[1] - top2[0])
    err = float(np.max(np.abs(e - o)))
    if margin <= 4.0 * err:
        return True
    return int(engine_token) == argmax_first(o)
