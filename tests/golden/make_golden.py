"""Generate tests/golden/reference_goldens.json from the REFERENCE itself.

Runs oracle/_ref/gdn_ref_driver -- the reference's c_impl/gdn_model.cpp
compiled natively through oracle/hls_shim by oracle/Makefile -- and digests
its outputs:

  primitives  the reference's BF16 RNE (gdn_test_fp32_to_bf16_rne_bits) and
              BF16 product (gdn_native_bf16_mul_to_fp32) over fixed input
              grids (oracle/ref_driver.cpp dump_primitives): SHA-256 of the
              outputs plus an explicit sample.
  layouts     the reference's host image helpers (oracle/ref_driver.cpp
              dump_layouts): SHA-256 of the 32 packed weight shards and the aux
              image of a small seeded model, of the four recurrent-state
              stripes of a seeded state and of the conv-tail packing.
  decode      gdn_decode_step_host on seeded GDN-1.3B weights
              (gateddeltanet_b200/csrc/gdn_synth.h) and seeded token streams:
              per step the input token, the kernel's argmax, SHA-256 of the
              FP32 logits and of the final hidden vector, the top-5 logits;
              after the run SHA-256 of the recurrent state and conv tails in
              the .gdnstate layouts.

tests/test_oracle_golden.py recomputes all of it with the CPU oracle and
requires bit equality. Needs the reference sources (only in the build
container): `make -C oracle ref && python tests/golden/make_golden.py`.

  --config0 [DUMP]   BASELINE config[0] as specified: 256 teacher-forced
              steps from zero state on the seeded GDN-1.3B weights (seed 1234,
              token stream seed 99, stream 0) through the reference's
              gdn_decode_step_host, digested into
              tests/golden/reference_config0_256.json (per step: token, argmax,
              SHA-256 of the FP32 logits and hidden vector, top-5; the final
              recurrent state and conv tails). The reference takes 7-14 s per
              token single-threaded (30-60 minutes); DUMP reuses a driver
              output written earlier with
              `gdn_ref_driver --seed 1234 --stream-seed 99 --stream 0 --steps 256 --out DUMP`.
"""
from __future__ import annotations

import hashlib
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
DRIVER = os.path.join(REPO, "oracle", "_ref", "gdn_ref_driver")
sys.path.insert(0, os.path.dirname(HERE))
import oracle_lib  # noqa: E402

DECODE_CASES = [
    dict(name="zero_state", seed=1234, stream_seed=99, stream=0, steps=4, state_seed=0),
    dict(name="seeded_state", seed=1234, stream_seed=99, stream=1, steps=3, state_seed=7),
]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def primitives(tmp: str) -> dict:
    path = os.path.join(tmp, "prims.bin")
    subprocess.run([DRIVER, "--primitives", path], check=True)
    data = open(path, "rb").read()
    assert data[:8] == b"GDNPRIM1"
    n_rne, n_prod = np.frombuffer(data[8:16], dtype=np.uint32)
    rne = np.frombuffer(data[16:16 + 2 * n_rne], dtype=np.uint16)
    prod = np.frombuffer(data[16 + 2 * n_rne:16 + 2 * n_rne + 4 * n_prod], dtype=np.uint32)
    idx_r = np.arange(0, len(rne), 4099)
    idx_p = np.arange(0, len(prod), 4099)
    return {
        "rne_set_a_sha256": sha(rne[:65536]),
        "rne_set_b_sha256": sha(rne[65536:]),
        "product_grid_sha256": sha(prod),
        "rne_sample": {"index": idx_r.tolist(), "bits": rne[idx_r].tolist()},
        "product_sample": {"index": idx_p.tolist(), "bits": prod[idx_p].tolist()},
    }


def layouts(tmp: str) -> dict:
    path = os.path.join(tmp, "layouts.bin")
    subprocess.run([DRIVER, "--layouts", path], check=True)
    data = open(path, "rb").read()
    assert data[:8] == b"GDNLAYT1"
    sb, na, stb, nh = (int(x) for x in np.frombuffer(data[8:40], dtype=np.uint64))
    off = 40
    parts = {}
    for name, n in (("shards", 32 * sb), ("aux", na), ("stripes", 4 * stb), ("conv_head", nh)):
        parts[name] = np.frombuffer(data, dtype=np.uint8, count=64 * n, offset=off)
        off += 64 * n
    shard = parts["shards"].reshape(32, -1)
    return {
        "model": dict(vocab=4096, hidden=512, layers=2, heads=2, head_dim=256, inter=1536, conv=4, seed=4321),
        "state_seed": 77, "conv_seed_full_dims": 78,
        "shard_beats": sb, "aux_beats": na, "stripe_beats": stb, "conv_head_beats": nh,
        "shard_sha256": [sha(shard[c]) for c in range(32)],
        "aux_sha256": sha(parts["aux"]),
        "stripes_sha256": sha(parts["stripes"]),
        "conv_head_sha256": sha(parts["conv_head"]),
    }


def decode_case(tmp: str, c: dict) -> dict:
    path = os.path.join(tmp, f"{c['name']}.bin")
    cmd = [DRIVER, "--seed", str(c["seed"]), "--stream-seed", str(c["stream_seed"]), "--stream", str(c["stream"]),
           "--steps", str(c["steps"]), "--out", path]
    if c["state_seed"]:
        cmd += ["--state-seed", str(c["state_seed"])]
    subprocess.run(cmd, check=True)
    steps, rest = oracle_lib.read_ref_dump(path)
    d = oracle_lib.FULL_DIMS
    nrec = d["layers"] * d["heads"] * d["head_dim"] * d["head_dim"]
    rec, conv = rest[:nrec], rest[nrec:]
    out = dict(c)
    out["steps_out"] = []
    for s in steps:
        top = np.argsort(-s["logits"], kind="stable")[:5]
        out["steps_out"].append({
            "token": s["token"], "argmax": s["argmax"],
            "logits_sha256": sha(s["logits"]), "hidden_sha256": sha(s["hidden"]),
            "top5_index": top.tolist(), "top5_value": [float(s["logits"][i]) for i in top],
            "reference_ms": s["ms"],
        })
    out["rec_sha256"] = sha(rec)
    out["conv_sha256"] = sha(conv)
    out["rec_sample"] = [float(x) for x in rec[:: len(rec) // 16][:16]]
    return out


CONFIG0 = dict(name="config0_256", seed=1234, stream_seed=99, stream=0, steps=256, state_seed=0)


def digest_dump(c: dict, path: str) -> dict:
    steps, rest = oracle_lib.read_ref_dump(path)
    assert len(steps) == c["steps"], f"dump has {len(steps)} steps, expected {c['steps']}"
    d = oracle_lib.FULL_DIMS
    nrec = d["layers"] * d["heads"] * d["head_dim"] * d["head_dim"]
    rec, conv = rest[:nrec], rest[nrec:]
    out = dict(c)
    out["steps_out"] = []
    for s in steps:
        top = np.argsort(-s["logits"], kind="stable")[:5]
        out["steps_out"].append({
            "token": s["token"], "argmax": s["argmax"],
            "logits_sha256": sha(s["logits"]), "hidden_sha256": sha(s["hidden"]),
            "top5_index": top.tolist(), "top5_value": [float(s["logits"][i]) for i in top],
        })
    out["mean_reference_ms"] = float(np.mean([s["ms"] for s in steps]))
    out["rec_sha256"] = sha(rec)
    out["conv_sha256"] = sha(conv)
    return out


def config0(dump: str | None) -> None:
    with tempfile.TemporaryDirectory() as tmp:
        if dump is None:
            dump = os.path.join(tmp, "config0.bin")
            subprocess.run([DRIVER, "--seed", str(CONFIG0["seed"]), "--stream-seed", str(CONFIG0["stream_seed"]),
                            "--stream", str(CONFIG0["stream"]), "--steps", str(CONFIG0["steps"]), "--out", dump],
                           check=True)
        gold = digest_dump(CONFIG0, dump)
    gold["generator"] = ("tests/golden/make_golden.py --config0 via oracle/_ref/gdn_ref_driver (reference "
                         "c_impl/gdn_model.cpp compiled natively through oracle/hls_shim)")
    path = os.path.join(HERE, "reference_config0_256.json")
    with open(path, "w") as f:
        json.dump(gold, f, indent=0)
    print("wrote", path)


def main() -> None:
    if len(sys.argv) > 1 and sys.argv[1] == "--config0":
        config0(sys.argv[2] if len(sys.argv) > 2 else None)
        return
    if not os.path.exists(DRIVER):
        raise SystemExit("build the reference first: make -C oracle ref")
    with tempfile.TemporaryDirectory() as tmp:
        gold = {
            "generator": "tests/golden/make_golden.py via oracle/_ref/gdn_ref_driver "
                         "(reference c_impl/gdn_model.cpp compiled natively through oracle/hls_shim)",
            "primitives": primitives(tmp),
            "layouts": layouts(tmp),
            "decode": [decode_case(tmp, c) for c in DECODE_CASES],
        }
    with open(os.path.join(HERE, "reference_goldens.json"), "w") as f:
        json.dump(gold, f, indent=1)
    print("wrote", os.path.join(HERE, "reference_goldens.json"))


if __name__ == "__main__":
    main()
