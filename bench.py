#!/usr/bin/env python3
"""Benchmark: GDN-1.3B batch-1 decode on B200 (BASELINE config[2] workload).

One step = one decoded token of one batch-1 stream of GatedDeltaNet-1.3B
(seeded synthetic BF16 weights, seeded uniform token stream). Per rank: a
seeded prompt (default 4096 tokens) builds the recurrent state, W warm-up
tokens, then exactly K timed tokens of the cyclic teacher-forced stream.

  value    tokens/s of the whole job with inputs resident in HBM: the
           device-resident decode loop (gdn_b200_decode_tokens), timed with
           CUDA events on the engine's stream, max over ranks. Weights
           (2.8 GB/token) exceed L2, so no flush is needed between steps.
  e2e      the same metric through the reference-facing C ABI,
           gdn_decode_step_host per token: the token id as a kernel argument
           (the kernel gathers its embedding row), the 128-byte status block
           with the token line read back, host wall clock.
  roofline algorithmic bytes per token / measured time per token against
           MEASURED_PEAKS.json hbm_gbs.
  cpu_baseline  the CPU oracle port (multi-threaded restatement of the
           reference arithmetic) on a bounded sample, rank 0 at N=1.

N > 1 (torchrun): one process per GPU, each decoding its own stream with no
collective (weak scaling); value = N * K / max-over-ranks time. Beside it
the line carries `tp` (one stream decoded by all N GPUs
together, its speed-up over one GPU and a bit-equality check against a
one-GPU decode of the same tokens) and, at every N, `streams` (config[3]:
64 streams per GPU, and 64 in total at N > 1, through gdn_b200_batch_*).

--impl reference: the reference's own CPU decode (c_impl/gdn_model.cpp built
natively by oracle/Makefile into oracle/_ref/gdn_ref_driver) timed on the host
cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "GDN-1.3B batch-1 decode ms/token (inner+outer) & % HBM roofline; streams tok/s"
WORKLOAD_TEXT = ("BASELINE config[2]: GDN-1.3B batch-1 sustained decode, seeded BF16 weights, seeded prompt then a "
                 "cyclic seeded 4096-token teacher stream")
FPGA_INNER_MS = 8.141  # the reference's published kernel ms/token on its Alveo U55C (c_impl/doc/architecture.md:37)
from gateddeltanet_b200.workload import (PROMPT_OFFSET, SEED, SHAPE, STREAM_SEED, job_tokens_per_s,  # noqa: E402
                                         max_over_ranks, rank_streams, token_stream)


NUMERICS = {  # gdn_b200_set_numerics contracts
    "cimpl": (True, True, True),    # the reference's own arithmetic (default; BF16 state)
    "engine": (True, False, False),  # exact products, FP32 state
    "fp32": (False, False, False),   # the FP32 control
}
KERNEL_MODE = {"cimpl": 11, "engine": 1, "fp32": 0}


def state_bytes_per_value(numerics: str) -> int:
    return 2 if NUMERICS[numerics][2] else 4


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def algorithmic_bytes_per_token(s=SHAPE, numerics: str = "cimpl") -> int:
    """Per-token HBM bytes at batch 1 (weights read once, state read+written
    once, in the contract's storage: BF16 for c_impl, FP32 otherwise)."""
    H, I, V, L, nh = s["hidden"], s["inter"], s["vocab"], s["layers"], s["heads"]
    gemv = 2 * (L * (4 * H * H + 2 * nh * H + H * H + 2 * I * H + I * H) + V * H)
    aux = 4 * (L * (H + 256 + H + 12 * H + 2 * nh) + H)
    state = 2 * L * nh * 256 * 256 * state_bytes_per_value(numerics)
    tails = L * 3 * H * 16 * 2
    io = 2 * H + 4 * V + 4
    return gemv + aux + state + tails + io


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_from_profiles():
    """DRAM bytes per launch of the decode kernel from the committed ncu summary."""
    path = os.path.join(REPO, "profiles", "gdn_decode_kernel_full_1p3b.md")
    try:
        for line in open(path):
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.samples.append(parts)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def energy_meter(device: int):
    """NVML meter of this rank's GPU and its loaded-idle power (1 s), or (None, None)."""
    try:
        from gateddeltanet_b200.energy import EnergyMeter
        m = EnergyMeter(device)
        return m, m.idle_watts(1.0)
    except Exception:
        return None, None


def energy_line(window, tokens: int, idle_w):
    """Energy of the timed window of this rank's GPU (gateddeltanet_b200/energy.py)."""
    if window is None:
        return {"unavailable": "NVML energy queries not available"}
    from gateddeltanet_b200.energy import summarize
    out = summarize(window, tokens, idle_w)
    out["scope"] = "rank 0's GPU over the timed decode window (host and server power not included)"
    return out


def cpu_baseline_port(n_tokens: int = 3):
    """Oracle port (reference arithmetic) on all host cores, bounded sample."""
    sys.path.insert(0, os.path.join(REPO, "tests"))
    import oracle_lib as ol
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    o = ol.Oracle(ol.FULL_DIMS, seed=SEED, threads=threads)
    setup = time.perf_counter() - t0
    times = []
    for i in range(n_tokens):
        t = time.perf_counter()
        o.step(o.token(STREAM_SEED, 0, i), ol.REFERENCE_MODE)
        times.append(time.perf_counter() - t)
    ms = statistics.median(times) * 1000.0
    return {"value": round(1000.0 / ms, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
            "cpu_model": cpu_model(),
            "sample": f"{n_tokens} GDN-1.3B decode tokens (oracle/gdn_oracle.c, reference arithmetic: BF16 products, "
                      f"BF16 state), median {ms:.1f} ms/token, weight synthesis {setup:.1f} s untimed"}


def run_reference(args):
    """--impl reference: the reference's own native decode on the host CPU."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    driver = os.path.join(REPO, "oracle", "_ref", "gdn_ref_driver")
    if not os.path.exists(driver):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/gdn_ref_driver was not built "
                          "(the reference sources are needed to build it)"}))
        return 0
    warm = min(args.warmup, 1)
    out = subprocess.run([driver, "--seed", str(SEED), "--stream-seed", str(STREAM_SEED), "--warmup", str(warm),
                          "--steps", str(args.steps)],
                         capture_output=True, text=True, check=True)
    res = json.loads(out.stdout.strip().splitlines()[-1])
    ms = float(res["mean_ms_per_token"])
    tps = 1000.0 / ms
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tps, 5), "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": int(res["steps"]), "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD_TEXT,
                   "batch_per_gpu": 1, "numerics": "cimpl (the reference's own arithmetic)",
                   "note": "the reference's per-token CPU cost does not depend on the recurrent state, so its "
                           "stream starts from zero state instead of the prefilled prompt state"},
        "cpu_baseline": {"value": round(tps, 5), "unit": "tokens/s", "cores": 1, "kind": "reference",
                         "cpu_model": cpu_model(),
                         "sample": f"{res['steps']} timed tokens after {warm} warm-up (reference gdn_decode_step_host, "
                                   f"native build, single-threaded monolith)"},
        "e2e": {"value": round(tps, 5), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def run_delta_rule(args):
    """--workload delta_rule: BASELINE config[1], the gated delta rule alone on
    24 x 8 FP32 256x256 states (inputs as in tests/test_gpu_delta_rule.py),
    L2 flushed before every step; value = state GB/s of one step."""
    import numpy as np
    import gateddeltanet_b200 as gdn
    from gateddeltanet_b200 import build
    build.build()
    L = gdn.lib()
    gdn.check(L.gdn_b200_set_device(int(os.environ.get("LOCAL_RANK", "0"))), "gdn_b200_set_device")
    slices = SHAPE["layers"] * SHAPE["heads"]
    rng = np.random.default_rng(SEED)
    S = rng.normal(0, 0.1, (slices, 256, 256)).astype(np.float32)
    q = rng.normal(0, 1, (slices, 256)).astype(np.float32)
    k = rng.normal(0, 1, (slices, 256)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    k /= np.linalg.norm(k, axis=1, keepdims=True)
    v = rng.normal(0, 1, (slices, 256)).astype(np.float32)
    decay = np.exp(-np.log1p(np.exp(rng.normal(-4, 1, slices)))).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.normal(0, 1, slices)))).astype(np.float32)
    gdn.delta_rule_step(S, q, k, v, decay, beta, steps=max(args.warmup, 1))
    _, _, ms = gdn.delta_rule_step(S, q, k, v, decay, beta, steps=args.steps)
    state_bytes = 2 * slices * 256 * 256 * 4
    io_bytes = slices * (3 * 256 * 4 + 256 * 4 + 8)
    gbs = (state_bytes + io_bytes) / (ms / 1000.0) / 1e9
    peak, peak_kind = peaks()
    print(json.dumps({
        "metric": "gated delta-rule step: state GB/s (BASELINE config[1])", "value": round(gbs, 1), "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "BASELINE config[1]: 24 layers x 8 heads, S 256x256 fp32 N(0,0.1), q/k/v N(0,1) "
                               "with q,k L2-normalised, decay=exp(-softplus(N(-4,1))), beta=sigmoid(N(0,1))",
                   "l2": "flushed (256 MB write) before every step"},
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": state_bytes + io_bytes, "kernel": "delta_rule_kernel"},
        "gpu_launches": args.steps}))
    return 0


def step_bytes_streams(b: int, s=SHAPE) -> int:
    """HBM bytes of one multi-stream step: every weight byte once, plus per
    stream its FP32 state read and written, conv tails, embedding row, logits."""
    H, I, V, L, nh = s["hidden"], s["inter"], s["vocab"], s["layers"], s["heads"]
    weights = 2 * (L * (4 * H * H + 2 * nh * H + H * H + 2 * I * H + I * H) + V * H)
    aux = 4 * (L * (H + 256 + H + 12 * H + 2 * nh) + H)
    per_stream = 2 * L * nh * 256 * 256 * 4 + 2 * L * 9 * H * 4 + 2 * H + 4 * V + 4
    return weights + aux + b * per_stream


def run_prefill(args):
    """--workload prefill: the config[2] prompt (--prompt seeded tokens) through
    gdn_b200_prefill on a fresh run state; value = prompt tokens per second of
    device time (median of --steps runs after --warmup)."""
    import gateddeltanet_b200 as gdn
    from gateddeltanet_b200 import build
    build.build()
    L = gdn.lib()
    gdn.check(L.gdn_b200_set_device(int(os.environ.get("LOCAL_RANK", "0"))), "gdn_b200_set_device")
    model = gdn.Model(header=gdn.make_header(**SHAPE), seed=SEED)
    rs = gdn.RunState(model)
    prompt = token_stream(0, args.prompt, SHAPE["vocab"], offset=PROMPT_OFFSET)
    for _ in range(max(args.warmup, 1)):
        rs.prefill(prompt)
    times = [rs.prefill(prompt) for _ in range(max(args.steps, 1))]
    ms = statistics.median(times)
    print(json.dumps({
        "metric": "GDN-1.3B prompt prefill tokens/s", "value": round(args.prompt / (ms / 1000.0), 1),
        "unit": "tokens/s", "n_gpus": 1, "steps": len(times), "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"BASELINE config[2] prompt: {args.prompt} seeded uniform tokens into a zero state "
                               "(gdn_b200_prefill: tensor-core projections over up to 240 tokens, recurrence in "
                               "token order, FP32)"},
        }))
    rs.free()
    model.free()
    return 0


def run_streams(args):
    """--workload streams: BASELINE config[3], B independent streams from zero
    state, sharded over the ranks (B / N per GPU, no collective); one step
    advances every stream by one token (gdn_b200_batch_*)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=120))
    if args.streams % world:
        raise SystemExit("--streams must be a multiple of the GPU count")
    per_rank = args.streams // world

    import gateddeltanet_b200 as gdn
    from gateddeltanet_b200 import build
    build.build()
    L = gdn.lib()
    gdn.check(L.gdn_b200_set_device(local), "gdn_b200_set_device")

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    shape = dict(SHAPE, layers=args.layers)
    model = gdn.Model(header=gdn.make_header(**shape), seed=SEED)
    batch = gdn.Batch(model, per_rank)
    V = SHAPE["vocab"]
    ids = rank_streams(rank, world, per_rank)
    n_all = args.warmup + args.steps + args.e2e_steps
    toks = np.array([token_stream(i, n_all, V) for i in ids], dtype=np.int32).T.copy()  # [n_all, per_rank]
    if args.warmup:
        batch.decode(toks[:args.warmup])
    meter, idle_w = energy_meter(local)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier()
    if meter is not None:
        meter.start()
    _, dev_ms = batch.decode(toks[args.warmup:args.warmup + args.steps])
    window = meter.stop() if meter is not None else None
    barrier()
    dev_ms = max_over_ranks(dev_ms, device="cuda")
    # e2e: host tokens in, argmax out, every step through gdn_b200_batch_step_host
    e2e_n = max(1, min(args.e2e_steps, args.steps))
    barrier()
    t0 = time.perf_counter()
    for i in range(e2e_n):
        batch.step(toks[args.warmup + args.steps + i % max(args.e2e_steps, 1)])
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0, device="cuda")
    barrier()
    sampler.stop()
    launches = batch.launches_per_step
    ms_step = dev_ms / args.steps
    value = args.streams * args.steps / (dev_ms / 1000.0)
    e2e_value = args.streams * e2e_n / e2e_s
    alg = step_bytes_streams(per_rank, shape)
    peak, peak_kind = peaks()
    achieved = alg / (ms_step / 1000.0) / 1e9
    line = {
        "metric": "GDN-1.3B multi-stream decode tokens/s (BASELINE config[3])", "value": round(value, 1),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"BASELINE config[3]: {args.streams} independent GDN-1.3B streams from zero fp32 "
                               "state, seeded uniform teacher-forced tokens per stream, sharded over the GPUs",
                   "streams": args.streams, "streams_per_gpu": per_rank, "layers": args.layers,
                   "state": "fp32", "boundaries": "fp32",
                   "projections": "tcgen05 tile GEMM, activations as three BF16 terms, FP32 accumulation",
                   "l2": "no flush: 2.8 GB of weights plus the streams' state per step exceed the 126 MB L2",
                   "parallelism": f"stream-dp{world}"},
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 4 * per_rank,
                "d2h_bytes_per_step": 4 * per_rank + 8,
                "api": "gdn_b200_batch_step_host (C ABI), synchronous per step"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": alg,
                     "kernel": f"whole step ({launches} launches: tile GEMMs, recurrence, norms; one CUDA graph)"},
        "gpu_launches": launches * args.steps,
        "clocks": sampler.summary(),
        "energy": energy_line(window, per_rank * args.steps, idle_w),
    }
    batch.free()
    model.free()
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


def sustained_window(rs, teacher, start, seconds, device, idle_w, barrier):
    """Decode the cyclic teacher stream for >= `seconds` of device time in
    4096-token device-resident calls (inner ms/token, clocks and NVML energy
    over that window), then for about as long through gdn_decode_step_host
    with host buffers (outer ms/token)."""
    meter, _ = energy_meter(device)
    sampler = ClockSampler(device)
    sampler.start()
    time.sleep(0.3)
    barrier()
    if meter is not None:
        meter.start()
    dev_ms, tokens, pos = 0.0, 0, start
    t0 = time.perf_counter()
    while dev_ms < seconds * 1000.0:
        chunk = [teacher[(pos + i) % 4096] for i in range(4096)]
        _, ms = rs.decode(chunk)
        dev_ms += ms
        tokens += len(chunk)
        pos += len(chunk)
    wall = time.perf_counter() - t0
    win = meter.stop() if meter is not None else None
    barrier()
    sampler.stop()
    out_n, t1 = 0, time.perf_counter()
    while time.perf_counter() - t1 < min(seconds, 20.0):
        for _ in range(256):
            rs.step(teacher[(pos + out_n) % 4096])
            out_n += 1
    outer_s = time.perf_counter() - t1
    return {"tokens": tokens, "device_s": round(dev_ms / 1000.0, 3), "wall_s": round(wall, 3),
            "inner_ms_per_token": round(dev_ms / tokens, 5),
            "outer_tokens": out_n, "outer_ms_per_token": round(outer_s * 1000.0 / out_n, 5),
            "clocks": sampler.summary(), "energy": energy_line(win, tokens, idle_w),
            "note": "after the main timed tokens; inner = device-resident loop (CUDA events), outer = "
                    "gdn_decode_step_host per token with host buffers (wall clock)"}


def contract_timing(model, teacher, numerics, steps, warmup):
    """ms/token and roofline of another numeric contract on its own run state
    (zero state; up to 64 warm-up and 1024 timed tokens, no more than the
    headline's own)."""
    import gateddeltanet_b200 as gdn
    n_w, n = min(warmup, 64), max(1, min(steps, 1024))
    rs = gdn.RunState(model)
    rs.set_numerics(*NUMERICS[numerics])
    if n_w:
        rs.decode([teacher[i] for i in range(n_w)])
    _, ms = rs.decode([teacher[(n_w + i) % 4096] for i in range(n)])
    rs.free()
    ms_tok = ms / n
    alg = algorithmic_bytes_per_token(numerics=numerics)
    peak, peak_kind = peaks()
    return {"numerics": numerics, "ms_per_token": round(ms_tok, 5), "tokens_per_s": round(1000.0 / ms_tok, 2),
            "roofline": {"achieved": round(alg / (ms_tok / 1000.0) / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(alg / (ms_tok / 1000.0) / 1e9 / peak, 4), "algorithmic_bytes_per_launch": alg,
                         "kernel": f"gdn_decode_kernel<{KERNEL_MODE[numerics]}>"}}


def tp_record(model, teacher, args, world, rank, barrier):
    """BASELINE config[4] beside the stream-DP line at N > 1: one stream (the
    seeded teacher stream from zero state) decoded by all N GPUs together
    (gdn_b200_tp_attach; the kernel's row and column partitions over every
    GPU's CTAs, peer stores over NVLink, no NCCL call on the data path),
    max-over-ranks device time. Rank 0 then decodes the same tokens on one
    GPU: tokens and final logits must be bit-identical on every rank, and so
    must each rank's owned part of the recurrent state and conv tails."""
    import hashlib
    import torch.distributed as dist
    import gateddeltanet_b200 as gdn
    from gateddeltanet_b200 import tensor_parallel as tp
    from gateddeltanet_b200.workload import max_over_ranks
    n_w, n = min(args.warmup, 64), min(args.steps, 1024)
    toks = [teacher[i % 4096] for i in range(n_w + n)]
    dims = dict(SHAPE)
    rs = gdn.RunState(model)
    rs.set_numerics(*NUMERICS[args.numerics])
    tp.attach(rs)
    rs.decode(toks[:n_w])
    barrier()
    picks, ms = rs.decode(toks[n_w:])
    barrier()
    ms = max_over_ranks(ms, device="cuda")
    logits, _ = rs.outputs()
    rec, conv, grid, _, _ = rs.read_state_part()
    # one traced step on every rank at once (after the checked values are read)
    phases = phase_medians(rs.trace(toks[0]), dims["layers"])
    rs.tp_detach()
    barrier()
    rs.free()
    mine = (hashlib.sha256(tp.owned_values(rec, conv, dims, grid, rank, world)).hexdigest(),
            hashlib.sha256(picks.tobytes()).hexdigest(), hashlib.sha256(logits.tobytes()).hexdigest())
    seen = [None] * world
    dist.all_gather_object(seen, mine)
    rec_d = None
    if rank == 0:
        ref = gdn.RunState(model)
        ref.set_numerics(*NUMERICS[args.numerics])
        ref.decode(toks[:n_w])
        r_picks, r_ms = ref.decode(toks[n_w:])
        r_logits, _ = ref.outputs()
        r_rec, r_conv = ref.read_state()
        ref.free()
        want = [(hashlib.sha256(tp.owned_values(r_rec, r_conv, dims, grid, r, world)).hexdigest(),
                 hashlib.sha256(r_picks.tobytes()).hexdigest(), hashlib.sha256(r_logits.tobytes()).hexdigest())
                for r in range(world)]
        rec_d = {"gpus": world, "grid_per_gpu": grid, "steps": n, "warmup": n_w,
                 "ms_per_token": round(ms / n, 5), "tokens_per_s": round(1000.0 * n / ms, 2),
                 "one_gpu_ms_per_token": round(r_ms / n, 5), "speedup_vs_one_gpu": round(r_ms / ms, 3),
                 "bit_identical_to_one_gpu": seen == want,
                 "checked": "every rank's tokens, final logits and owned state part vs a one-GPU decode of the same "
                            "tokens (SHA-256)",
                 "numerics": args.numerics,
                 "workload": "BASELINE config[4]: one GDN-1.3B stream over all GPUs from zero state, seeded "
                             "teacher-forced tokens",
                 "exchange": "row-split partitions over all GPUs' CTAs; every output stored into every GPU's "
                             "exchange region by peer stores over NVLink (no NCCL call on the data path)",
                 "timing": "CUDA events on each rank's stream, max over ranks",
                 "phases_us": phases,
                 "phases_note": "one traced step after the timed ones, %globaltimer stamps: medians over rank 0's "
                                "CTAs and layers 1..L-2 of [arrive, input built, chunk work, total] per phase "
                                "(A QKVG, B state, C O, D gate/up, E down; LM head)"}
    barrier()
    return rec_d


def phase_medians(tr, layers: int) -> dict:
    """Per-phase medians, us, of a gdn_b200_trace_step stamp array [cta,
    phase, slot] over the CTAs that ran and layers 1..layers-2: slot 1 - 0
    (inputs arrived), 2 - 1 (input built), 3 - 2 (chunk work), 3 - 0."""
    import numpy as np
    tr = tr.astype(np.int64)
    tr = tr[tr[:, 0, 3] != 0]
    out = {}

    def med(t):
        return [round(float(np.median(t[..., a] - t[..., b])) / 1e3, 2) for a, b in ((1, 0), (2, 1), (3, 2), (3, 0))]
    for k, name in enumerate("ABCDE"):
        out[name] = med(tr[:, [l * 5 + k for l in range(1, layers - 1)], :])
    out["LM"] = med(tr[:, layers * 5, :])
    return out


def streams_record(model, args, world, rank, barrier, per_gpu: int = 64, steps: int = 32, warmup: int = 4):
    """BASELINE config[3] beside the batch-1 line: independent streams from
    zero state advanced together (gdn_b200_batch_*, tcgen05 projections),
    sharded over the ranks with no collective. weak: `per_gpu` streams on
    every GPU; strong: `per_gpu` streams in total (split over the GPUs)."""
    import numpy as np
    import gateddeltanet_b200 as gdn
    from gateddeltanet_b200.workload import max_over_ranks
    out = {}
    peak, peak_kind = peaks()
    for kind, total in (("weak", per_gpu * world), ("strong", per_gpu)):
        if (kind == "strong" and world == 1) or total % world:
            continue
        per = total // world
        batch = gdn.Batch(model, per)
        ids = rank_streams(rank, world, per)
        toks = np.array([token_stream(i, warmup + steps, SHAPE["vocab"]) for i in ids], dtype=np.int32).T.copy()
        batch.decode(toks[:warmup])
        barrier()
        _, ms = batch.decode(toks[warmup:])
        barrier()
        ms = max_over_ranks(ms, device="cuda")
        launches = batch.launches_per_step
        batch.free()
        alg = step_bytes_streams(per)
        out[kind] = {"streams": total, "streams_per_gpu": per, "steps": steps, "warmup": warmup,
                     "ms_per_step": round(ms / steps, 5), "tokens_per_s": round(total * steps / (ms / 1000.0), 1),
                     "roofline_frac": round(alg / (ms / steps / 1000.0) / 1e9 / peak, 4),
                     "algorithmic_bytes_per_gpu_step": alg, "launches_per_step": launches}
    out["config"] = ("BASELINE config[3]: independent GDN-1.3B streams from zero fp32 state, seeded teacher-forced "
                     "tokens per stream, FP32-boundary numerics, tcgen05 tile GEMMs; one CUDA graph per step; "
                     f"CUDA events, max over ranks; peak {peak_kind}")
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2048)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=4096)
    ap.add_argument("--e2e-steps", type=int, default=256)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--numerics", default="cimpl", choices=sorted(NUMERICS),
                    help="numeric contract of the timed decode: cimpl (default, the reference's own arithmetic, "
                         "bit-exact), engine (exact products, FP32 state), fp32 (the FP32 control)")
    ap.add_argument("--sustain-s", type=float, default=20.0,
                    help="length of the sustained window (config[2], energy per token); 0 skips it")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="leave out the tp (N > 1) and streams sub-records beside the headline")
    ap.add_argument("--workload", default="decode", choices=["decode", "delta_rule", "streams", "prefill", "tp"],
                    help="decode: the headline batch-1 decode (default); delta_rule: BASELINE config[1]; "
                         "streams: BASELINE config[3] multi-stream decode; tp: BASELINE config[4], one stream "
                         "decoded by all --gpus GPUs together (tensor-parallel)")
    ap.add_argument("--streams", type=int, default=64, help="total streams of --workload streams")
    ap.add_argument("--layers", type=int, default=SHAPE["layers"],
                    help="--workload streams only: fewer layers for a small profiling case (same per-layer shapes)")
    args = ap.parse_args()
    if args.workload == "delta_rule" and args.impl == "b200":
        return run_delta_rule(args)
    if args.workload == "streams" and args.impl == "b200":
        return run_streams(args)
    if args.workload == "prefill" and args.impl == "b200":
        return run_prefill(args)
    if args.impl == "reference":
        return run_reference(args)
    tp_mode = args.workload == "tp"

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=120))

    import gateddeltanet_b200 as gdn
    from gateddeltanet_b200 import build
    build.build()
    L = gdn.lib()
    gdn.check(L.gdn_b200_set_device(local), "gdn_b200_set_device")

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    model = gdn.Model(header=gdn.make_header(**SHAPE), seed=SEED)
    rs = gdn.RunState(model)
    rs.set_numerics(*NUMERICS[args.numerics])
    # token streams: each rank decodes its own independent stream (stream-DP),
    # or every rank the same one (tensor-parallel)
    stream = 0 if tp_mode else rank_streams(rank, world)[0]
    V = SHAPE["vocab"]
    prompt = token_stream(stream, args.prompt, V, offset=PROMPT_OFFSET)
    teacher = token_stream(stream, 4096, V)
    prompt_ms = rs.prefill(prompt) if args.prompt else 0.0
    if tp_mode and world > 1:
        from gateddeltanet_b200 import tensor_parallel
        tensor_parallel.attach(rs)
    n_w = args.warmup
    rs.decode([teacher[i % 4096] for i in range(n_w)]) if n_w else None
    timed = [teacher[(n_w + i) % 4096] for i in range(args.steps)]

    meter, idle_w = energy_meter(local)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier()
    if meter is not None:
        meter.start()
    picks, kernel_ms = rs.decode(timed)
    window = meter.stop() if meter is not None else None
    barrier()
    kernel_ms = max_over_ranks(kernel_ms, device="cuda")

    # e2e through the C ABI (gdn_decode_step_host), host buffers; one untimed
    # call first (the host path's own warm-up)
    e2e_n = min(args.e2e_steps, max(args.steps, 1))
    rs.step(teacher[(n_w + args.steps + e2e_n) % 4096])
    barrier()
    t0 = time.perf_counter()
    for i in range(e2e_n):
        rs.step(teacher[(n_w + args.steps + i) % 4096])
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0, device="cuda")
    barrier()
    sampler.stop()

    # sustained window (config[2]): >= --sustain-s of device-resident decode of
    # the cyclic teacher stream, then as long through gdn_decode_step_host,
    # with NVML energy and clocks over the inner window
    sustained = None
    if args.sustain_s > 0 and not tp_mode:
        sustained = sustained_window(rs, teacher, n_w + args.steps, args.sustain_s, local, idle_w, barrier)
    # the other contract beside the headline one: a short timing of the
    # engine contract (exact products, FP32 state) on its own run state
    other = None
    if not tp_mode and args.numerics == "cimpl":
        other = contract_timing(model, teacher, "engine", args.steps, args.warmup)
    ms_per_tok = kernel_ms / args.steps
    streams_in_job = 1 if tp_mode else world
    value = job_tokens_per_s(streams_in_job, args.steps, kernel_ms / 1000.0)
    e2e_ms = e2e_s * 1000.0 / e2e_n
    e2e_value = job_tokens_per_s(streams_in_job, e2e_n, e2e_s)
    alg = algorithmic_bytes_per_token(numerics=args.numerics)
    peak, peak_kind = peaks()
    achieved = alg / (ms_per_tok / 1000.0) / 1e9
    if tp_mode:
        # one stream's bytes over the job's GPUs: against the sum of their peaks
        peak = peak * world
        peak_kind = f"{peak_kind} x {world} GPUs"
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_tok, 5), "higher_is_better": True,
        "scaling": "strong" if tp_mode else "weak",
        "vs_baseline": round(value / streams_in_job / (1000.0 / FPGA_INNER_MS), 3),
        "vs_baseline_ref": f"per-GPU tokens/s vs the reference-published FPGA inner {FPGA_INNER_MS} ms/token",
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": ("BASELINE config[4]: GDN-1.3B batch-1 decode of one stream over all GPUs "
                                "(tensor-parallel), " if tp_mode else
                                "BASELINE config[2]: GDN-1.3B batch-1 sustained decode, ") +
                               "seeded BF16 weights, "
                               f"{args.prompt}-token seeded prompt then a cyclic seeded 4096-token teacher stream" +
                               ("" if tp_mode else "; one independent stream per GPU"),
                   "batch_per_gpu": 1, "numerics": args.numerics,
                   "state": "bf16" if NUMERICS[args.numerics][2] else "fp32",
                   "boundaries": "bf16" if NUMERICS[args.numerics][0] else "fp32",
                   "products": "bf16-rounded (reference)" if NUMERICS[args.numerics][1] else "exact",
                   "l2": "no flush: 2.8 GB of weights per step exceed the 126 MB L2",
                   "prompt_build": f"gdn_b200_prefill, {prompt_ms:.1f} ms device time (untimed)",
                   "parallelism": f"tp{world}" if tp_mode else f"stream-dp{world}"},
        "inner_ms_per_token": round(ms_per_tok, 5),
        "outer_ms_per_token": round(e2e_ms, 5),
        "e2e": {"value": round(e2e_value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 128,
                "api": "gdn_decode_step_host (C ABI), synchronous per token: the token id travels as a kernel "
                       "argument, the 128-byte status block (token line + error word) comes back"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic_from_profiles(),
                     "peak_kind": peak_kind, "algorithmic_bytes_per_launch": alg,
                     "kernel": (f"gdn_decode_kernel<{KERNEL_MODE[args.numerics] + 4}> (tensor-parallel, {args.numerics} "
                                "contract; one launch per token per GPU)" if tp_mode and world > 1 else
                                f"gdn_decode_kernel<{KERNEL_MODE[args.numerics]}> ({args.numerics} contract; one "
                                "launch per token)")},
        "gpu_launches": args.steps,
        "clocks": sampler.summary(),
        "energy": energy_line(window, args.steps, idle_w),
        **({"sustained": sustained} if sustained is not None else {}),
        **({"other_contract": other} if other is not None else {}),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = cpu_baseline_port()
        except Exception as e:  # the baseline is reported, never the target
            line["cpu_baseline"] = {"value": None, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                                    "sample": f"failed: {e}"}
    if tp_mode and world > 1:
        rs.tp_detach()  # every rank unmaps its peers before any rank frees its region
        barrier()
    rs.free()
    # beside the headline: config[4] (one stream over all GPUs) at N > 1 and
    # config[3] (64 streams per GPU, and 64 in total at N > 1)
    if world > 1 and not args.no_extra:
        line["tp"] = tp_record(model, teacher if tp_mode else token_stream(0, 4096, V), args, world, rank, barrier)
    if not tp_mode and not args.no_extra:
        line["streams"] = streams_record(model, args, world, rank, barrier)
    model.free()
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
