#!/usr/bin/env python
"""Benchmark of the jero-kernels-rvv quantized-matmul hot path on B200 (sm_100a).

Headline workload (`--workload 8b`): the Llama-3-8B decode GEMV set at
batch 1 -- Q4_K_M q/o 4096->4096, k/v 4096->1024, gate/up 4096->14336, down 14336->4096 and the
Q6_K lm_head 4096->128256, each fed by its own Q8_K-quantized activation. One step runs the
matrices through the C ABI (jkb200), grouped by the activation stream that feeds them, as a
decoder layer allows (q/k/v, o, gate/up, down, lm_head): the layer groups with the f32-input
entries (vec_dot_grouped_rvv, the quantization inside the GEMV launch) and the lm_head as
quantize_row_q8_k + gemv_q6_k_q8_k (--prequant picks which streams get their own quantize
launch); with --unfused as five quantize launches plus eight GEMV launches. Weights are
synthetic N(0, 0.02) rows quantized by this file's numpy quantizers (a seeded pool of rows tiled
to full size; GEMV time does not depend on the values), activations N(0, 1).

Metric: algorithmic bytes per step (GGUF weight blocks + Q8_K activation blocks + f32 outputs)
/ step time, in GB/s. The seven layer matrices exist in two copies used on alternate steps and
the lm_head is 431 MB, so every step streams 554 MB (> 4x the 126 MB L2).

With --gpus N (torchrun, one rank per GPU) every matrix is sharded by output rows; each rank
runs its slices, and one launch of this library's all-gather kernel per step pushes the output
slices to every peer over NVLink (--collective push: the GEMV kernels store every row into
every peer's buffer as they compute it, and one signal kernel completes the step; nccl: one
NCCL all-gather). Strong scaling: the same total work at every N.

Sections of the same JSON line: the Llama-3-70B decode set at batch 1 and 16, the
Q4_0 GEMV, the Q8_0 prefill GEMM and BitNet BitLinear.

`--impl reference` times the CPU restatement of the reference's scalar path (oracle/) on all
host cores over the same workload (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "jero-kernels-rvv_b200"))

Q4_0, Q4_K, Q6_K, Q8_0, TQ2_0, I2_S = 2, 12, 14, 8, 35, 36
BLOCK = {Q4_0: (32, 18), Q4_K: (256, 144), Q6_K: (256, 210), Q8_0: (32, 34), TQ2_0: (256, 66),
         I2_S: (128, 32)}
# BitNet-b1.58-2B FFN: hidden 2560, intermediate 6912
BITNET_HIDDEN, BITNET_FFN = 2560, 6912

# (name, quant, rows, cols, activation stream)
DECODE_8B = [
    ("attn_q", Q4_K, 4096, 4096, "x"), ("attn_k", Q4_K, 1024, 4096, "x"),
    ("attn_v", Q4_K, 1024, 4096, "x"), ("attn_o", Q4_K, 4096, 4096, "attn"),
    ("ffn_gate", Q4_K, 14336, 4096, "h"), ("ffn_up", Q4_K, 14336, 4096, "h"),
    ("ffn_down", Q4_K, 4096, 14336, "a"), ("lm_head", Q6_K, 128256, 4096, "f"),
]
ACTS = {"x": 4096, "attn": 4096, "h": 4096, "a": 14336, "f": 4096}
# Llama-3-70B decode: Q4_K_M gate/up 8192->28672, down 28672->8192, Q6_K
# lm_head 8192->128256, weights N(0, 0.015), batch 1 and 16, sharded over 1/2/4/8 GPUs
DECODE_70B = [
    ("ffn_gate", Q4_K, 28672, 8192, "h"), ("ffn_up", Q4_K, 28672, 8192, "h"),
    ("ffn_down", Q4_K, 8192, 28672, "a"), ("lm_head", Q6_K, 128256, 8192, "f"),
]
ACTS_70B = {"h": 8192, "a": 28672, "f": 8192}
DECODE_SETS = {
    "8b": {"key": "llama3_8b_decode", "config": "configs[1]", "mats": DECODE_8B, "acts": ACTS,
           "copies": 2, "sigma": 0.02, "workload": "llama3-8b-decode-gemv-set",
           "lm_profile": "gemv_q6_k_lm_head_4096x128256",
           "l2": "inputs larger than L2 (554 MB per step, layer weights in 2 alternating "
                 "copies)"},
    "70b": {"key": "llama3_70b_decode", "config": "configs[4]", "mats": DECODE_70B,
            "acts": ACTS_70B, "copies": 1, "sigma": 0.015, "batch16": True,
            "workload": "llama3-70b-decode-gemv-set",
            "lm_profile": "gemv_q6_k_lm_head_4096x128256",
            "l2": "inputs larger than L2 (1.26 GB per step)"},
}
POOL_ROWS = 512


# ----------------------------------------------------------------------------- synthetic data

def _f16(x):
    return np.asarray(x, np.float32).astype(np.float16)


def _rnd(x):
    """Round half away from zero (C roundf / Rust f32::round), evaluated exactly in f64."""
    x = np.asarray(x, np.float64)
    return np.sign(x) * np.floor(np.abs(x) + 0.5)


def quantize_q4_k(w: np.ndarray) -> np.ndarray:
    """Q4_K blocks from f32 rows: per 32-element sub-block an affine (scale, min) pair
    re-quantized to 6 bits against f16 super-block d / dmin (same rule as the oracle's own
    quantizer, written with numpy)."""
    R, K = w.shape
    x = w.reshape(R, K // 256, 8, 32)
    lo = np.minimum(x.min(-1), 0.0)
    hi = x.max(-1)
    scale = (hi - lo) / np.float32(15.0)
    minv = -lo
    d = _f16(scale.max(-1) / np.float32(63.0)).astype(np.float32)
    dmin = _f16(minv.max(-1) / np.float32(63.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d[..., None] > 0, _rnd(scale / d[..., None]), 0).clip(0, 63).astype(np.uint8)
        m = np.where(dmin[..., None] > 0, _rnd(minv / dmin[..., None]), 0).clip(0, 63).astype(np.uint8)
        ds = d[..., None] * sc.astype(np.float32)
        dm = dmin[..., None] * m.astype(np.float32)
        q = np.where(ds[..., None] > 0, _rnd((x + dm[..., None]) / ds[..., None]), 0)
    q = q.clip(0, 15).astype(np.uint8).reshape(R, K // 256, 4, 2, 32)
    out = np.zeros((R, K // 256, 144), np.uint8)
    out[..., 0:2] = _f16(d).view(np.uint8).reshape(R, K // 256, 2)
    out[..., 2:4] = _f16(dmin).view(np.uint8).reshape(R, K // 256, 2)
    s = out[..., 4:16]
    s[..., 0:4] = (sc[..., 0:4] & 63) | ((sc[..., 4:8] >> 4) << 6)
    s[..., 4:8] = (m[..., 0:4] & 63) | ((m[..., 4:8] >> 4) << 6)
    s[..., 8:12] = (sc[..., 4:8] & 15) | ((m[..., 4:8] & 15) << 4)
    out[..., 16:] = (q[..., 0, :] | (q[..., 1, :] << 4)).reshape(R, K // 256, 128)
    return out.reshape(-1)


def quantize_q6_k(w: np.ndarray) -> np.ndarray:
    """Q6_K blocks from f32 rows: 16-element sub-block scales absmax/31 as i8 against an f16
    super-block d, values q+32 packed into ql/qh."""
    R, K = w.shape
    x = w.reshape(R, K // 256, 16, 16)
    s = np.abs(x).max(-1) / np.float32(31.0)
    d = _f16(s.max(-1) / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d[..., None] > 0, _rnd(s / d[..., None]), 0).clip(-128, 127).astype(np.int8)
        ds = d[..., None] * sc.astype(np.float32)
        q = np.where(ds[..., None] != 0, _rnd(x / ds[..., None]), 0)
    u = (q.clip(-32, 31) + 32).astype(np.uint8).reshape(R, K // 256, 2, 4, 32)
    out = np.zeros((R, K // 256, 210), np.uint8)
    for h in range(2):
        ql = out[..., 64 * h:64 * h + 64]
        ql[..., 0:32] = (u[..., h, 0, :] & 15) | ((u[..., h, 2, :] & 15) << 4)
        ql[..., 32:64] = (u[..., h, 1, :] & 15) | ((u[..., h, 3, :] & 15) << 4)
        out[..., 128 + 32 * h:160 + 32 * h] = ((u[..., h, 0, :] >> 4) | ((u[..., h, 1, :] >> 4) << 2)
                                               | ((u[..., h, 2, :] >> 4) << 4)
                                               | ((u[..., h, 3, :] >> 4) << 6))
    out[..., 192:208] = sc.view(np.uint8)
    out[..., 208:210] = _f16(d).view(np.uint8).reshape(R, K // 256, 2)
    return out.reshape(-1)


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    R, K = w.shape
    x = w.reshape(R, K // 32, 32)
    d = np.abs(x).max(-1) / np.float32(127.0)
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = np.where(d > 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
        q = _rnd(x * inv[..., None]).clip(-127, 127).astype(np.int8)
    out = np.zeros((R, K // 32, 34), np.uint8)
    out[..., 0:2] = _f16(d).view(np.uint8).reshape(R, K // 32, 2)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(-1)


def quantize_q4_0(w: np.ndarray) -> np.ndarray:
    """Q4_0 blocks from f32 rows: the signed value of largest magnitude over -8 as the f16 block
    scale, q = min(15, trunc(x / d + 8.5)) in f32 (the oracle's rule, written with numpy)."""
    R, K = w.shape
    x = np.ascontiguousarray(w, np.float32).reshape(R, K // 32, 32)
    mx = np.take_along_axis(x, np.abs(x).argmax(-1)[..., None], -1)[..., 0]
    d = (mx / np.float32(-8.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        idv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    q = np.trunc((x * idv[..., None]).astype(np.float32) + np.float32(8.5)).clip(0, 15)
    q = q.astype(np.uint8)
    out = np.zeros((R, K // 32, 18), np.uint8)
    out[..., 0:2] = _f16(d).view(np.uint8).reshape(R, K // 32, 2)
    out[..., 2:] = q[..., :16] | (q[..., 16:] << 4)
    return out.reshape(-1)


QUANTIZERS = {Q4_0: quantize_q4_0, Q4_K: quantize_q4_k, Q6_K: quantize_q6_k, Q8_0: quantize_q8_0}


def synth_matrix(quant, rows, cols, seed, row_begin=0, row_end=None, sigma=0.02):
    """GGUF bytes of rows [row_begin, row_end) of a seeded N(0, sigma) matrix: a pool of
    POOL_ROWS quantized rows tiled over the matrix."""
    row_end = rows if row_end is None else row_end
    rng = np.random.default_rng(seed)
    pool = rng.standard_normal((min(POOL_ROWS, rows), cols), dtype=np.float32) * np.float32(sigma)
    qp = QUANTIZERS[quant](pool).reshape(pool.shape[0], -1)
    idx = np.arange(row_begin, row_end) % pool.shape[0]
    return np.ascontiguousarray(qp[idx]).reshape(-1)


def algorithmic_bytes(quant, rows, cols, batch=1):
    """GGUF weight block bytes + per token the Q8 activation blocks (Q8_K for the K-quants,
    Q8_0 otherwise) and the f32 outputs."""
    be, bb = BLOCK[quant]
    act = cols // 256 * 292 if quant in (Q4_K, Q6_K) else cols // 32 * 36
    return rows * (cols // be) * bb + batch * (act + 4 * rows)


# ----------------------------------------------------------------------------- helpers

def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(kernel_key):
    """dram bytes per launch recorded from an ncu capture in profiles/<kernel_key>.txt
    ("traffic_bytes_per_launch: N" line), or None."""
    p = os.path.join(ROOT, "profiles", f"{kernel_key}.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- reference arm

def cpu_oracle_step(O, mats, xq, nthreads):
    for name, quant, rows, cols, stream, w in mats:
        O.gemv_mt(quant, w, rows, cols, xq[stream], nthreads)


def cpu_workload(O, spec):
    """The whole decode set on the host (CPU arms): every matrix once (the host has no L2 to
    defeat at this size), the Q8_K activations of the same seeded streams."""
    mats = []
    for i, (name, quant, rows, cols, stream) in enumerate(spec["mats"]):
        mats.append((name, quant, rows, cols, stream,
                     synth_matrix(quant, rows, cols, 1000 + i, sigma=spec["sigma"])))
    rng = np.random.default_rng(7)
    xq = {s: O.quantize_row_q8_k(rng.standard_normal(n, dtype=np.float32))
          for s, n in spec["acts"].items()}
    nbytes = sum(algorithmic_bytes(q, r, c) for _, q, r, c, _, _ in mats)
    return mats, xq, nbytes


def cpu_model():
    """The host CPU's model name (/proc/cpuinfo), or the platform's processor string."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.lower().startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def run_reference(args):
    """The reference's scalar path (the oracle's C restatement; the Rust crate cannot be built
    here) on the host cores, on the same workload, metric and config as the GPU arm: each step
    is one whole decode step, every matrix's rows split over all host threads (the reference's
    own row-range parallelism, gemv_repacked_rows repack.rs:4014). Rank 0 only."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as O

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    spec = DECODE_SETS[args.workload]
    cores = os.cpu_count() or 1
    mats, xq, nbytes = cpu_workload(O, spec)
    for _ in range(args.warmup):
        cpu_oracle_step(O, mats, xq, cores)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_oracle_step(O, mats, xq, cores)
    dt = (time.perf_counter() - t0) / args.steps
    gbs = nbytes / dt / 1e9
    sample = (f"{args.steps} whole decode steps ({nbytes / 1e6:.1f} MB each), oracle scalar "
              f"port, every matrix's rows split over {cores} threads")
    print(json.dumps({
        "impl": "reference", "metric": "quant GEMV weight GB/s", "value": round(gbs, 3),
        "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8 dot / f32 scale", "data": "synthetic",
        "config": decode_config(spec, args.gpus, args.collective),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores,
                         "kind": "port", "sample": sample, "cpu_model": cpu_model()},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def cpu_baseline_single(spec):
    """Oracle port on one host core over whole decode steps of the same workload, repeated for
    about 10 s."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as O

    mats, xq, nbytes = cpu_workload(O, spec)
    n, t0 = 0, time.perf_counter()
    while True:
        cpu_oracle_step(O, mats, xq, 1)
        n += 1
        if time.perf_counter() - t0 > 10.0:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": round(nbytes / dt / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
            "cpu_model": cpu_model(),
            "sample": f"{n} whole decode steps ({nbytes / 1e6:.1f} MB each), single thread"}


# ----------------------------------------------------------------------------- GPU arm

class DecodeSet:
    """This rank's part of one decode GEMV set (BASELINE configs[1] or configs[4]): the output-row
    shard of every matrix as a jkb200 Weight, the f32 activation streams in one device buffer,
    and the calls of one step through the public API.

    A step runs, per activation stream in order, the matrices that stream feeds (a decoder layer
    computes q/k/v from one input, gate/up from another, ...):
      * batch 1, streams not in `prequant`: one f32-input launch, grouped when several matrices
        share the stream (vec_dot_grouped_rvv; the input is quantized to Q8_K inside the launch);
      * batch 1, streams in `prequant` (default: the lm_head's): quantize_row_q8_k, then one
        pre-quantized gemv_rows launch per matrix;
      * batch m > 1: quantize_rows_q8_k of the m tokens, then one gemv_batch launch per matrix;
      * `unfused`: every stream quantized by its own launch, one GEMV launch per matrix.
    With world > 1 the output shards are collected once per step, by the library's all-gather
    kernel over NVLink peer memory (`peer`) or by one NCCL all-gather.
    Layer matrices can exist in `layer_copies` copies used on alternate steps, so that a step
    never finds its weights in the L2."""

    def __init__(self, jkb, mats, acts, world, rank, *, peer=True, push=False, batch=1,
                 layer_copies=1, prequant=("f",), unfused=False, seed=1000, sigma=0.02,
                 tc=False):
        import torch
        from jkb200.shard import PeerOutputs, ShardedOutputs

        self.jkb, self.mats, self.acts = jkb, mats, acts
        self.world, self.rank, self.batch = world, rank, batch
        self.peer = peer and world > 1
        self.push = push and self.peer
        self.unfused, self.prequant = unfused, set(prequant) - {""}
        # token batches on the tensor cores: i8 RepackedWeights and one QuantizedActQ8 per
        # activation stream (gemm_repacked) instead of GGUF-layout weights and gemv_batch
        self.tc = tc and batch > 1
        names = [(name, rows) for name, _, rows, _, _ in mats]
        # two output slots alternate by step parity (a step's outputs stay readable while the
        # next step runs): the peer group's two slots, or two flat NCCL / single-GPU buffers
        self.outs = (PeerOutputs(names, world, rank, batch=batch, push=self.push) if self.peer
                     else ShardedOutputs(names, world, rank, batch=batch))
        self.outs2 = (None if self.peer
                      else [self.outs, ShardedOutputs(names, world, rank, batch=batch)])
        self.weights, self.shards, self.bytes_per_step = {}, [], 0
        for i, (name, quant, rows, cols, s) in enumerate(mats):
            rr = self.outs.rows_of(name)
            self.bytes_per_step += algorithmic_bytes(quant, rows, cols, batch)
            copies = 1 if name == "lm_head" else layer_copies
            for c in range(copies):
                raw = synth_matrix(quant, rows, cols, seed + i + 97 * c, rr.start, rr.stop, sigma)
                view = jkb.TensorView(f"{name}.{c}", quant, [len(rr), cols], raw)
                self.weights[(name, c)] = (jkb.RepackedWeight.from_tensor(view, len(rr), cols)
                                           if self.tc else jkb.Weight(view, len(rr), cols))
            self.shards.append((name, quant, len(rr), cols, s, copies))
        g = torch.Generator(device="cpu").manual_seed(7)
        # all activation streams in one device buffer: the e2e loop moves a step's inputs with
        # one host-to-device copy
        # (two input slots alternate by step parity like the outputs: the e2e loop copies the
        # next step's inputs in while a step runs)
        x0 = torch.cat([torch.randn(batch * n, generator=g) for n in acts.values()])
        self.x_slots = [x0.cuda(), x0.cuda()]
        self.x_all = self.x_slots[0]
        self.xs_slots, self.xq, off = [{}, {}], {}, 0
        for s, n in acts.items():
            for k in range(2):
                self.xs_slots[k][s] = self.x_slots[k][off:off + batch * n]
            self.xq[s] = (jkb.QuantizedActQ8(batch, n) if self.tc
                          else jkb.empty_q8_k_blocks(batch * n // 256))
            off += batch * n
        self.xs = self.xs_slots[0]
        self.groups = {}  # activation stream -> matrices fed by it, in mats order
        for name, quant, per, cols, s, copies in self.shards:
            self.groups.setdefault(s, []).append((name, copies))
        self.lm_stream = mats[-1][4]
        self.launches_per_step = self._count_launches()

    def _count_launches(self):
        n = 1 if self.peer else 0
        for s, items in self.groups.items():
            if self.batch > 1 or self.unfused or s in self.prequant:
                n += 1 + len(items)
            else:
                n += 1
        return n

    def lslice(self, name, i):
        if self.peer:
            return self.outs.local_slice(name, i % 2)
        return self.outs2[i % 2].local_slice(name)

    def run_group(self, s, i):
        jkb = self.jkb
        items = [(self.lslice(n, i), self.weights[(n, i % c)]) for n, c in self.groups[s]]
        xs = self.xs_slots[i % 2]
        if self.tc:
            self.xq[s].quantize_into(xs[s], self.batch, self.acts[s])
            for out, w in items:
                w.gemm(out, self.xq[s])
        elif self.batch > 1:
            jkb.quantize_rows_q8_k(xs[s], self.batch, self.acts[s], self.xq[s])
            for out, w in items:
                jkb.gemv_batch(out, w, self.xq[s], self.batch)
        elif self.unfused or s in self.prequant:
            jkb.quantize_row_q8_k(xs[s], self.xq[s])
            for out, w in items:
                jkb.gemv_rows(out, w, self.xq[s], range(0, w.rows))
        else:
            jkb.vec_dot_grouped_rvv(items, xs[s])

    def layer_part(self, i):
        for s in self.groups:
            if s != self.lm_stream:
                self.run_group(s, i)

    def collect(self, i):
        if self.peer:
            self.outs.gather(i % 2)
        else:
            self.outs2[i % 2].gather()

    def step(self, i, marks=None, stream=None):
        """One step. `marks`: 4 events recorded before the layer GEMVs, before the lm_head group,
        after it and after the collection of the shards."""
        if marks is not None:
            marks[0].record(stream)
        self.layer_part(i)
        if marks is not None:
            marks[1].record(stream)
        self.run_group(self.lm_stream, i)
        if marks is not None:
            marks[2].record(stream)
        self.collect(i)
        if marks is not None:
            marks[3].record(stream)

    def c_calls(self, k, stream):
        """Step calls of output/input slot k (steps i with i % 2 == k) as C-ABI function +
        argument tuples with every pointer resolved, for a caller that replays them each step
        (the e2e loop): the same calls layer_part / run_group / collect make, validated by a
        first eager step. Returns (compute calls before the collection, collection calls);
        a call is (cfunc, args) or a Python callable (the NCCL all-gather)."""
        import ctypes as C
        from jkb200 import _lib

        L = _lib.load()
        xs = self.xs_slots[k]
        keep = []  # ctypes arrays referenced by the argument tuples
        calls = []

        def group(s):
            items = [(self.lslice(n, k), self.weights[(n, k % c)]) for n, c in self.groups[s]]
            if self.tc:
                calls.append((L.jkb_act_q8_quantize, (self.xq[s]._h, xs[s].data_ptr(),
                              xs[s].numel(), self.batch, self.acts[s], stream)))
                for out, w in items:
                    calls.append((L.jkb_gemm_repacked, (out.data_ptr(), out.numel(), w._h,
                                  self.xq[s]._h, stream)))
            elif self.batch > 1:
                calls.append((L.jkb_quantize_rows_q8_k, (xs[s].data_ptr(), self.batch,
                              self.acts[s], self.xq[s].data_ptr(), self.xq[s].numel() // 292,
                              stream)))
                for out, w in items:
                    calls.append((L.jkb_gemv_batch, (out.data_ptr(), out.numel(), w.handle,
                                  self.xq[s].data_ptr(), self.xq[s].numel() // 292, self.batch,
                                  stream)))
            elif self.unfused or s in self.prequant:
                calls.append((L.jkb_quantize_row_q8_k, (xs[s].data_ptr(), xs[s].numel(),
                              self.xq[s].data_ptr(), self.xq[s].numel() // 292, stream)))
                for out, w in items:
                    calls.append((L.jkb_gemv_rows, (out.data_ptr(), out.numel(), w.handle,
                                  self.xq[s].data_ptr(), self.xq[s].numel() // 292, 0, w.rows,
                                  stream)))
            else:
                arr = (_lib.jkb_vec_dot_item * len(items))()
                for j, (out, w) in enumerate(items):
                    arr[j].out, arr[j].out_len, arr[j].w = out.data_ptr(), out.numel(), w.handle
                keep.append(arr)
                calls.append((L.jkb_vec_dot_grouped_rvv, (arr, len(items), xs[s].data_ptr(),
                                                          xs[s].numel(), stream)))

        for s in self.groups:
            if s != self.lm_stream:
                group(s)
        group(self.lm_stream)
        coll = []
        if self.push:
            coll.append((L.jkb_peer_group_signal, (self.outs.group.handle, stream)))
        elif self.peer:
            if not hasattr(self.outs, "_chunks"):
                self.outs._chunks = [self.outs.group.chunk_arrays(self.outs.chunks(j))
                                     for j in range(self.outs.SLOTS)]
            offs, lens, n = self.outs._chunks[k]
            coll.append((L.jkb_peer_group_allgather, (self.outs.group.handle, offs, lens, n,
                                                      stream)))
        elif self.world > 1:
            coll.append(lambda: self.outs2[k].gather())
        self._keep_c = getattr(self, "_keep_c", []) + keep
        return calls, coll

    def output(self, name, i):
        """Full output of matrix `name` after step i: [rows], or [batch][rows]."""
        if self.peer:
            return self.outs.output(name, i % 2)
        o = self.outs2[i % 2]
        if self.world == 1:
            t = o.local_slice(name)
            return t if self.batch == 1 else t.view(self.batch, -1)
        return o.output(name)

    def full(self, i):
        """The buffer holding every matrix's full output after step i (the e2e read-back)."""
        if self.peer:
            return self.outs.full(i % 2)
        return self.outs2[i % 2].gathered

    def destroy(self):
        for w in self.weights.values():
            w.destroy()
        if self.tc:
            for a in self.xq.values():
                a.destroy()
        if self.peer:
            self.outs.destroy()


def _max_over_ranks(v, world, op="max"):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.MIN)
    return float(t.item())


def time_decode(ds, steps, warmup, stream, world, local=0, sample_clocks=False):
    """Times `steps` decode steps of DecodeSet `ds` captured as one CUDA graph (a launch-bound
    loop), with CUDA events on the launching stream, max over ranks. A second graph of the same
    steps carries events at the group boundaries of every step (layer GEMVs | lm_head group |
    collection of the shards): an event between two kernels ends the programmatic overlap of
    their launches, so it is timed separately and gives the split, not the headline."""
    import torch
    import torch.distributed as dist

    for i in range(warmup):  # eager warm-up (also sets kernel attributes)
        ds.step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    marks = [[torch.cuda.Event(enable_timing=True, external=True) for _ in range(4)]
             for _ in range(steps)]
    graph, graph_ev = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(steps):
            ds.step(i)
    with torch.cuda.graph(graph_ev, stream=stream):
        for i in range(steps):
            ds.step(i, marks[i], stream)
    graph.replay()  # untimed first replays (graph upload)
    graph_ev.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks, sampler = None, None
    if sample_clocks:
        t_start.record(stream)
        graph.replay()
        t_end.record(stream)
        torch.cuda.synchronize()
        # nvidia-smi samples every 100 ms and the timed replay lasts milliseconds: about 0.5 s of
        # untimed replays of the same graph run right before it, so the clock samples are taken
        # under this workload.
        # the same count on every rank (each replay holds one exchange per step)
        n_load = max(1, int(500.0 / max(_max_over_ranks(t_start.elapsed_time(t_end), world),
                                        1e-3)))
        sampler = ClockSampler(local)
        sampler.start()
        time.sleep(0.2)
        for _ in range(n_load):
            graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_start.record(stream)
    graph.replay()  # the K timed steps
    t_end.record(stream)
    graph_ev.replay()  # K more steps with the split events, under the same clocks
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if sampler is not None:
        clocks = sampler.stop()
        clocks["window"] = (f"nvidia-smi every 100 ms over {n_load} untimed replays of the timed "
                            "graph and the timed replays")
    ms = _max_over_ranks(t_start.elapsed_time(t_end), world)
    split = [sum(m[j].elapsed_time(m[j + 1]) for m in marks) / steps for j in range(3)]
    split = [_max_over_ranks(v, world) for v in split]
    del graph, graph_ev
    return {"ms_step": ms / steps, "layer_ms": split[0], "lm_head_ms": split[1],
            "gather_ms": split[2], "clocks": clocks}


def e2e_decode(ds, steps, warmup, world, stream):
    """The same steps through the public C ABI with host buffers, the way a compiled caller
    drives it: each step's calls are prebuilt once per slot as ctypes function and argument
    tuples (DecodeSet.c_calls: validation and pointer lookup happen once, as an engine holding
    handles would do), and the copies and events go straight to the CUDA runtime. Every step
    copies its f32 inputs in from pinned host memory and its full outputs out to pinned host
    memory. The copies run on a second stream and overlap the neighbouring steps' kernels: step
    i's inputs arrive in input slot i % 2 while step i - 1 runs, and its outputs leave from
    output slot i % 2 while step i + 1 runs; events order each copy after what it depends on and
    before what would overwrite it (including a peer's push into the slot, which cannot happen
    before this rank's all-gather of step i + 1, so that all-gather waits for the read-back of
    step i). Timed with CUDA events on the compute stream from before the first copy in to after
    the last copy out, max over ranks. Also reports the host's time per step to enqueue."""
    import ctypes as C

    import torch
    import torch.distributed as dist

    rt = C.CDLL("libcudart.so.12")  # the CUDA runtime torch has loaded
    rt.cudaMemcpyAsync.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_void_p]
    rt.cudaEventRecord.argtypes = [C.c_void_p, C.c_void_p]
    rt.cudaStreamWaitEvent.argtypes = [C.c_void_p, C.c_void_p, C.c_uint]
    rt.cudaEventCreateWithFlags.argtypes = [C.POINTER(C.c_void_p), C.c_uint]
    copy = torch.cuda.Stream()
    cs, ks = stream.cuda_stream, copy.cuda_stream
    host_in = [ds.x_slots[0].cpu().pin_memory(), ds.x_slots[1].cpu().pin_memory()]
    n_out = ds.full(0).numel()
    host_out = [torch.empty(n_out, dtype=torch.float32).pin_memory() for _ in range(2)]
    in_bytes, out_bytes = host_in[0].numel() * 4, n_out * 4

    def event():
        e = C.c_void_p()
        assert rt.cudaEventCreateWithFlags(C.byref(e), 2) == 0  # cudaEventDisableTiming
        return e
    # Events (one per slot): comp[k] after a step of slot k; inp[k] on the copy stream after the
    # read-back of step j - 2 and the copy-in of step j (slot k = j % 2); back[k] after the
    # read-back of a step of slot k. The compute stream takes one wait and one record a step
    # (two with peers, whose pushes into a slot must follow its read-back): every stream
    # operation between two kernels ends their programmatic launch overlap.
    ev = {name: [event(), event()] for name in ("comp", "inp", "back")}
    plan = [ds.c_calls(k, cs) for k in range(2)]
    slot_io = [(ds.x_slots[k].data_ptr(), host_in[k].data_ptr(), ds.full(k).data_ptr(),
                host_out[k].data_ptr()) for k in range(2)]

    def call(c):
        if callable(c):
            c()
            return
        rc = c[0](*c[1])
        if rc:
            raise RuntimeError(f"{c[0].__name__} failed ({rc}): {ds.jkb._lib.load().jkb_last_error()}")

    def copy_in(j):
        """Copy stream: the inputs of step j into slot j % 2, after step j - 2 (same slot) has
        finished and its outputs have been read back."""
        k = j % 2
        dx, hx, _, _ = slot_io[k]
        rt.cudaStreamWaitEvent(ks, ev["comp"][k], 0)
        rt.cudaMemcpyAsync(dx, hx, in_bytes, 1, ks)
        rt.cudaEventRecord(ev["inp"][k], ks)

    def run(i0, n):
        for i in range(i0, i0 + n):
            k = i % 2
            _, _, dy, hy = slot_io[k]
            rt.cudaStreamWaitEvent(cs, ev["inp"][k], 0)
            calls, coll = plan[k]
            for c in calls:
                call(c)
            if coll:
                rt.cudaStreamWaitEvent(cs, ev["back"][1 - k], 0)  # read-back of step i - 1
                for c in coll:
                    call(c)
            rt.cudaEventRecord(ev["comp"][k], cs)
            # copy stream: this step's outputs out, then the inputs of step i + 2 (same slot)
            rt.cudaStreamWaitEvent(ks, ev["comp"][k], 0)
            rt.cudaMemcpyAsync(hy, dy, out_bytes, 2, ks)
            rt.cudaEventRecord(ev["back"][k], ks)
            copy_in(i + 2)

    ds.step(0)  # one eager step through the checked API first
    torch.cuda.synchronize()
    copy_in(1)
    copy_in(2)
    run(1, warmup)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    copy.wait_event(e0)
    t0 = time.perf_counter()
    run(1 + warmup, steps)  # step numbers continue, so the slots alternate across the boundary
    host_s = time.perf_counter() - t0
    rt.cudaStreamWaitEvent(cs, ev["back"][(warmup + steps) % 2], 0)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1), world)
    return {"ms_step": ms / steps, "h2d_bytes_per_step": in_bytes,
            "d2h_bytes_per_step": out_bytes, "host_us_per_step": round(host_s / steps * 1e6, 2)}


def decode_section(jkb, spec, world, rank, stream, steps, warmup, batch, peer, push, tc=False):
    """configs[4]-style numbers for one decode set and batch: GB/s of the whole job, the
    fraction of measured HBM per GPU, and the per-step split (max over ranks)."""
    mats, acts, copies, sigma = spec["mats"], spec["acts"], spec["copies"], spec["sigma"]
    ds = DecodeSet(jkb, mats, acts, world, rank, peer=peer, push=push, batch=batch,
                   layer_copies=copies, sigma=sigma, tc=tc)
    t = time_decode(ds, steps, warmup, stream, world)
    peak, _ = measured_peaks()
    gbs = ds.bytes_per_step / (t["ms_step"] * 1e-3) / 1e9
    res = {"batch": batch, "bytes_per_step": ds.bytes_per_step,
           "us_per_step": round(t["ms_step"] * 1e3, 2), "gbs": round(gbs, 1),
           "hbm_frac_per_gpu": round(gbs / world / peak, 4),
           "split_us": {"layer_gemvs": round(t["layer_ms"] * 1e3, 2),
                        "lm_head": round(t["lm_head_ms"] * 1e3, 2),
                        "gather": round(t["gather_ms"] * 1e3, 2)},
           "launches_per_step": ds.launches_per_step,
           "weights": ("i8 RepackedWeight, gemm_repacked (tensor cores, 32-token tile: two "
                       "CTAs per SM with more tiles than SMs, K split over a cluster with few); "
                       "GB/s counts the GGUF bytes of the same matrices" if ds.tc else
                       "GGUF blocks, " + ("gemv_batch" if batch > 1 else "f32-input GEMV"))}
    ds.destroy()
    return res


def run_gpu(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    import jkb200 as jkb

    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    peer, push = args.collective in ("push", "peer"), args.collective == "push"
    spec = DECODE_SETS[args.workload]
    # --- the headline: this rank's row shard of every matrix of the decode set
    ds = DecodeSet(jkb, spec["mats"], spec["acts"], world, rank, peer=peer, push=push,
                   layer_copies=spec["copies"], prequant=args.prequant.split(","),
                   unfused=args.unfused, sigma=spec["sigma"])
    t = time_decode(ds, args.steps, args.warmup, stream, world, local, sample_clocks=True)
    total_bytes = ds.bytes_per_step
    ms_step = t["ms_step"]
    value = total_bytes / (ms_step * 1e-3) / 1e9
    e2e = e2e_decode(ds, args.steps, args.warmup, world, stream)
    e2e_val = total_bytes / (e2e["ms_step"] * 1e-3) / 1e9
    launches = ds.launches_per_step
    ds.destroy()
    torch.cuda.synchronize()

    sections = {}
    if not args.no_sections:
        other = "70b" if args.workload == "8b" else "8b"
        sections[DECODE_SETS[other]["key"]] = {
            "config": DECODE_SETS[other]["config"],
            "batch1": decode_section(jkb, DECODE_SETS[other], world, rank, stream, args.steps,
                                     args.warmup, 1, peer, push)}
        for key, sp in DECODE_SETS.items():
            if sp.get("batch16"):
                sec = sections.setdefault(sp["key"], {"config": sp["config"]})
                sec["batch16"] = decode_section(jkb, sp, world, rank, stream,
                                                max(4, args.steps // 4), args.warmup, 16, peer,
                                                push)
                # the same batch on the tensor cores: i8 RepackedWeights + gemm_repacked
                sec["batch16_tc"] = decode_section(jkb, sp, world, rank, stream,
                                                   max(4, args.steps // 4), args.warmup, 16,
                                                   peer, push, tc=True)
        sections["q4_0_gemv_4096"] = run_q4_0_gemv(jkb, world)
        sections["per_shape_" + spec["key"]] = run_decode_shapes(jkb, spec, world, rank)
    prefill = None if args.no_gemm else run_prefill_gemm(world, rank)
    bitnet = None if args.no_bitnet else run_bitnet(world, rank)

    if rank == 0:
        peak, peak_kind = measured_peaks()
        lm_q, lm_rows, lm_cols = spec["mats"][-1][1:4]
        lm_bytes = algorithmic_bytes(lm_q, lm_rows, lm_cols) / world
        lm_ms = t["lm_head_ms"]
        achieved = lm_bytes / (lm_ms * 1e-3) / 1e9
        # DRAM bytes per launch of the ncu capture, scaled from the 8B lm_head (431,457,856
        # algorithmic bytes) to this launch's algorithmic bytes
        traffic = profile_traffic(spec["lm_profile"])
        if traffic is not None:
            traffic = round(traffic * lm_bytes / algorithmic_bytes(Q6_K, 128256, 4096))
        lm_kernel = ("gemv_kernel<FQ6_K, ActQ8K>" if args.unfused or "f" in args.prequant
                     else "gemv_kernel<FQ6_K, ActQ8KF32>")
        res = {
            "metric": "quant GEMV weight GB/s", "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8 dot / f32 scale", "data": "synthetic",
            "config": decode_config(spec, world, args.collective),
            "split_us": {"layer_gemvs": round(t["layer_ms"] * 1e3, 2),
                         "lm_head": round(t["lm_head_ms"] * 1e3, 2),
                         "gather": round(t["gather_ms"] * 1e3, 2),
                         "note": "a second graph of the same steps with events at the group "
                                 "boundaries (events end the launch overlap there)"},
            "roofline": {"bound": "hbm",
                         "kernel": f"{lm_kernel} lm_head {lm_cols}->{lm_rows}"
                                   + (f" (row shard 1/{world})" if world > 1 else ""),
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "traffic": traffic, "algorithmic_bytes": lm_bytes,
                         "avg_ms": round(lm_ms, 5),
                         "timed": "lm_head group (its quantize_row_q8_k launch + the GEMV) "
                                  "between events, averaged over the K steps"},
            "gpu_launches": args.steps * launches,
            "clocks": t["clocks"],
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": e2e["h2d_bytes_per_step"],
                    "d2h_bytes_per_step": e2e["d2h_bytes_per_step"],
                    "host_us_per_step": e2e["host_us_per_step"],
                    "copies": "pinned host buffers, copies on a second stream overlapping "
                              "the neighbouring steps' kernels",
                    "calls": "the C ABI through prebuilt ctypes call tuples"},
        }
        res.update(sections)
        if prefill is not None:
            res["prefill_gemm"] = prefill
        if bitnet is not None:
            res["bitnet"] = bitnet
        if world == 1 and not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline_single(spec)
        print(json.dumps(res), flush=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def decode_config(spec, world, collective):
    return {"workload": f"{spec['workload']} (BASELINE {spec['config']})", "batch": 1,
            "weights": "Q4_K_M layers + Q6_K lm_head",
            "l2": spec["l2"],
            "parallelism": f"row-shard x{world}" + (
                "" if world == 1 else
                " + rows pushed to the peers by the GEMVs over NVLink, one signal kernel"
                if collective == "push" else
                " + one-kernel all-gather over NVLink peer memory" if collective == "peer"
                else " + NCCL all-gather")}


def run_decode_shapes(jkb, spec, world, rank, launches=40):
    """Each activation group of a decode set on its own (this rank's row shards), with the step's
    own calls -- the grouped f32-input launch for the layer groups, quantize_row_q8_k + the
    pre-quantized GEMV for the lm_head -- over weight copies rotating past 2x the L2: us per
    group and GB/s of its algorithmic bytes (max over ranks for the time, whole-job bytes)."""
    import torch
    from jkb200.shard import shard_rows

    peak, _ = measured_peaks()
    groups = {}
    for i, (name, quant, rows, cols, st) in enumerate(spec["mats"]):
        groups.setdefault(st, []).append((i, name, quant, rows, cols))
    res = {}
    for st, mats in groups.items():
        nbytes = sum(algorithmic_bytes(q, r, c) for _, _, q, r, c in mats)
        shard_bytes = max(1, nbytes // world)
        copies = max(1, min(64, -(-260_000_000 // shard_bytes)))
        cols = mats[0][4]
        raws = {}
        for i, name, quant, rows, _ in mats:
            rr = shard_rows(rows, world, rank)
            raws[name] = (rr, synth_matrix(quant, rows, cols, 1000 + i, rr.start, rr.stop,
                                           spec["sigma"]))
        sets = []
        for c in range(copies):  # copies of the same bytes (GEMV time does not depend on them)
            items = []
            for i, name, quant, rows, _ in mats:
                rr, raw = raws[name]
                w = jkb.Weight(jkb.TensorView(name, quant, [len(rr), cols], raw), len(rr), cols)
                items.append((torch.empty(len(rr), dtype=torch.float32, device="cuda"), w))
            sets.append(items)
        x = torch.randn(cols, generator=torch.Generator().manual_seed(9)).cuda()
        xq = jkb.empty_q8_k_blocks(cols // 256)
        lm = st == spec["mats"][-1][4]
        it = [0]

        def one():
            items = sets[it[0] % copies]
            if lm:
                jkb.quantize_row_q8_k(x, xq)
                for out, w in items:
                    jkb.gemv_rows(out, w, xq, range(0, w.rows))
            else:
                jkb.vec_dot_grouped_rvv(items, x)
            it[0] += 1

        us = _max_over_ranks(_graph_time(one, max(launches, copies)), world)
        gbs = nbytes / (us * 1e-6) / 1e9
        res["+".join(n for _, n, _, _, _ in mats)] = {
            "us": round(us, 2), "gbs": round(gbs, 1),
            "hbm_frac_per_gpu": round(gbs / world / peak, 4), "bytes": nbytes}
        for items in sets:
            for _, w in items:
                w.destroy()
        del sets
        torch.cuda.empty_cache()
    return res


def run_q4_0_gemv(jkb, world, launches=60):
    """Q4_0 x Q8_0 GEMV, N = K = 4096, batch 1, weights N(0, 0.02). Each
    rank runs the whole matrix (replicas: 9.4 MB is below what sharding pays for); weight copies
    rotate so the graph of `launches` back-to-back calls streams more than 2x the L2. Two entry
    points: gemv_q4_0_q8_0 over a pre-quantized Q8_0 input, and vec_dot_q4_0_rvv with the f32
    input quantized inside the launch. Max over ranks."""
    import torch

    rows = cols = 4096
    nbytes = algorithmic_bytes(Q4_0, rows, cols)
    copies = -(-260_000_000 // nbytes)
    raw = synth_matrix(Q4_0, rows, cols, 4240)
    ws = [jkb.Weight(jkb.TensorView("q4_0", Q4_0, [rows, cols], raw), rows, cols)
          for _ in range(copies)]
    x = torch.randn(cols, generator=torch.Generator().manual_seed(3)).cuda()
    xq = jkb.empty_q8_0_blocks(cols // 32)
    jkb.quantize_row_q8_0(x, xq)
    out = torch.empty(rows, dtype=torch.float32, device="cuda")
    peak, _ = measured_peaks()
    res = {"config": "configs[0]", "rows": rows, "cols": cols, "algorithmic_bytes": nbytes,
           "l2": f"{copies} weight copies rotating ({copies * nbytes / 1e6:.0f} MB)"}
    for key, fn, inp in (("prequantized", jkb.gemv_q4_0_q8_0, xq),
                         ("f32_input", jkb.vec_dot_q4_0_rvv, x)):
        it = [0]

        def one():
            fn(out, ws[it[0] % copies], inp)
            it[0] += 1

        us = _max_over_ranks(_graph_time(one, max(launches, copies)), world)
        gbs = nbytes / (us * 1e-6) / 1e9
        res[key] = {"us": round(us, 3), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
    for w in ws:
        w.destroy()
    return res


PREFILL = [(512, 14336, 4096), (512, 4096, 14336), (2048, 14336, 4096), (2048, 4096, 14336)]


def synth_ternary(quant, rows, cols, seed, scale=0.02):
    """iid ternary weights (-1, 0, +1 with p = 1/3 each) packed as TQ2_0 (every block's f16
    scale = the tensor scale; byte i of a block holds elements 4i..4i+3, two bits each, value+1)
    or I2_S (byte g of a 128-element block holds elements g, 32+g, 64+g, 96+g in bits 7:6, 5:4,
    3:2, 1:0; the f32 tensor scale in a 32-byte trailer)."""
    t = np.random.default_rng(seed).integers(0, 3, size=(rows, cols), dtype=np.uint8)
    if quant == TQ2_0:
        c = t.reshape(rows, cols // 256, 64, 4)
        blk = np.empty((rows, cols // 256, 66), np.uint8)
        blk[..., 0:2] = np.frombuffer(np.float16(scale).tobytes(), np.uint8)
        blk[..., 2:] = c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)
        return blk.reshape(-1)
    c = t.reshape(rows, cols // 128, 4, 32)
    out = np.zeros(rows * cols // 4 + 32, np.uint8)
    out[:-32] = ((c[:, :, 0] << 6) | (c[:, :, 1] << 4) | (c[:, :, 2] << 2) | c[:, :, 3]).reshape(-1)
    out[-32:-28] = np.frombuffer(np.float32(scale).tobytes(), np.uint8)
    return out


def run_bitnet(world, rank, launches=20):
    """BitNet-b1.58-2B ternary BitLinear, TQ2_0 and I2_S weights, hidden
    2560 -> ffn 6912 and back, activations i8 per-token absmax-quantized (the SubLN quantizer
    with unit norm weights) from N(0, 1). Output rows are sharded over the ranks; every number is
    the max over ranks of a CUDA-event-timed CUDA graph of `launches` back-to-back calls.
      batch 1:   bitlinear_i8 per shape, weight copies rotating so that each launch reads from
                 HBM (GB/s of weight blocks + i8 activation + f32 output);
      batch 128: bitlinear_i8_batch (the GEMV kernel: each token one bitlinear_i8 call, up to
                 eight tokens sharing every weight load) and bitlinear_i8_gemm (tcgen05, one
                 TMEM accumulator per BitLinear block; default and bit-exact epilogue), in TOPS
                 (2*M*N*K);
      FFN:       the whole chain SubLN -> gate/up -> ReLU^2 + SubLN -> down (jkb_bitnet_ffn) at
                 1 token (GEMV kernels) and 128 tokens (tensor-core projections), in
                 microseconds per call (unsharded, on every rank)."""
    import torch
    import torch.distributed as dist
    import jkb200 as jkb

    def maxr(us):
        if world > 1:
            t = torch.tensor([us], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            us = float(t.item())
        return us

    H, F, M = BITNET_HIDDEN, BITNET_FFN, 128
    peak, peak_kind = measured_peaks()
    res = {"shapes": [], "note": "hidden 2560, ffn 6912; ternary iid p=1/3, scale 0.02",
           "batch1_roofline": "hbm: weight blocks + i8 activation + f32 output per launch "
                              f"over the launch time, of the {peak_kind} {peak} GB/s"}
    norm = {n: torch.ones(n, device="cuda") for n in (H, F)}

    def act_i8(n, m, seed):
        x = torch.randn(m * n, generator=torch.Generator().manual_seed(seed)).cuda()
        q = torch.empty(m * n, dtype=torch.int8, device="cuda")
        sc = torch.empty(m, dtype=torch.float32, device="cuda")
        jkb.subln_quantize_absmax_i8_rows(q, x, norm[n], m, n, 1e-5, sc)
        return x, q, sc

    for quant, qname in ((TQ2_0, "tq2_0"), (I2_S, "i2_s")):
        for rows, cols in ((F, H), (H, F)):
            per = rows // world
            be, bb = BLOCK[quant]
            wbytes = per * (cols // be) * bb
            copies = max(2, -(-300_000_000 // wbytes))
            raws = [synth_ternary(quant, per, cols, 77 + c) for c in range(min(copies, 4))]
            ws = [jkb.Weight(jkb.TensorView("w", quant, [per, cols], raws[c % len(raws)]), per,
                             cols) for c in range(copies)]
            x1, q1, s1 = act_i8(cols, 1, 5)
            out = torch.empty(per, dtype=torch.float32, device="cuda")
            scale1 = float(s1.item())
            it = [0]

            def one():
                jkb.bitlinear_i8(out, ws[it[0] % copies], q1, scale1)
                it[0] += 1

            us1 = maxr(_graph_time(one, max(launches, copies)))
            nbytes = (rows // world) * (cols // be) * bb + cols + per * 4
            gbs1 = nbytes * world / (us1 * 1e-6) / 1e9
            row = {"quant": qname, "rows": rows, "cols": cols,
                   "batch1_us": round(us1, 2),
                   "batch1_gbs": round(gbs1, 1),
                   "batch1_hbm_frac_per_gpu": round(gbs1 / world / peak, 4)}
            for w in ws[1:]:
                w.destroy()
            w = ws[0]
            xm, qm, sm = act_i8(cols, M, 6)
            ob = torch.empty(M * per, dtype=torch.float32, device="cuda")
            usb = maxr(_graph_time(lambda: jkb.bitlinear_i8_batch(ob, w, qm, sm), launches))
            row["batch128_bitlinear_us"] = round(usb, 2)
            row["batch128_bitlinear_tops"] = round(2.0 * M * rows * cols / (usb * 1e-6) / 1e12,
                                                   1)
            rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", quant, [per, cols], raws[0]),
                                                per, cols)
            act = jkb.QuantizedActQ8(M, cols)
            for exact, key in ((False, "batch128_tc"), (True, "batch128_tc_exact")):
                with jkb.gemm_exact(exact):
                    usg = maxr(_graph_time(
                        lambda: jkb.bitlinear_i8_gemm(ob, rw, qm, sm, M, act), launches))
                row[key + "_us"] = round(usg, 2)
                row[key + "_tops"] = round(2.0 * M * rows * cols / (usg * 1e-6) / 1e12, 1)
            res["shapes"].append(row)
            rw.destroy()
            act.destroy()
            w.destroy()
            del ob, xm, qm, sm
        # the FFN chain (each rank runs the whole chain)
        wg = jkb.Weight(jkb.TensorView("gate", quant, [F, H], synth_ternary(quant, F, H, 91)), F, H)
        wu = jkb.Weight(jkb.TensorView("up", quant, [F, H], synth_ternary(quant, F, H, 92)), F, H)
        wd = jkb.Weight(jkb.TensorView("down", quant, [H, F], synth_ternary(quant, H, F, 93)), H, F)
        raws = {"gate": (F, H, 91), "up": (F, H, 92), "down": (H, F, 93)}
        rep = tuple(jkb.RepackedWeight.from_tensor(
            jkb.TensorView(n, quant, [r, c], synth_ternary(quant, r, c, sd)), r, c)
            for n, (r, c, sd) in raws.items())
        for m in (1, M):
            ffn = jkb.BitNetFFN(wg, wu, wd, norm[H], norm[F], 1e-5, m,
                                repacked=rep if m >= 32 else None)
            x = torch.randn(m * H, generator=torch.Generator().manual_seed(8)).cuda()
            out = torch.empty(m * H, dtype=torch.float32, device="cuda")
            us = maxr(_graph_time(lambda: ffn.forward(out, x, m), launches))
            res[f"ffn_{qname}_m{m}_us"] = round(us, 2)
            ffn.destroy()
        for w in (wg, wu, wd) + rep:
            w.destroy()
    torch.cuda.empty_cache()
    return res


def int8_peak_tops(launches=10):
    """cuBLAS int8 GEMM throughput (torch._int_mm, 8192^3) on this GPU: the int8 tensor-core
    roofline denominator (MEASURED_PEAKS.json has none)."""
    import torch
    a = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device="cuda").t()
    us = _graph_time(lambda: torch._int_mm(a, b), launches)
    del a, b
    return 2.0 * 8192 ** 3 / (us * 1e-6) / 1e12


def run_prefill_gemm(world, rank, launches=10):
    """the repacked Q8_0 x Q8_0 prefill GEMM at M in {512, 2048} tokens for
    4096 -> 14336 and 14336 -> 4096, output rows sharded over the ranks. Per shape, `launches`
    back-to-back GEMMs (weight copies rotating so every launch reads more than the L2 holds) in
    a CUDA graph, timed with CUDA events, max over ranks; reported for the default (fused
    multiply-add) and the bit-exact epilogue. Activations are quantized once per shape
    (QuantizedActQ8), outside the timed region."""
    import torch
    import torch.distributed as dist
    import jkb200 as jkb

    res = {"shapes": [], "note": "tcgen05 int8 MMA + per-32-group f32 scale epilogue"}
    tot_ops = {False: 0.0, True: 0.0}
    tot_us = {False: 0.0, True: 0.0}
    for m, n, k in PREFILL:
        per = n // world
        raw = synth_matrix(Q8_0, n, k, 4243 + n, rank * per, (rank + 1) * per)
        nbytes = per * (k // 32) * 34
        copies = max(2, -(-300_000_000 // nbytes))
        ws = [jkb.RepackedWeight.from_tensor(jkb.TensorView("w", Q8_0, [per, k], raw), per, k)
              for _ in range(copies)]
        x = torch.randn(m * k, generator=torch.Generator().manual_seed(2)).cuda()
        act = jkb.QuantizedActQ8.quantize(x, m, k)
        out = torch.empty(m * per, dtype=torch.float32, device="cuda")
        row = {"m": m, "n": n, "k": k}
        for exact in (False, True):
            it = [0]

            def one():
                ws[it[0] % copies].gemm(out, act)
                it[0] += 1

            with jkb.gemm_exact(exact):
                us = _graph_time(one, launches)
            if world > 1:
                t = torch.tensor([us], device="cuda")
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                us = float(t.item())
            ops = 2.0 * m * n * k
            row["exact_tops" if exact else "tops"] = round(ops / (us * 1e-6) / 1e12, 1)
            row["exact_us" if exact else "us"] = round(us, 2)
            tot_ops[exact] += ops
            tot_us[exact] += us
        res["shapes"].append(row)
        for w in ws:
            w.destroy()
        del act, out, x
        torch.cuda.empty_cache()
    # Q4_K_M (min terms) and Q6_K (16-element groups) weights on one shape each, for reference
    # (not part of configs[2])
    m, n, k = 2048, 14336, 4096
    per = n // world
    x = torch.randn(m * k, generator=torch.Generator().manual_seed(3)).cuda()
    act = jkb.QuantizedActQ8.quantize(x, m, k)
    out = torch.empty(m * per, dtype=torch.float32, device="cuda")
    for key, quant in (("q4_k_m", Q4_K), ("q6_k", Q6_K)):
        raw = synth_matrix(quant, n, k, 4250, rank * per, (rank + 1) * per)
        w = jkb.RepackedWeight.from_tensor(jkb.TensorView(key, quant, [per, k], raw), per, k)
        us = _graph_time(lambda: w.gemm(out, act), launches)
        if world > 1:
            t = torch.tensor([us], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            us = float(t.item())
        res[key] = {"m": m, "n": n, "k": k, "us": round(us, 2),
                    "tops": round(2.0 * m * n * k / (us * 1e-6) / 1e12, 1)}
        w.destroy()
    # the same Q4_K_M weights as a PackedNibbleMatrix: 4-bit codes on the device (the GGUF
    # bytes), expanded to int8 in shared memory by the kernel's converter warps
    raw = synth_matrix(Q4_K, n, k, 4250, rank * per, (rank + 1) * per)
    nm = jkb.PackedNibbleMatrix.from_tensor(jkb.TensorView("nibble", Q4_K, [k, per], raw), per, k)
    us = _graph_time(lambda: nm.gemm(out, act), launches)
    if world > 1:
        t = torch.tensor([us], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t.item())
    res["nibble_q4_k_m"] = {"m": m, "n": n, "k": k, "us": round(us, 2),
                            "tops": round(2.0 * m * n * k / (us * 1e-6) / 1e12, 1),
                            "device_bytes": nm.packed_bytes(),
                            "i8_repacked_device_bytes": per * k + 2 * per * (k // 32) * 4}
    nm.destroy()
    del act, out, x
    res["tops"] = round(tot_ops[False] / (tot_us[False] * 1e-6) / 1e12, 1)
    res["exact_tops"] = round(tot_ops[True] / (tot_us[True] * 1e-6) / 1e12, 1)
    peak = int8_peak_tops()
    if world > 1:
        t = torch.tensor([peak], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        peak = float(t.item()) * world
    res["roofline"] = {"bound": "tensor", "achieved": res["tops"], "peak": round(peak, 1),
                       "unit": "TOPS", "frac": round(res["tops"] / peak, 4),
                       "peak_source": "measured in this run: cuBLAS int8 (torch._int_mm 8192^3)"
                                      + (f" x {world} GPUs" if world > 1 else "")}
    return res


def run_kernel_case(args):
    """One GEMV shape (the single-kernel case the ncu captures in profiles/ use). The weight
    exists in enough copies to exceed 2x the L2 size; `--launches` back-to-back launches over
    rotating copies are captured in a CUDA graph and the replay is timed with CUDA events.
    Under ncu, the eager warm-up launches come first (use -s to skip them)."""
    import torch
    import jkb200 as jkb

    quant = {"q4_k": Q4_K, "q6_k": Q6_K, "q8_0": Q8_0}[args.kernel]
    rows, cols = args.rows, args.cols
    nbytes = algorithmic_bytes(quant, rows, cols)
    copies = max(1, min(args.launches, -(-256_000_000 // nbytes)))
    raw = synth_matrix(quant, rows, cols, 4242)
    ws = [jkb.Weight(jkb.TensorView(args.kernel, quant, [rows, cols], raw), rows, cols)
          for _ in range(copies)]
    x = torch.randn(cols, generator=torch.Generator().manual_seed(1)).cuda()
    if not args.unfused:
        xq = x  # f32 input, quantized inside the GEMV launch
        fn = {Q8_0: jkb.vec_dot_q8_0_rvv, Q4_K: jkb.vec_dot_q4_k_m_rvv,
              Q6_K: jkb.vec_dot_q6_k_rvv}[quant]
    elif quant == Q8_0:
        xq = jkb.empty_q8_0_blocks(cols // 32)
        jkb.quantize_row_q8_0(x, xq)
        fn = jkb.gemv_q8_0_q8_0
    else:
        xq = jkb.empty_q8_k_blocks(cols // 256)
        jkb.quantize_row_q8_k(x, xq)
        fn = jkb.gemv_q4_k_q8_k if quant == Q4_K else jkb.gemv_q6_k_q8_k
    out = torch.empty(rows, dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for i in range(3):
            fn(out, ws[i % copies], xq)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(args.launches):
                fn(out, ws[i % copies], xq)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        g.replay()
        e1.record(s)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.launches
    print(json.dumps({"kernel": args.kernel, "fused": not args.unfused, "rows": rows,
                      "cols": cols, "copies": copies,
                      "us_per_launch": round(ms * 1e3, 3),
                      "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1)}))


def _graph_time(fn, launches, warm=3):
    """us per call of fn() over a CUDA graph of `launches` back-to-back calls."""
    import torch
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(launches):
                fn()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        g.replay()
        e1.record(s)
        torch.cuda.synchronize()
    return e0.elapsed_time(e1) / launches * 1e3


def run_gemm_case(args):
    """The repacked GEMM (BASELINE configs[2] kind) with Q8_0 (--kernel gemm_q8_0), Q4_K_M
    (gemm_q4_k) or Q6_K (gemm_q6_k) weights, or the compact nibble GEMM on Q4_K_M weights
    (gemm_nib_q4_k, PackedNibbleMatrix): M tokens x --rows x --cols, activations quantized once
    (QuantizedActQ8), `--launches` GEMMs timed in a CUDA graph."""
    import torch
    import jkb200 as jkb

    M, N, K = args.m, args.rows, args.cols
    # the formats without a quantizer in this file: seeded random bytes (GEMM time does not
    # depend on the values; non-finite f16 scales decode to 0 as in the reference)
    raw_fmt = {"gemm_q4_1": (3, 32, 20), "gemm_q5_1": (7, 32, 24), "gemm_iq4_nl": (20, 32, 18),
               "gemm_q2_k": (10, 256, 84), "gemm_q3_k": (11, 256, 110)}
    if args.kernel in raw_fmt:
        quant, be, bb = raw_fmt[args.kernel]
        raw = np.random.default_rng(4243).integers(0, 256, N * (K // be) * bb, dtype=np.uint8)
    else:
        quant = {"gemm_q4_k": Q4_K, "gemm_q6_k": Q6_K, "gemm_nib_q4_k": Q4_K}.get(args.kernel,
                                                                                   Q8_0)
        raw = synth_matrix(quant, N, K, 4243)
    if args.kernel == "gemm_nib_q4_k":
        rw = jkb.PackedNibbleMatrix.from_tensor(jkb.TensorView("w", quant, [N, K], raw), N, K)
    else:
        rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", quant, [N, K], raw), N, K)
    x = torch.randn(M * K, generator=torch.Generator().manual_seed(2)).cuda()
    act = jkb.QuantizedActQ8.quantize(x, M, K)
    out = torch.empty(M * N, dtype=torch.float32, device="cuda")
    with jkb.gemm_exact(args.exact):
        us = _graph_time(lambda: rw.gemm(out, act), args.launches)
    print(json.dumps({"kernel": args.kernel, "m": M, "rows": N, "cols": K, "exact": args.exact,
                      "us_per_launch": round(us, 2),
                      "tops": round(2.0 * M * N * K / (us * 1e-6) / 1e12, 2)}))


def run_bitlinear_case(args):
    """The tensor-core BitLinear (bitlinear_i8_gemm) on TQ2_0 weights: M tokens x --rows x
    --cols, i8 activations from the SubLN quantizer, `--launches` calls timed in a CUDA graph
    (the profiling case of the BitNet section)."""
    import torch
    import jkb200 as jkb

    M, N, K = args.m, args.rows, args.cols
    raw = synth_ternary(TQ2_0, N, K, 77)
    rw = jkb.RepackedWeight.from_tensor(jkb.TensorView("w", TQ2_0, [N, K], raw), N, K)
    x = torch.randn(M * K, generator=torch.Generator().manual_seed(6)).cuda()
    q = torch.empty(M * K, dtype=torch.int8, device="cuda")
    sc = torch.empty(M, dtype=torch.float32, device="cuda")
    jkb.subln_quantize_absmax_i8_rows(q, x, torch.ones(K, device="cuda"), M, K, 1e-5, sc)
    act = jkb.QuantizedActQ8(M, K)
    out = torch.empty(M * N, dtype=torch.float32, device="cuda")
    us = _graph_time(lambda: jkb.bitlinear_i8_gemm(out, rw, q, sc, M, act), args.launches)
    print(json.dumps({"kernel": "bitlinear_tc", "m": M, "rows": N, "cols": K,
                      "us_per_call": round(us, 2),
                      "tops": round(2.0 * M * N * K / (us * 1e-6) / 1e12, 2)}))


def run_bitlinear_gemv_case(args):
    """bitlinear_i8 at batch 1 on TQ2_0 (--kernel bitlinear) or I2_S (bitlinear_i2s) weights,
    --rows x --cols, i8 activation from the SubLN quantizer, weight copies rotating past 2x the
    L2, `--launches` calls in a CUDA graph (the profiling case of the BitNet batch-1 path)."""
    import torch
    import jkb200 as jkb

    quant = I2_S if args.kernel == "bitlinear_i2s" else TQ2_0
    N, K = args.rows, args.cols
    be, bb = BLOCK[quant]
    nbytes = N * (K // be) * bb + K + 4 * N
    copies = max(1, min(128, -(-260_000_000 // nbytes)))
    raw = synth_ternary(quant, N, K, 77)
    ws = [jkb.Weight(jkb.TensorView("w", quant, [N, K], raw), N, K) for _ in range(copies)]
    x = torch.randn(K, generator=torch.Generator().manual_seed(6)).cuda()
    q = torch.empty(K, dtype=torch.int8, device="cuda")
    sc = torch.empty(1, dtype=torch.float32, device="cuda")
    jkb.subln_quantize_absmax_i8_rows(q, x, torch.ones(K, device="cuda"), 1, K, 1e-5, sc)
    scale = float(sc.item())
    out = torch.empty(N, dtype=torch.float32, device="cuda")
    it = [0]

    def one():
        jkb.bitlinear_i8(out, ws[it[0] % copies], q, scale)
        it[0] += 1

    us = _graph_time(one, max(args.launches, copies) if args.launches > 3 else args.launches)
    print(json.dumps({"kernel": args.kernel, "rows": N, "cols": K, "copies": copies,
                      "us_per_launch": round(us, 3), "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}))


def run_int8_peak(args):
    """cuBLAS int8 GEMM throughput through torch._int_mm (the int8 roofline denominator)."""
    import torch
    res = {"kernel": "int8_peak"}
    for name, (M, N, K) in (("8192^3", (8192, 8192, 8192)),
                            ("gemm_shape", (args.m, args.rows, args.cols))):
        a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
        b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda").t()
        us = _graph_time(lambda: torch._int_mm(a, b), args.launches)
        res[name] = {"m": M, "n": N, "k": K, "us": round(us, 2),
                     "tops": round(2.0 * M * N * K / (us * 1e-6) / 1e12, 1)}
    print(json.dumps(res))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="jkb", choices=["jkb", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--collective", choices=["push", "peer", "nccl"], default="peer",
                    help="N > 1: collect the output-row shards by pushing them to the peers "
                         "from the GEMV kernels over NVLink plus one signal kernel (push), by "
                         "this library's one-kernel all-gather over NVLink peer memory (peer) "
                         "or by one NCCL all-gather per step (nccl)"),
    ap.add_argument("--prequant", default="f",
                    help="comma list of activation streams (x, attn, h, a, f) quantized by their "
                         "own quantize_row_q8_k launch ahead of pre-quantized GEMVs instead of "
                         "inside the f32-input GEMV launch (default: f, the lm_head input)")
    ap.add_argument("--workload", choices=sorted(DECODE_SETS), default="8b",
                    help="the decode GEMV set of the headline: 8b (BASELINE configs[1]) or 70b "
                         "(configs[4]); the other set is reported as a section")
    ap.add_argument("--no-sections", action="store_true",
                    help="leave out the other decode set, the batch-16 70B step and the Q4_0 "
                         "GEMV (configs[0]) sections")
    ap.add_argument("--no-gemm", action="store_true",
                    help="leave out the prefill GEMM section (BASELINE configs[2])")
    ap.add_argument("--no-bitnet", action="store_true",
                    help="leave out the BitNet BitLinear section (BASELINE configs[3])")
    ap.add_argument("--m", type=int, default=2048, help="tokens of --kernel gemm_q8_0 / int8_peak")
    ap.add_argument("--kernel", choices=["q4_k", "q6_k", "q8_0", "gemm_q8_0", "gemm_q4_k",
                                         "gemm_q6_k", "gemm_nib_q4_k", "gemm_q4_1", "gemm_q5_1",
                                         "gemm_iq4_nl", "gemm_q2_k", "gemm_q3_k", "int8_peak",
                                         "bitlinear_tc", "bitlinear", "bitlinear_i2s",
                                         "per_shape"],
                    help="run one GEMV shape (profiling case) instead of the benchmark")
    ap.add_argument("--rows", type=int, default=65536)
    ap.add_argument("--cols", type=int, default=4096)
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--exact", action="store_true",
                    help="--kernel gemm_*: the bit-exact epilogue (gemm_exact) instead of the "
                         "default fused multiply-add")
    ap.add_argument("--unfused", action="store_true",
                    help="quantize each activation in its own launch and run one GEMV launch "
                         "per matrix (jkb_quantize_row_q8_k + jkb_gemv_*) instead of the "
                         "f32-input vec_dot_*_rvv / grouped launches")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.kernel == "bitlinear_tc":
        run_bitlinear_case(args)
    elif args.kernel in ("bitlinear", "bitlinear_i2s"):
        run_bitlinear_gemv_case(args)
    elif args.kernel == "per_shape":  # each group of the --workload decode set on its own
        import torch
        import jkb200 as jkb

        torch.cuda.set_device(0)
        print(json.dumps(run_decode_shapes(jkb, DECODE_SETS[args.workload], 1, 0)))
    elif args.kernel and args.kernel.startswith("gemm_"):
        run_gemm_case(args)
    elif args.kernel == "int8_peak":
        run_int8_peak(args)
    elif args.kernel:
        run_kernel_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
