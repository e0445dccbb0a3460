#!/usr/bin/env python
"""Decode benchmark: tokens/s of the Llama-2-70B-shaped Q4_K model (BASELINE.json
config 4) on B200, through libchatnet_cuda.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--config 4|1]
    python bench.py --config 3 ...           # prefill: 512 tokens through one 7B layer
    python bench.py --config 0|2 ...         # Q-matvec HBM GB/s (one JSON line per shape/batch)
    python bench.py --impl reference ...     # the reference's CPU algorithm (oracle port)

A step is one decode step of `batch` sequences (each at position 2047 of a
2048-token fp16 KV cache filled with seeded N(0,1) values), all 80 layers
plus lm_head and argmax.  Weights (38.5 GB of Q4_K blocks) and the KV cache
are generated on the device from the seeded generator (synthetic data of
the config's shapes and distributions).  Inputs are far larger than L2.

Printed JSON line (rank 0):
  value      tokens/s of the whole job with inputs resident in HBM
             (CUDA-graph steps timed with CUDA events, max over ranks)
  e2e        the same through cn_llama_decode with host buffers: token ids
             and positions copied in, logits and argmax copied out per step
  roofline   the dominant kernel (the fused Q4_K dequant-GEMV of the FFN
             gate and up projections, 57344 x 8192 as the one launch the
             step runs) timed alone on the context stream, cycling through
             the 80 layers' matrices: algorithmic bytes per launch / mean
             launch time
  cpu_baseline  the oracle port of the reference's C# CPU path timed on the
             host's cores over the whole step (CpuSample)
With --gpus N > 1 the ranks run the model tensor-parallel (default; the
same sequences, strong scaling) or as independent replicas (--parallel
replicas, weak scaling).

--config 3 (prefill): a step is one pass of 512 tokens' hidden states through
one Llama-2-7B-shaped Q4_0 layer (cn_llama_prefill_hidden_dev); `value` is
tokens/s, `e2e` adds the copy of the 8 MiB input from pinned host memory and
of the output back, and the roofline is the gate/up matmul's TFLOP/s against
the measured dense bf16 peak.  With N > 1 the ranks run replicas.

--config 0 / --config 2 (Q-matvec GB/s): a step is one fused dequant-GEMV
(x-prep + GEMV, the work of cn_matvec_dev) of config 0's Q4_0 5632x2048 matrix
or of each config-2 shape (Q4_K 4096x4096, 11008x4096, 4096x11008; Q6_K
32000x4096) at batches 1, 4, 16 and 32.  The calls cycle through enough
distinct seeded copies of the matrix to fill twice the 126 MB L2 (cold L2)
and run from one CUDA graph of >= 100 calls (no host gaps); `value` is the
algorithmic bytes (weights + x + y) per call over the median of the
replays' per-call times, `e2e` the same through cn_matvec with host buffers
(x in, y out, synchronous), and `cpu_baseline` the oracle's MatVecMul port
on the same matrix on all host cores.
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
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s"
CPU_SAMPLE_LAYERS = 2


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per step (default 1; --config 2: all of 1, 4, 16, 32 unless given)")
    ap.add_argument("--config", type=int, default=4, choices=(0, 1, 2, 3, 4))
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--parallel", default="tp", choices=("tp", "replicas"),
                    help="N > 1: tensor parallelism over the N GPUs (default), or N independent replicas")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=None,
                    help="decode configs: build only the first N layers (small cases for ncu captures; "
                         "not a bench line)")
    ap.add_argument("--gemv", default=None, metavar="TYPE:ROWSxCOLS:BATCH",
                    help="kernel mode: run one fused dequant-GEMV (e.g. q4_k:28672x8192:1) "
                         "--steps times on one GPU and print its mean time (ncu captures)")
    ap.add_argument("--nvtx-step", action="store_true",
                    help="after warm-up run one step inside the NVTX range 'timed_step' and exit "
                         "(for ncu --nvtx --nvtx-include timed_step/ launch lists)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# clocks: nvidia-smi sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak_tflops() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured burst"
        except (KeyError, ValueError):
            pass
    return 1590.0, "fallback"


def measured_peak_gbs() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return 6650.0, "fallback"


def gemv_kernel_name(config: int, batch: int) -> str:
    """The GEMV kernel family the library runs for the config's projections
    (Q4_K decode at batch 1..16: the integer mma.sync kernel unless the
    environment selects another; Q4_0 and larger batches: the fp16 one)."""
    choice = os.environ.get("CHATNET_GEMV", "i8")
    if config == 4 and batch <= 16 and choice not in ("tc", "mma"):
        return "gemv_i8_q4k"
    if config == 4 and batch <= 5 and choice == "tc":
        return "gemv_tc_q4k"
    return "gemv_q4_k" if config == 4 else "gemv_q4_0"


def gemv_dtype(config: int, batch: int) -> str:
    name = gemv_kernel_name(config, batch)
    if name in ("gemv_i8_q4k", "gemv_tc_q4k"):
        return "q4_k x int22 activation digits (int8 mma, exact) -> s32 -> f32"
    return ("q4_k" if config == 4 else "q4_0") + " x fp16(hi+lo) -> f32"


def committed_traffic(kernel_key: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get(kernel_key)
        except ValueError:
            return None
    return None


# ---------------------------------------------------------------------------
# CPU baseline: the oracle port of the reference's C# path
# ---------------------------------------------------------------------------
class CpuSample:
    """The oracle port of the reference's C# CPU path, one token through every
    layer and lm_head, timed on the host's cores (the oracle's row split over
    all threads, as Parallel.For does).  The tensors come from the oracle's own
    generator, so this leg never loads libchatnet_cuda.  A model too large for
    host memory (config 4: 38.5 GB) keeps the seeded weights of its first
    `sample_layers` layers and runs layer l with those of layer
    l % sample_layers: each layer still streams its 481 MB of weights from
    DRAM (far above the host's caches), so the step costs what the full model's
    would.  Batches cost batch x one sequence (the reference has no batching)."""

    def __init__(self, dc_full, batch: int):
        import ctypes as C
        from chatnet_b200 import configs as cf
        from chatnet_b200.llama import tensor_names
        from tests import _oracle
        self.C, self._o = C, _oracle
        self.full, self.batch = dc_full, batch
        self.orc = orc = _oracle.load()
        L = dc_full.model.n_layers
        self.sample_layers = L if L <= 22 else CPU_SAMPLE_LAYERS
        dc = cf.with_layers(dc_full, self.sample_layers)
        self.dc = dc
        host = _oracle.host_tensors(orc, dc)
        names = tensor_names(self.sample_layers)
        types = [cf.tensor_type(dc, n) for n in names]
        k, v = _oracle.host_kv(orc, dc, 0)
        self.ol = _oracle.OracleLlama(orc, dc.model, host, types, names, k, v)
        self.x0 = orc.dequantize(types[0], host["token_embd.weight"][_oracle.token(orc, dc, 0)],
                                 dc.model.dim)
        self.logits = np.empty(dc.model.vocab, np.float32)

    def run_once(self) -> float:
        """Seconds for one step of `batch` sequences."""
        C, fp, ol, orc = self.C, self._o.fp, self.ol, self.orc
        x = self.x0.copy()
        S, L = self.sample_layers, self.full.model.n_layers
        rc = 0
        t0 = time.perf_counter()
        for l0 in range(0, L, S):
            rc |= orc.lib.or_llama_layers(C.byref(ol.cfg), ol.ptrs, ol.types, ol.k.ctypes.data,
                                          ol.v.ctypes.data, fp(x), self.dc.decode_pos, 0, min(S, L - l0), 0)
        rc |= orc.lib.or_llama_head(C.byref(ol.cfg), ol.ptrs, ol.types, fp(x), fp(self.logits), 0)
        t1 = time.perf_counter()
        assert rc == 0
        return self.batch * (t1 - t0)

    def describe(self, reps: int) -> str:
        m = self.full.model
        reuse = ("" if self.sample_layers == m.n_layers else
                 f" (weights of {self.sample_layers} seeded layers reused cyclically; each layer's "
                 f"weights exceed the host caches)")
        per = "" if self.batch == 1 else f", x{self.batch} sequences (batch = {self.batch} x one sequence)"
        return (f"all {m.n_layers} layers + lm_head per token{reuse}, {m.dim}-dim, position "
                f"{self.dc.decode_pos}{per}, median of {reps} runs, oracle port on {os.cpu_count()} host threads")


# ---------------------------------------------------------------------------
# configs 0 and 2: Q-matvec GB/s
# ---------------------------------------------------------------------------
MATVEC_CASES = {
    0: [("q4_0", 5632, 2048, (1,))],
    2: [("q4_k", 4096, 4096, (1, 4, 16, 32)), ("q4_k", 11008, 4096, (1, 4, 16, 32)),
        ("q4_k", 4096, 11008, (1, 4, 16, 32)), ("q6_k", 32000, 4096, (1, 4, 16, 32))],
}
L2_BYTES = 126 * 2**20


def matvec_dtype(name: str, batch: int) -> str:
    if name == "q4_k" and batch <= 8 and os.environ.get("CHATNET_GEMV", "i8") not in ("tc", "mma"):
        return "q4_k x int22 activation digits (int8 mma, exact) -> s32 -> f32"
    return f"{name} x fp16(hi+lo) -> f32"


def matvec_bytes(type_bytes_per_row: int, rows: int, cols: int, batch: int) -> int:
    """Algorithmic bytes of one call: the weight blocks once, x and y once."""
    return type_bytes_per_row * rows + 4 * batch * (rows + cols)


def matvec_main(a, world: int, rank: int, local: int) -> int:
    """One JSON line per (shape, batch) of config 0 or 2."""
    from chatnet_b200.llama import LlamaConfig  # noqa: F401  (package import only; no library load)
    tmap = {"q4_0": 2, "q4_k": 12, "q6_k": 14}
    cases = [(nm, r, c, b) for nm, r, c, bs in MATVEC_CASES[a.config] for b in bs
             if a.batch is None or b == a.batch]
    steps = max(a.steps, 1)
    reps = max(5, min(steps, 20))

    def seed_name(nm, r, c, i):
        return f"cfg{a.config}.{nm}.{r}x{c}.copy{i}"

    def cpu_time(orc, nm, r, c, b, seconds=3.0):
        """Median seconds per call of the oracle's MatVecMul port (all host threads)."""
        t = tmap[nm]
        W = orc.synth_fill(t, r, c, orc.synth_seed(a.config, seed_name(nm, r, c, 0)))
        x = orc.synth_fill(0, b, c, orc.synth_seed(a.config, f"cfg{a.config}.x.{c}.{b}"))
        times, t_end = [], time.perf_counter() + seconds
        while len(times) < 3 or (time.perf_counter() < t_end and len(times) < 50):
            t0 = time.perf_counter()
            orc.matvec(t, W, x, r)
            times.append(time.perf_counter() - t0)
        return statistics.median(times), len(times)

    workload0 = {"config_id": a.config, "parallelism": "single GPU" if world == 1 else f"replicas x{world}",
                 "l2": "cold: calls cycle through distinct copies of the matrix filling 2x the 126 MB L2"}
    if a.impl == "reference":
        if rank != 0:
            return 0
        from tests import _oracle
        orc = _oracle.load()
        for nm, r, c, b in cases:
            rb = int(orc.lib.or_byte_size(tmap[nm], c))
            nbytes = matvec_bytes(rb, r, c, b)
            sec, n = cpu_time(orc, nm, r, c, b, seconds=max(2.0, 0.1 * (steps + a.warmup)))
            val = nbytes / sec / 1e9
            wl = dict(workload0, workload=f"{nm} {r}x{c} batch {b}", rows=r, cols=c, batch=b)
            print(json.dumps({
                "metric": "Q-matvec GB/s", "value": val, "unit": "GB/s", "n_gpus": 0, "steps": n,
                "warmup": a.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference", "config": wl,
                "cpu_baseline": {"value": val, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                                 "sample": f"{n} calls of the oracle's MatVecMul port, median"},
                "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
                flush=True)
        return 0

    import ctypes as C
    import torch
    import chatnet_b200 as cn
    from chatnet_b200 import _native as N
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    ctx = cn.Context(local)
    ext = torch.cuda.ExternalStream(ctx.stream)
    peak, peak_kind = measured_peak_gbs()
    orc = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        from tests import _oracle
        orc = _oracle.load()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for nm, r, c, b in cases:
        t = tmap[nm]
        rb = cn.byte_size(t, c)
        nbytes = matvec_bytes(rb, r, c, b)
        copies = max(2, -(-2 * L2_BYTES // (rb * r)))
        Ws = [ctx.synth(t, r, c, cn.synth_seed(a.config, seed_name(nm, r, c, i))) for i in range(copies)]
        x = torch.from_numpy(cn.synth_fill(cn.TYPE_F32, b, c, cn.synth_seed(a.config, f"cfg{a.config}.x.{c}.{b}")))
        xd = x.to(f"cuda:{local}")
        yd = torch.empty(b, r, device=f"cuda:{local}")
        torch.cuda.synchronize()
        launches = -(-max(100, copies) // copies) * copies
        handles = (C.c_void_p * copies)(*[w.handle for w in Ws])
        us = np.zeros(reps, np.float32)
        kpl = C.c_int(0)
        for _ in range(max(1, a.warmup // 5)):  # warm-up replays (the call itself warms up twice)
            N.check(N.lib().cn_time_matvec(ctx.handle, handles, copies, xd.data_ptr(), yd.data_ptr(), b,
                                           launches, 1, us.ctypes.data_as(C.POINTER(C.c_float)),
                                           C.byref(kpl)), "cn_time_matvec")
        if dist is not None:
            dist.barrier()
        clk = ClockSampler(local)
        clk.start()
        time.sleep(0.2)
        N.check(N.lib().cn_time_matvec(ctx.handle, handles, copies, xd.data_ptr(), yd.data_ptr(), b, launches,
                                       reps, us.ctypes.data_as(C.POINTER(C.c_float)), C.byref(kpl)),
                "cn_time_matvec")
        clocks = clk.stop()
        us_med = max_over_ranks(float(np.median(us)))
        value = world * nbytes / (us_med * 1e-6) / 1e9
        # end to end: cn_matvec with pinned host buffers (x in, y out, synchronous)
        xh = x.pin_memory()
        yh = torch.empty(b, r).pin_memory()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_e2e = max(steps, copies)
        xp = C.cast(xh.data_ptr(), C.POINTER(C.c_float))
        yp = C.cast(yh.data_ptr(), C.POINTER(C.c_float))
        for i in range(3):
            N.check(N.lib().cn_matvec(ctx.handle, Ws[i % copies].handle, xp, yp, b), "cn_matvec")
        e0.record(ext)
        for i in range(n_e2e):
            N.check(N.lib().cn_matvec(ctx.handle, Ws[i % copies].handle, xp, yp, b), "cn_matvec")
        e1.record(ext)
        e1.synchronize()
        us_e2e = max_over_ranks(e0.elapsed_time(e1) * 1e3 / n_e2e)
        assert torch.isfinite(yh).all()
        cpu = None
        if orc is not None:
            sec, n = cpu_time(orc, nm, r, c, b)
            cpu = {"value": nbytes / sec / 1e9, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                   "sample": f"{n} calls of the oracle's MatVecMul port on copy 0 of the matrix, median "
                             f"({sec * 1e3:.2f} ms per call)"}
        if rank == 0:
            wl = dict(workload0, workload=f"{nm} {r}x{c} batch {b}", rows=r, cols=c, batch=b,
                      weight_copies=copies, calls_per_graph=launches, replays=reps)
            achieved = nbytes / (us_med * 1e-6) / 1e9
            print(json.dumps({
                "metric": "Q-matvec GB/s", "value": value, "unit": "GB/s", "n_gpus": world, "steps": reps,
                "warmup": a.warmup, "ms_per_step": us_med * 1e-3, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": matvec_dtype(nm, b),
                "data": "synthetic (seeded generator, config shapes and distributions)", "config": wl,
                "e2e": {"value": nbytes / (us_e2e * 1e-6) / 1e9, "unit": "GB/s", "us_per_call": us_e2e,
                        "h2d_bytes_per_step": 4 * b * c, "d2h_bytes_per_step": 4 * b * r},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "traffic": committed_traffic(f"gemv_{nm}_{r}x{c}_b{b}"),
                             "kernel": f"x-prep + fused dequant-GEMV {nm} {r}x{c} batch {b}",
                             "us_per_launch": us_med, "bytes_per_launch": nbytes,
                             "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})"},
                "cpu_baseline": cpu, "gpu_launches": int(kpl.value) * launches * reps, "clocks": clocks}),
                flush=True)
        del xd, yd
        for w in Ws:
            w.free()
    ctx.close()
    if dist is not None:
        dist.destroy_process_group()
    return 0


def gemv_mode(a) -> int:
    """One GEMV, seeded synthetic weights, launched --steps times after --warmup."""
    import torch
    import chatnet_b200 as cn
    from chatnet_b200 import _native as N
    name, shape, batch = a.gemv.split(":")
    rows, cols = (int(v) for v in shape.split("x"))
    batch = int(batch)
    t = {"q4_0": cn.TYPE_Q4_0, "q4_k": cn.TYPE_Q4_K, "q6_k": cn.TYPE_Q6_K, "q8_0": cn.TYPE_Q8_0,
         "q5_k": cn.TYPE_Q5_K, "q4_1": cn.TYPE_Q4_1, "q5_0": cn.TYPE_Q5_0, "q5_1": cn.TYPE_Q5_1}[name]
    ctx = cn.Context(0)
    # no seeded generator: seeded random blocks (block elements, bytes, has a
    # second fp16 field), fp16 scales (and minima) 0.01
    raw_fmt = {cn.TYPE_Q8_0: (32, 34, False), cn.TYPE_Q5_K: (256, 176, True), cn.TYPE_Q4_1: (32, 20, True),
               cn.TYPE_Q5_0: (32, 22, False), cn.TYPE_Q5_1: (32, 24, True)}
    if t in raw_fmt:
        blk, bpb, second = raw_fmt[t]
        raw = np.random.default_rng(cn.synth_seed(2, f"gemv.{name}.{rows}x{cols}")).integers(
            0, 256, size=(rows * cols // blk, bpb), dtype=np.uint8)
        raw[:, 0:2] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
        if second:
            raw[:, 2:4] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
        W = ctx.upload(raw.ravel(), t, rows, cols)
    else:
        W = ctx.synth(t, rows, cols, cn.synth_seed(2, f"gemv.{name}.{rows}x{cols}"))
    x = torch.from_numpy(cn.synth_fill(cn.TYPE_F32, batch, cols, cn.synth_seed(2, "gemv.x"))).cuda()
    y = torch.empty(batch, rows, device="cuda")
    ext = torch.cuda.ExternalStream(ctx.stream)

    def run():
        N.check(N.lib().cn_matvec_dev(ctx.handle, t, W.device_ptr, rows, cols, x.data_ptr(),
                                      y.data_ptr(), batch), "cn_matvec_dev")
    for _ in range(a.warmup):
        run()
    ctx.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    for _ in range(a.steps):
        run()
    e1.record(ext)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / a.steps
    nbytes = cn.byte_size(t, cols) * rows + 4 * batch * (rows + cols)
    print(json.dumps({"gemv": a.gemv, "us_per_call": us, "GBps_incl_prep": nbytes / us / 1e3,
                      "note": "warm L2 when the matrix fits in it; prep + GEMV launches"}))
    ctx.close()
    return 0


# ---------------------------------------------------------------------------
# config 3: prefill
# ---------------------------------------------------------------------------
PREFILL_FLOPS = 209.38e9  # projections 207.23 GFLOP + causal attention 2.15 GFLOP


class CpuPrefillSample:
    """The oracle port of the reference's CPU path for config 3: the first
    `n` prompt tokens through the layer one at a time (as ChatNet's prompt
    loop runs them), timed together."""

    def __init__(self, dc, n: int):
        from chatnet_b200 import configs as cf
        from chatnet_b200.llama import tensor_names
        from tests import _oracle
        self.n = n
        orc = _oracle.load()
        host = _oracle.host_tensors(orc, dc)  # the oracle's generator: no product library here
        names = tensor_names(dc.model.n_layers)
        types = [cf.tensor_type(dc, nm) for nm in names]
        m = dc.model
        k = np.zeros((m.n_layers * m.ctx_len, m.kv_dim), np.float32)
        self.ol = _oracle.OracleLlama(orc, m, host, types, names, k, k.copy())
        self.x = _oracle.prefill_x(orc, dc)

    def run_once(self) -> float:
        """Seconds per token."""
        t0 = time.perf_counter()
        for t in range(self.n):
            self.ol.layers(self.x[t], t)
        return (time.perf_counter() - t0) / self.n

    def describe(self, reps: int) -> str:
        return (f"prompt tokens 0..{self.n - 1} of 512 through the layer one at a time (attention "
                f"over <= {self.n} positions, so slightly cheaper per token than the full prompt), "
                f"median of {reps} runs, per-token time")


def prefill_main(a, world: int, rank: int, local: int, dc) -> int:
    n = dc.prefill
    m = dc.model
    workload = {"workload": dc.name, "config_id": 3, "tokens": n, "n_layers": m.n_layers, "dim": m.dim,
                "ffn": m.hidden_dim, "heads": f"{m.n_heads}/{m.n_kv_heads}", "head_dim": m.head_dim,
                "positions": f"0..{n - 1}", "weights": "Q4_0", "kv_cache": "fp32",
                "parallelism": "single GPU" if world == 1 else f"replicas x{world}",
                "l2": "weights 113.8 MB and activations re-read each step; L2 not flushed (a layer's "
                      "working set is about 200 MB, above the 126 MB L2)",
                "flops_per_step": PREFILL_FLOPS}
    if a.impl == "reference":
        if rank != 0:
            return 0
        cs = CpuPrefillSample(dc, 16)
        times = []
        for i in range(a.warmup + a.steps):
            t = cs.run_once()
            if i >= a.warmup:
                times.append(t)
        val = 1.0 / statistics.median(times)
        line = {"metric": "prefill tok/s", "value": val, "unit": "tok/s", "n_gpus": 0, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": n * 1e3 / val, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "impl": "reference", "config": workload,
                "cpu_baseline": {"value": val, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                                 "sample": cs.describe(a.steps)},
                "e2e": {"value": val, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    import chatnet_b200 as cn
    from chatnet_b200 import configs as cf
    from chatnet_b200.llama import CudaLlamaModel

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    ctx = cn.Context(local)
    ext = torch.cuda.ExternalStream(ctx.stream)
    tensors = cf.device_tensors(ctx, dc)
    model = CudaLlamaModel(ctx, m, tensors)
    xh = torch.from_numpy(cf.prefill_x(dc)).pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    xd = xh.to(f"cuda:{local}")
    od = torch.empty_like(xd)
    torch.cuda.synchronize()

    def step():
        model.prefill_hidden_dev(xd.data_ptr(), n, 0, od.data_ptr())

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        ctx.synchronize()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(a.warmup, 3)):
        step()
    ctx.synchronize()
    if a.nvtx_step:
        torch.cuda.nvtx.range_push("timed_step")
        step()
        ctx.synchronize()
        torch.cuda.nvtx.range_pop()
        print(json.dumps({"nvtx_step": True, "kernels": model.prefill_kernels()}), flush=True)
        return 0

    barrier()
    clk = ClockSampler(local)
    clk.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    for _ in range(a.steps):
        step()
    e1.record(ext)
    e1.synchronize()
    clocks = clk.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    value = world * n * 1000.0 / ms

    # the same passes at the two faster precisions (1: only the attention path
    # split, 0: every operand rounded to fp16 once), then back to the default
    ms_at = {}
    for prec in (1, 0):
        model.set_prefill_precision(prec)
        for _ in range(2):
            step()
        barrier()
        e0.record(ext)
        for _ in range(a.steps):
            step()
        e1.record(ext)
        e1.synchronize()
        ms_at[prec] = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    model.set_prefill_precision(2)

    # end to end: host activations in, host output back, every step
    barrier()
    e0.record(ext)
    for _ in range(a.steps):
        with torch.cuda.stream(ext):
            xd.copy_(xh, non_blocking=True)
        step()
        with torch.cuda.stream(ext):
            oh.copy_(od, non_blocking=True)
    e1.record(ext)
    e1.synchronize()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    e2e = world * n * 1000.0 / ms_e2e
    assert torch.isfinite(oh).all()

    # roofline: the gate/up matmul (the largest launch) timed alone
    us, flops = model.time_matmul(2, n, iters=20)
    peak, peak_kind = measured_peak_tflops()
    achieved = flops / (us * 1e-6) / 1e12
    us_by_group = {g: model.time_matmul(i, n, iters=20)[0] for i, g in enumerate(("qkv", "o", "gate_up", "down"))}
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cs = CpuPrefillSample(dc, 16)
        per_tok = statistics.median([cs.run_once() for _ in range(3)])
        cpu = {"value": 1.0 / per_tok, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
               "sample": cs.describe(3)}
    if rank == 0:
        line = {
            "metric": "prefill tok/s", "value": value, "unit": "tok/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": "q4_0 weights x activations on tcgen05 kind::f16 -> f32, every projection and the "
                     "attention's operands as exact hi+lo fp16 pairs (3 MMAs per k-step; precision 2, the default)",
            "other_precisions": {
                "1_attention_path_split": {"ms_per_step": ms_at[1], "tok_s": world * n * 1000.0 / ms_at[1]},
                "0_fp16_operands": {"ms_per_step": ms_at[0], "tok_s": world * n * 1000.0 / ms_at[0]},
                "note": "cn_llama_set_prefill_precision; the parity bar on trained-model-like weights needs 2"},
            "data": "synthetic (seeded generator, config shapes and distributions)", "config": workload,
            "layer_tflops": PREFILL_FLOPS / (ms * 1e-3) / 1e12,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": int(xh.numel() * 4),
                    "d2h_bytes_per_step": int(oh.numel() * 4)},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak,
                         "issued_frac": 3 * achieved / peak,
                         "note": "achieved = algorithmic FLOPs / time; at the default precision every k-step "
                                 "issues three MMAs (hi*hi, hi*lo, lo*hi), so the tensor pipe runs 3x the "
                                 "algorithmic FLOPs (issued_frac)",
                         "traffic": committed_traffic(f"matmul_q4_0_{2 * m.hidden_dim}x{m.dim}_m{n}"),
                         "kernel": f"matmul_q4_0_kernel gate/up {2 * m.hidden_dim}x{m.dim} M{n}",
                         "us_per_launch": us, "flops_per_launch": flops,
                         "us_per_launch_by_group": us_by_group,
                         "peak_source": f"MEASURED_PEAKS.json bf16_tflops ({peak_kind})"},
            "cpu_baseline": cpu,
            "gpu_launches": model.prefill_kernels() * a.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    ctx.synchronize()
    del xd, od, xh, oh  # torch's buffers go before the library's context
    torch.cuda.synchronize()
    model.close()
    for t in tensors:
        t.free()
    if dist is not None:
        dist.destroy_process_group()
    ctx.close()
    return 0


# ---------------------------------------------------------------------------
# tensor-parallel parity, checked before the timed run
# ---------------------------------------------------------------------------
def tp_parity(ctx, rank: int, world: int, dist, steps: int = 3) -> dict | None:
    """A 2-layer Q4_K model with shapes that shard over 2, 4 and 8 ranks
    (dim 2048, 32 query / 8 kv heads of 64, hidden 2048, vocab 512, fp16
    cache) runs tensor-parallel on the same ranks as the benchmark; rank 0
    compares the all-gathered logits of `steps` decode steps with the
    oracle's single-CPU Forward.  Returns the record for the JSON line (rank 0)."""
    import chatnet_b200 as cn
    from chatnet_b200 import configs as cf
    from chatnet_b200.llama import CudaLlamaModel, tensor_names
    dc = cf.with_layers(cf.CONFIGS[4], 2, 1)
    m = cf.replace(dc.model, dim=2048, hidden_dim=2048, n_heads=32, n_kv_heads=8, head_dim=64, vocab=512,
                   ctx_len=64, kv_f16=True)
    dc = cf.replace(dc, model=m, kv_filled=20, decode_pos=20)
    tp = cn.TensorParallel(ctx, rank, world, 1, m.dim, m.vocab)
    handles = [None] * world
    dist.all_gather_object(handles, tp.ipc_handle())
    tp.connect(handles)
    ts = cf.device_tensors(ctx, dc, rank=rank, size=world)
    model = CudaLlamaModel(ctx, m, ts, tp=tp)
    model.kv_synth(0, dc.kv_filled, *cf.kv_seeds(dc, 0))
    model.prepare(1)
    dist.barrier()
    got = []
    for st in range(steps):
        lg, am = model.decode([cf.token(dc, 0, st)], [dc.decode_pos + st])
        got.append((lg[0].copy(), int(am[0])))
    model.close()
    for t in ts:
        t.free()
    dist.barrier()  # no rank unmaps its exchange buffer while a peer may still store into it
    tp.close()
    if rank != 0:
        return None
    from tests import _oracle  # the checker
    from tests.parity import rel_err
    orc = _oracle.load()
    host = _oracle.host_tensors(orc, dc)
    names = tensor_names(m.n_layers)
    k, v = _oracle.host_kv(orc, dc, 0)
    ol = _oracle.OracleLlama(orc, m, host, [cf.tensor_type(dc, n) for n in names], names, k, v)
    errs, same = [], True
    for st, (lg, am) in enumerate(got):
        ref = ol.forward([_oracle.token(orc, dc, 0, st)], dc.decode_pos + st)
        errs.append(rel_err(lg, ref))
        same = same and am == int(np.argmax(ref))
    return {"max_rel_err": max(errs), "argmax_equal": same, "ranks": world, "steps": steps,
            "model": "2-layer Q4_K, dim 2048, 32/8 heads x 64, hidden 2048, vocab 512, fp16 KV",
            "tolerance": 1e-3}


def main():
    a = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.gemv:
        return gemv_mode(a)
    if a.config in (0, 2):
        return matvec_main(a, world, rank, local)
    if a.batch is None:
        a.batch = 1
    from chatnet_b200 import configs as cf
    dc = cf.with_batch(cf.CONFIGS[a.config], a.batch)
    if a.layers and a.config in (1, 4):
        dc = cf.with_layers(dc, a.layers, a.batch)
    workload = {"workload": dc.name, "config_id": a.config, "batch": a.batch,
                "n_layers": dc.model.n_layers, "dim": dc.model.dim, "ffn": dc.model.hidden_dim,
                "heads": f"{dc.model.n_heads}/{dc.model.n_kv_heads}", "head_dim": dc.model.head_dim,
                "vocab": dc.model.vocab, "ctx": dc.model.ctx_len, "position": dc.decode_pos,
                "weights": "Q4_K" if a.config == 4 else "Q4_0",
                "kv_cache": "fp16" if dc.model.kv_f16 else "fp32",
                "parallelism": ("single GPU" if world == 1 else
                                f"tp{world} (row/column-sharded projections, exchange fused into the "
                                f"GEMV epilogue over NVLink)" if a.parallel == "tp" else f"replicas x{world}"),
                "l2": "inputs larger than L2 (weights 38.5 GB)" if a.config == 4 else
                      "inputs larger than L2 (weights 0.58 GB)"}

    if a.config == 3:
        return prefill_main(a, world, rank, local, dc)

    if a.impl == "reference":
        if rank != 0:
            return 0
        cs = CpuSample(dc, a.batch)
        times = []
        for i in range(a.warmup + a.steps):
            t = cs.run_once()
            if i >= a.warmup:
                times.append(t)
        sample = cs.describe(a.steps)
        per_step = statistics.median(times)
        val = a.batch / per_step
        line = {"metric": METRIC, "value": val, "unit": "tok/s", "n_gpus": 0, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "impl": "reference", "config": workload,
                "cpu_baseline": {"value": val, "unit": "tok/s", "cores": os.cpu_count(),
                                 "kind": "port", "sample": sample},
                "e2e": {"value": val, "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    import chatnet_b200 as cn
    from chatnet_b200.llama import CudaLlamaModel

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))

    ctx = cn.Context(local)
    ext = torch.cuda.ExternalStream(ctx.stream)
    t0 = time.time()
    tp_mode = world > 1 and a.parallel == "tp"
    tp = None
    B = a.batch
    parity = tp_parity(ctx, rank, world, dist) if tp_mode else None
    if tp_mode:
        # one rank per GPU: join the group through the exchange buffers' IPC handles
        tp = cn.TensorParallel(ctx, rank, world, B, dc.model.dim, dc.model.vocab)
        handles = [None] * world
        dist.all_gather_object(handles, tp.ipc_handle())
        tp.connect(handles)
        tensors = cf.device_tensors(ctx, dc, rank=rank, size=world)  # this rank's shards
    else:
        tensors = cf.device_tensors(ctx, dc)  # seeded generator, on the device
    model = CudaLlamaModel(ctx, dc.model, tensors, tp=tp)
    for b in range(B):
        model.kv_synth(b, dc.kv_filled, *cf.kv_seeds(dc, b))
    toks = [cf.token(dc, b) for b in range(B)]
    pos = [dc.decode_pos] * B
    model.set_inputs(toks, pos)
    model.prepare(B)  # capture the step graph before any rank starts a step
    if dist is not None:
        dist.barrier()
    setup_s = time.time() - t0

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        ctx.synchronize()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # warm-up (captures the graph on the first step)
    for _ in range(max(a.warmup, 3)):
        model.step(B)
    ctx.synchronize()

    if a.nvtx_step:
        ctx.synchronize()
        torch.cuda.nvtx.range_push("timed_step")
        model.step(B)
        ctx.synchronize()
        torch.cuda.nvtx.range_pop()
        print(json.dumps({"nvtx_step": True, "kernels": model.step_kernels(B)}), flush=True)
        return 0

    # timed region: device-resident steps
    barrier()
    clk = ClockSampler(local)
    clk.start()
    time.sleep(0.3)  # let the sampler start before the timed region
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    for _ in range(a.steps):
        model.step(B)
    e1.record(ext)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / a.steps
    clocks = clk.stop()
    ctx.synchronize()
    ms = max_over_ranks(ms)
    tokens_per_step = B if tp_mode else world * B  # tp: all ranks decode the same B sequences
    value = tokens_per_step * 1000.0 / ms

    # end to end through cn_llama_decode (host buffers)
    barrier()
    e0.record(ext)
    for _ in range(a.steps):
        lg, am = model.decode(toks, pos, logits=True, argmax=True)
    e1.record(ext)
    e1.synchronize()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1) / a.steps)
    e2e = tokens_per_step * 1000.0 / ms_e2e
    assert np.isfinite(lg).all()

    # roofline: the dominant kernel timed alone -- the FFN gate and up matrices as
    # the one launch the step runs (a model that runs them apart: the gate GEMV)
    hid = dc.model.hidden_dim // (world if tp_mode else 1)  # this rank's shard
    try:
        us, nbytes = model.time_gemv(9, B, iters=2 * dc.model.n_layers)
        shape, what = f"{2 * hid}x{dc.model.dim}", "gate/up, one launch"
    except cn.NotSupportedError:
        us, nbytes = model.time_gemv(4, B, iters=2 * dc.model.n_layers)
        shape, what = f"{hid}x{dc.model.dim}", "gate"
    peak, peak_kind = measured_peak_gbs()
    achieved = nbytes / (us * 1e-6) / 1e9
    gemv_name = gemv_kernel_name(a.config, B)
    traffic = committed_traffic(f"{gemv_name}_{shape}_b{B}")
    kernels = model.step_kernels(B)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cs = CpuSample(dc, B)
        per_step_s = statistics.median([cs.run_once() for _ in range(3)])
        cpu = {"value": B / per_step_s, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
               "sample": cs.describe(3)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if tp_mode else "weak",
            "vs_baseline": None,
            "dtype": gemv_dtype(a.config, B),
            "data": "synthetic (seeded generator, config shapes and distributions)",
            "config": workload,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": B * 8,
                    "d2h_bytes_per_step": B * (dc.model.vocab * 4 + 4)},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": f"{gemv_name} {shape} ({what}) batch {B}",
                         "us_per_launch": us, "bytes_per_launch": nbytes,
                         "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})"},
            "cpu_baseline": cpu,
            "gpu_launches": kernels * a.steps,
            "clocks": clocks,
            "setup_s": setup_s,
        }
        if parity is not None:
            line["tp_parity"] = parity
        print(json.dumps(line), flush=True)

    model.close()
    for t in tensors:
        t.free()
    if tp is not None:
        if dist is not None:
            dist.barrier()  # no rank unmaps its buffer while another may still store into it
        tp.close()
    ctx.close()
    if dist is not None:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
