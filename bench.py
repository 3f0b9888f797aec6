#!/usr/bin/env python
"""CyFA layer forward+backward benchmark on B200 (one JSON line on rank 0).

Workload (the config the headline metric is quoted on):
one CyclicFlowAttention layer, hidden 1024, 4 heads x head_dim 256, 128 slots,
B=8, T=2048, bf16, forward + backward seeded with dy ~ N(0,1), random-init
weights N(0, 0.02), synthetic x ~ N(0,1).  With --gpus N (torchrun) every rank
runs its own B=8 batch (weak scaling, batch-sharded data parallel) and the
weight gradients are averaged with one NCCL all-reduce per step.

--impl reference times the reference algorithm's CPU restatement (the oracle;
the reference itself has no CPU path and needs Jittor) on the host cores.
"""

import argparse
import csv
import datetime
import gc
import io
import json
import math
import os
import statistics
import subprocess
import sys
import time

# NCCL_DEBUG is left as the environment sets it: NCCL's own lines (version
# banner, communicator setup) may share stdout with the result, which is always
# printed last, as one JSON object on a line of its own.

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "cyfa-jittor_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "CyFA layer fwd+bwd tokens/s/GPU; decode tokens/s; % of TC/HBM roofline"
UNIT = "tokens/s"
CFG = dict(hidden=1024, heads=4, head_dim=256, slots=128, B=8, T=2048)
L2_BYTES = 126 * 2 ** 20
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# Algorithmic work (FLOPs, full 128x128 tiles as the tensor cores issue them) per
# 128-token tile of one (batch, head), by kernel, for K = V = 256, 128 slots.
# A tile has C = 128 tokens; per pass: pass 1 is (Dk, Dv) = (K, 128), pass 2 (128, V).
def _tile_flops(K=256, V=256, C=128, M=128):
    p1 = (K, M)
    p2 = (M, V)
    out = {}
    # forward output tiles: QK^T (2 C C Dk) + Q S (2 C Dk Dv) + P V (2 C C Dv)
    def fwd(dk, dv):
        return 2 * C * C * dk + 2 * C * dk * dv + 2 * C * C * dv
    out["tile_fwd_readout"] = fwd(*p1) + 2 * (2 * C * M * M)
    out["tile_fwd"] = fwd(*p2)
    # state scans: K^T V per tile (2 C Dk Dv) per pass
    out["state_scan_fwd"] = 2 * C * p1[0] * p1[1] + 2 * C * p2[0] * p2[1]
    out["state_scan_bwd"] = out["state_scan_fwd"]
    # scores: QK^T and dO V^T
    out["tile_scores"] = sum(2 * C * C * dk + 2 * C * C * dv for dk, dv in (p1, p2))
    # dual GEMMs: dq (N=Dk, KD=Dv), dk (N=Dk, KD=Dv), dv (N=Dv, KD=Dk): 2 C (C N + KD N)
    out["dual_gemm"] = sum(2 * C * (C * dk + dv * dk) * 2 + 2 * C * (C * dv + dk * dv)
                           for dk, dv in (p1, p2))
    out["readout_bwd"] = 5 * 2 * C * M * M
    return out


def _compulsory_bytes(K=256, V=256, M=128):
    """Compulsory HBM bytes per tok-head (one token of one (batch, head)) of the
    operation each core kernel implements, summed over all its launches of one
    layer step: the inputs the operation must read and the outputs it must write,
    once each, bf16 activations and fp32 gates.  Intermediates the kernels choose
    to keep in HBM (state histories and their adjoints, materialised score
    matrices) are not counted: they are the kernels' own traffic, reported
    separately as measured DRAM bytes.

    * ScalarGatedLA forward, per pass: read q, k (Dk each), v (Dv), the gate (4 B);
      write o (Dv) -> 1,540 B at Dk = Dv = 256 (pass 1 reads the 128-wide write
      vector as its values and writes raw/weights, the fused readout adding
      lambda, 4 B).
    * ScalarGatedLA backward (the dual GEMM forms every dq, dk, dv of both passes):
      pass 1 reads q, k (256 each), w (128), dY (128), the gate; writes dq, dk,
      dw, the gate gradient -> 2,824 B; pass 2 reads weights, w (128 each),
      v, dO (256 each), the gate; writes dweights, dw, dv, the gate gradient
      -> 2,568 B.
    * Readout adjoint: read raw, dweights (128 each), lambda; write draw, dlambda
      -> 776 B; forward readout (fused into the pass-1 tile) 516 B.
    * The scores and state scans form intermediates only: their compulsory bytes
      are the inputs they read (q, k, w, dO, v of both passes; k, w, v for the
      scans)."""
    b = 2
    fwd1 = b * (K + K + M + M) + 4 + 4            # q, k, w in; raw/weights out; G, lam
    fwd2 = b * (M + M + V + V) + 4                # weights, w, v in; o out; G
    bwd1 = b * (K + K + M + M) + 4 + b * (K + K + M) + 4     # in: q k w dY g; out: dq dk dw dg
    bwd2 = b * (M + M + V + V) + 4 + b * (M + M + V) + 4     # in: a w v dO g; out: da dw dv dg
    return {
        "tile_fwd_readout": fwd1,
        "tile_fwd": fwd2,
        "dual_gemm": bwd1 + bwd2,
        "readout_bwd": b * (M + M + M) + 4 + 4,
        "tile_scores": b * (K + K + M + M) + b * (M + M + V + V),
        "state_scan_fwd": b * (K + M) + b * (M + V),
        "state_scan_bwd": b * (K + M) + b * (M + V),
    }


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return PEAKS_FALLBACK, "fallback"


def _traffic_from_profiles(kernel):
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.txt")
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 2 and not line.startswith("#") and parts[0] == kernel:
                    return float(parts[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """SM clock and clock-event reasons of this process's GPU, sampled while the
    timed work runs: NVML is read from the host thread that waits for the timed
    region (`poll_until`), so every sample falls inside it.  Only reads: no clock
    or other setting is changed.  nvidia-smi at 200 ms is the fallback when NVML
    is unavailable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("hw_power_brake_slowdown", "nvmlClocksEventReasonHwPowerBrakeSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.nvml = None
        self.handle = None
        self.samples = []

    def _nvml_handle(self, nv):
        import torch

        props = torch.cuda.get_device_properties(self.index)
        uid = str(props.uuid)
        for u in (uid, "GPU-" + uid):
            try:
                return nv.nvmlDeviceGetHandleByUUID(u)
            except Exception:
                pass
        bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        return nv.nvmlDeviceGetHandleByPciBusId_v2(bus)

    def start(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.handle = self._nvml_handle(nv)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.handle, nv.NVML_CLOCK_SM)
            self.nvml = nv
            return
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.3)
        except OSError:
            self.proc = None

    def sample(self):
        if self.nvml is None:
            return
        nv = self.nvml
        try:
            mhz = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
            mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        except Exception:
            return
        self.samples.append((mhz, mask))

    def poll_until(self, event):
        """Samples every ~2 ms until `event` (recorded after the timed work) has
        completed on the device."""
        while not event.query():
            self.sample()
            time.sleep(0.002)

    def stop(self):
        if self.nvml is not None:
            nv = self.nvml
            try:
                nv.nvmlShutdown()
            except Exception:
                pass
            if not self.samples:
                return None
            reasons = sorted({name for name, attr in self.REASONS for _, m in self.samples
                              if hasattr(nv, attr) and m & getattr(nv, attr)})
            return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                    "sm_max_mhz": float(self.max_mhz), "reasons": reasons,
                    "samples": len(self.samples), "source": "NVML, inside the timed region"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r for r in csv.reader(io.StringIO(out)) if len(r) >= 9]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4)
                          if r[5 + i].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].strip().replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi, 200 ms"}


def _rank_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


# ---------------------------------------------------------------- CPU baseline
def cpu_model_name():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def _cpu_layer_step(T, cfg=None):
    """One step of the oracle layer forward + backward (fp32, all host threads)
    on one sequence of T tokens of the workload's layer config (or `cfg`): the
    reference's algorithm restated on the host cores."""
    import torch

    from oracle import cyfa_oracle as O

    cfg = cfg or CFG
    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator().manual_seed(0)
    H, hd, hid = cfg["heads"], cfg["head_dim"], cfg["hidden"]
    shapes = {
        "q_proj.weight": (H * hd, hid), "k_proj.weight": (H * hd, hid),
        "v_proj.weight": (H * hd, hid), "a_proj.weight": (H, hid), "b_proj.weight": (H, hid),
        "b_proj.bias": (H,), "d_proj.weight": (H, hid), "d_proj.bias": (H,),
        "q_conv1d.weight": (H * hd, 1, 4), "k_conv1d.weight": (H * hd, 1, 4),
        "v_conv1d.weight": (H * hd, 1, 4), "g_proj.0.weight": (hd, hid),
        "g_proj.1.weight": (H * hd, hd), "g_proj.1.bias": (H * hd,),
        "o_proj.weight": (hid, H * hd)}
    params = {n: torch.randn(*s, generator=gen) * 0.02 for n, s in shapes.items()}
    params["dt_bias"] = torch.full((H,), -4.0)
    params["A_log"] = torch.log(torch.rand(H, generator=gen) * 16 + 1e-3)
    params["readout"] = torch.eye(127).expand(H, -1, -1).clone()
    for n in ("q_norm.weight", "k_norm.weight", "o_norm.weight"):
        params[n] = torch.ones(hd)
    for p in params.values():
        p.requires_grad_(True)
    x = torch.randn(1, T, hid, generator=gen, requires_grad=True)
    dy = torch.randn(1, T, hid, generator=gen)

    def step():
        for p in params.values():
            p.grad = None
        x.grad = None
        y = O.cyfa_layer(params, x, H, hd, hd)
        (y * dy).sum().backward()

    return step


def cpu_layer_tokens_per_s(min_seconds=10.0, max_reps=20, T=None, warm=1):
    """Times the oracle layer fwd+bwd (fp32, all host threads) on one sequence:
    `warm` untimed steps, then steps until `min_seconds` or `max_reps`."""
    threads = os.cpu_count() or 1
    # long sequences: time 4096 tokens (the chunked cost is linear in T)
    T = T or min(CFG["T"], 4096)
    step = _cpu_layer_step(T)
    for _ in range(warm):
        step()
    t0 = time.perf_counter()
    reps = 0
    while reps < max_reps and (reps == 0 or time.perf_counter() - t0 < min_seconds):
        step()
        reps += 1
    dt = time.perf_counter() - t0
    note = "" if T == CFG["T"] else f" (tokens/s extrapolated to T={CFG['T']}: linear cost)"
    return reps * T / dt, threads, f"{reps} x (1 seq x {T} tokens) layer fwd+bwd, fp32 oracle{note}"


def cpu_decode_tokens_per_s(layers, batch, reps=3):
    """The decode leg's attention cores on the host: the oracle decode step
    (fp32, all host threads) for one layer at batch 32, timed over `reps` steps
    and scaled to `layers` layers and `batch` sequences (the step's cost is
    linear in both)."""
    import torch

    from oracle import cyfa_oracle as O

    torch.set_num_threads(os.cpu_count() or 1)
    H, K = DECODE["heads"], DECODE["head_dim"]
    b = min(32, batch)
    gen = torch.Generator().manual_seed(7)
    state = (0.01 * torch.randn(b, H, K, 128, generator=gen),
             0.01 * torch.randn(b, H, 128, K, generator=gen), torch.zeros(b, H))
    q, k, v = (torch.randn(b, 1, H, K, generator=gen) for _ in range(3))
    g = torch.full((b, 1, H), -0.05)
    d = torch.full((b, 1, H), 0.5)
    r = torch.eye(127).expand(H, -1, -1)
    w = torch.ones(K)
    with torch.no_grad():
        O.fused_recurrent_cyfa(q, k, v, g, d, d, r, w, w, initial_state=state,
                               output_final_state=True)
        t0 = time.perf_counter()
        for _ in range(reps):
            _, state = O.fused_recurrent_cyfa(q, k, v, g, d, d, r, w, w, initial_state=state,
                                              output_final_state=True)
        dt = (time.perf_counter() - t0) / reps
    per_token_step = dt * layers * batch / b
    return {"value": batch / per_token_step, "unit": "tokens/s", "cores": os.cpu_count() or 1,
            "kind": "port", "cpu": cpu_model_name(),
            "sample": f"{reps} decode steps of one layer's attention cores at batch {b}, fp32 "
                      f"oracle; scaled to {layers} layers x batch {batch} (extrapolated)"}


def run_reference(args, rank, world):
    """The reference arm: the reference algorithm's CPU implementation (its
    restatement in oracle/; the reference itself has no CPU path and needs
    Jittor) on the host cores.  Each step is one bounded sample of the workload:
    one sequence of the layer config, forward + backward.  `warmup` untimed
    steps, then exactly `steps` timed steps."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    T = min(CFG["T"], 4096)
    step = _cpu_layer_step(T)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    ms = 1000 * dt / args.steps
    tps = T / (ms / 1000.0)
    note = "" if T == CFG["T"] else f"; tokens/s extrapolated to T={CFG['T']} (linear cost)"
    sample = (f"each step: 1 seq x {T} tokens layer fwd+bwd, fp32 CPU oracle, "
              f"{threads} threads{note}")
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": ("cyfa_layer_fwd_bwd (BASELINE configs[2]) on host cores"
                                if args.workload == "c3" else
                                "cyfa_layer_fwd_bwd long context (BASELINE configs[4]) on host "
                                "cores"),
                   **CFG, "parallelism": "cpu"},
        "cpu_baseline": {"value": tps, "unit": UNIT, "cores": threads, "kind": "port",
                         "cpu": cpu_model_name(), "sample": sample},
        "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "timed_s": dt,
        "note": "the reference (Jittor) has no CPU path and cannot be installed here; "
                "this is its algorithm restated in oracle/",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- decode leg
DECODE = dict(layers=24, batch=256, heads=8, head_dim=256, slots=128)
# BASELINE configs[1] (c2): the public chunk_cyfa op alone, per GPU
OPCFG = dict(B=8, T=4096, H=4, K=256, V=256)
# per token-head FLOPs of the op (full 128x128 tiles), K = V = 256, 128 slots:
# forward 2 x 180,224 + readout 65,536; backward 393,216 + 376,832 + readout 196,608
OP_FLOPS_FWD, OP_FLOPS_BWD = 425_984, 966_656
# BASELINE configs[4] (c5): long-context layer, per GPU one 32768-token sequence
C5 = dict(hidden=2048, heads=8, head_dim=256, slots=128, B=1, T=32768)


def measure_op(args, rank, world, dev, peaks, barrier):
    """chunk_cyfa (q/k RMSNorm, both ScalarGatedLA passes and the
    readout) forward and forward+backward on seeded synthetic inputs with the
    reference benchmark's distributions (benchmarks/run.py:135-151), B = 8 per GPU,
    H = 4, T = 4096, K = V = 256.  CUDA events per step, L2 flushed between steps."""
    import torch
    import torch.distributed as dist

    from cyclic_flow_attention import ops
    from cyclic_flow_attention.graphs import GraphedStep

    B, T, H, K, V = (OPCFG[k] for k in ("B", "T", "H", "K", "V"))
    gen = torch.Generator(device=dev).manual_seed(11 + rank)
    bf = torch.bfloat16
    q = torch.randn(B, T, H, K, device=dev, generator=gen).to(bf).requires_grad_(True)
    k = torch.randn(B, T, H, K, device=dev, generator=gen).to(bf).requires_grad_(True)
    v = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf).requires_grad_(True)
    g = (-0.1 * torch.rand(B, T, H, device=dev, generator=gen)).requires_grad_(True)
    delta = torch.sigmoid(torch.randn(B, T, H, device=dev, generator=gen)).requires_grad_(True)
    beta = torch.sigmoid(torch.randn(B, T, H, device=dev, generator=gen)).requires_grad_(True)
    readout = (torch.eye(127, device=dev).expand(H, -1, -1)
               + 0.05 * torch.randn(H, 127, 127, device=dev, generator=gen)).requires_grad_(True)
    qw = (1 + 0.1 * torch.randn(K, device=dev, generator=gen)).requires_grad_(True)
    kw = (1 + 0.1 * torch.randn(K, device=dev, generator=gen)).requires_grad_(True)
    do = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf)
    leaves = [q, k, v, g, delta, beta, readout, qw, kw]
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)

    def fwd():
        with torch.no_grad():
            o, _ = ops.chunk_cyfa(q, k, v, g, delta, beta, readout, qw, kw)
        return o

    def fwd_bwd():
        for t in leaves:
            t.grad = None
        o, _ = ops.chunk_cyfa(q, k, v, g, delta, beta, readout, qw, kw)
        o.backward(do)
        return o.detach()

    def timed(step_graph):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(max(3, min(args.steps, 10)))]
        barrier()
        for a, b in evs:
            flush.fill_(1)
            a.record()
            step_graph.replay()
            b.record()
        barrier()
        t = torch.tensor([sum(a.elapsed_time(b) for a, b in evs) / len(evs)], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    gf = GraphedStep(fwd, [], [], warmup=3)
    ms_f = timed(gf)
    gfb = GraphedStep(fwd_bwd, [], leaves, warmup=3)
    ms_fb = timed(gfb)
    tok = B * T
    th = tok * H
    peak = peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
    out = {"workload": "chunk_cyfa op, BASELINE configs[1] (B=8 per GPU, H=4, T=4096, K=V=256, "
                       "bf16, seeded synthetic inputs)",
           "fwd": {"tokens_per_s": world * tok / (ms_f / 1000.0), "ms": ms_f,
                   "tflops": th * OP_FLOPS_FWD / (ms_f / 1000.0) / 1e12},
           "fwd_bwd": {"tokens_per_s": world * tok / (ms_fb / 1000.0), "ms": ms_fb,
                       "tflops": th * (OP_FLOPS_FWD + OP_FLOPS_BWD) / (ms_fb / 1000.0) / 1e12},
           "tensor_peak_tflops": peak,
           "l2": "flushed between timed steps"}
    del gf, gfb
    return out


def measure_decode(args, rank, world, dev, peaks, barrier):
    """One decode token step of the attention cores of BASELINE configs[3]
    (24 layers, batch 256 sharded over the ranks, 8 x 256 heads, fp32 states):
    24 calls of cyfa_decode_step (in place).  Reports tokens/s of the cores and
    the decode kernel's achieved HBM bandwidth."""
    import ctypes

    import torch
    import torch.distributed as dist

    from cyclic_flow_attention import _lib
    from cyclic_flow_attention.ops.chunk import readout_table

    Ly, H, K = DECODE["layers"], DECODE["heads"], DECODE["head_dim"]
    B = DECODE["batch"] // world
    gen = torch.Generator(device=dev).manual_seed(7 + rank)
    states = [(0.01 * torch.randn(B, H, K, 128, device=dev, generator=gen),
               0.01 * torch.randn(B, H, 128, K, device=dev, generator=gen),
               torch.zeros(B, H, device=dev)) for _ in range(Ly)]
    tables = [readout_table(torch.eye(127, device=dev).expand(H, -1, -1).contiguous())
              .contiguous() for _ in range(Ly)]
    q = torch.randn(B, 1, H, K, device=dev, generator=gen).to(torch.bfloat16)
    k = torch.randn(B, 1, H, K, device=dev, generator=gen).to(torch.bfloat16)
    v = torch.randn(B, 1, H, K, device=dev, generator=gen).to(torch.bfloat16)
    g = torch.full((B, 1, H), -0.05, device=dev)
    delta = torch.full((B, 1, H), 0.5, device=dev)
    beta = torch.full((B, 1, H), 0.5, device=dev)
    w = torch.ones(K, device=dev)
    out = torch.empty(B, 1, H, K, device=dev, dtype=torch.bfloat16)
    P = _lib.ptr
    stream = _lib.stream()

    def token_step():
        for (hk, hv, ck), tab in zip(states, tables):
            _lib.call("cyfa_decode_step", P(q), P(k), P(v), P(g), P(delta), P(beta), P(tab),
                      P(w), P(w), P(hk), P(hv), P(ck), P(hk), P(hv), P(ck), P(out),
                      B, H, K, K, 0, 1e-6, 1e-6, K ** -0.5, stream)

    for _ in range(3):
        token_step()
    barrier()
    n = max(3, min(args.steps, 10))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(n):
        token_step()
    b.record()
    barrier()
    t = torch.tensor([a.elapsed_time(b) / n], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item()
    per_bh = 2 * (K * 128 + 128 * K) * 4 + (2 * K + 2 * K) * 2 + 12
    nbytes = Ly * B * H * per_bh
    gbs = nbytes / (ms / 1000.0) / 1e9
    peak = peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])
    del states
    torch.cuda.empty_cache()
    return {"workload": "decode token step of the attention cores, BASELINE configs[3] "
                        "(24 layers, batch 256 over the ranks, 8x256 heads, fp32 states)",
            "tokens_per_s": world * B / (ms / 1000.0), "ms_per_token_step": ms,
            "bytes_per_step": nbytes * world, "achieved_gbs_per_gpu": gbs,
            "hbm_peak_gbs": peak, "frac": gbs / peak}


LMCFG = dict(hidden_size=2048, num_heads=8, head_dim=256, num_slots=128, num_hidden_layers=24,
             vocab_size=32000, batch=256, prompt=512, new_tokens=256)


def measure_lm_decode(args, rank, world, dev, peaks, barrier):
    """BASELINE configs[3] end to end: the random-init 24-layer CyFA LM (hidden
    2048, 8 x 256 heads, 128 slots, vocab 32000, bf16 weights, fp32 states),
    batch 256 sharded over the ranks, a 512-token prefill of uniform-random ids,
    then greedy decode steps, each one replay of the CUDA graph of the whole
    model step (GraphedDecoder).  Reports decode tokens/s (all ranks, device
    time, max over ranks), the prefill rate, and the step's HBM traffic (fp32
    states read + written, bf16 weights read once) against the copy bandwidth."""
    import torch
    import torch.distributed as dist

    from cyclic_flow_attention.generation import GraphedDecoder
    from cyclic_flow_attention.models.cyfa import CyclicFlowAttentionConfig
    from cyclic_flow_attention.utils import initialize_model

    c = dict(LMCFG)
    if args.lm_layers:
        c["num_hidden_layers"] = args.lm_layers
    if args.lm_batch:
        c["batch"] = args.lm_batch
    cfg = CyclicFlowAttentionConfig(**{k: c[k] for k in ("hidden_size", "num_heads", "head_dim",
                                                          "num_slots", "num_hidden_layers",
                                                          "vocab_size")})
    B = c["batch"] // world
    model = initialize_model(cfg, generator=torch.Generator(device=dev).manual_seed(11),
                             device=dev).eval()
    gen = torch.Generator(device=dev).manual_seed(13 + rank)
    ids = torch.randint(0, cfg.vocab_size, (B, c["prompt"]), device=dev, generator=gen)
    dec = GraphedDecoder(model)
    with torch.no_grad():  # one untimed prefill (first-call costs), then the timed one
        hidden, _ = model.model(ids, use_cache=False)
    del hidden
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    with torch.no_grad():
        hidden, _ = model.model(ids, use_cache=False)
    b.record()
    del hidden
    torch.cuda.synchronize()
    prefill_ms = a.elapsed_time(b)
    dec.prefill(ids)
    for _ in range(3):
        dec.step()
    barrier()
    n = c["new_tokens"]
    a.record()
    for _ in range(n):
        dec.step()
    b.record()
    barrier()
    t = torch.tensor([a.elapsed_time(b) / n, prefill_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, prefill_ms = t.tolist()
    H, K = cfg.num_heads, cfg.head_dim
    state_bytes = cfg.num_hidden_layers * B * H * 2 * (K * 128 + 128 * K) * 4
    weight_bytes = sum(p.numel() * p.element_size() for p in model.parameters())
    gbs = (state_bytes + weight_bytes) / (ms / 1000.0) / 1e9
    peak = peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])
    dec = model = None
    torch.cuda.empty_cache()
    return {"workload": f"CyFA LM greedy decode, BASELINE configs[3]: {cfg.num_hidden_layers} "
                        "layers, hidden 2048, 8x256 heads, vocab 32000, random-init bf16 weights, "
                        f"fp32 states, batch {c['batch']} over the ranks, 512-token prefill of "
                        "uniform-random ids",
            "tokens_per_s": world * B / (ms / 1000.0), "ms_per_token_step": ms,
            "timed_steps": n, "prefill_tokens_per_s": world * B * c["prompt"] / (prefill_ms / 1000.0),
            "bytes_per_step_per_gpu": state_bytes + weight_bytes, "achieved_gbs_per_gpu": gbs,
            "hbm_peak_gbs": peak, "frac": gbs / peak,
            "launch": "one CUDA graph replay per step (embedding, 24 layers, norm, lm_head, argmax)"}


def measure_c5(args, rank, world, dev, peaks, barrier):
    """BASELINE configs[4], long context: the layer forward + backward at hidden
    2048, 8 x 256 heads, 128 slots, one 32768-token sequence per GPU (weak
    scaling: the 8-sequence batch over 8 GPUs), bf16, the step captured as one
    CUDA graph with the weight-gradient all-reduce when N > 1.  CUDA events per
    step, L2 flushed between steps; the CPU baseline times the oracle on 4096
    tokens and scales linearly (the chunked cost is linear in T)."""
    import torch
    import torch.distributed as dist

    from cyclic_flow_attention import CyclicFlowAttention
    from cyclic_flow_attention.distributed import GradientBuckets
    from cyclic_flow_attention.graphs import GraphedStep

    B, T, hid = C5["B"], C5["T"], C5["hidden"]
    torch.manual_seed(0)
    layer = CyclicFlowAttention(hid, C5["heads"], C5["head_dim"], num_slots=C5["slots"])
    with torch.no_grad():
        for name, p in layer.named_parameters():
            if p.dim() >= 2 and name != "readout":
                p.normal_(0, 0.02)
    layer = layer.keep_fp32().to(dev)
    params = list(layer.parameters())
    gen = torch.Generator(device=dev).manual_seed(2000 + rank)
    x = torch.randn(B, T, hid, device=dev, generator=gen).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(B, T, hid, device=dev, generator=gen).to(torch.bfloat16)
    buckets = None
    if world > 1:
        buckets = GradientBuckets(params, groups=[sum(layer.grad_groups(), [])])
        layer.grad_ready = buckets.early

    def step(xin, dyin):
        for p in params:
            p.grad = None
        xin.grad = None
        y, _ = layer(xin)
        y.backward(dyin)
        if buckets is not None:
            buckets.finish()
        return y[:, -1].sum(dtype=torch.float32)

    graphed = GraphedStep(step, [x, dy], params, warmup=3)
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)
    n = max(3, min(args.steps, 8))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n)]
    barrier()
    for a, b in evs:
        flush.fill_(1)
        a.record()
        graphed.replay()
        b.record()
    barrier()
    t = torch.tensor([sum(a.elapsed_time(b) for a, b in evs) / n], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item()
    flop = T * B * (3 * 35_749_888 + C5["heads"] * (OP_FLOPS_FWD + OP_FLOPS_BWD))
    tf = peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
    out = {"workload": "cyfa_layer_fwd_bwd long context, BASELINE configs[4]: hidden 2048, "
                       "8x256 heads, 128 slots, one 32768-token sequence per GPU, bf16",
           "tokens_per_s": world * B * T / (ms / 1000.0), "ms_per_step": ms,
           "tensor_frac_of_burst": flop / (ms / 1000.0) / 1e12 / tf,
           "l2": "flushed between timed steps"}
    del graphed
    if buckets is not None:
        buckets.remove()
    torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not args.no_cpu:
        step_cpu = _cpu_layer_step(4096, C5)
        step_cpu()
        t0 = time.perf_counter()
        step_cpu()
        dt = time.perf_counter() - t0
        out["cpu_baseline"] = {
            "value": 4096 / dt, "unit": UNIT, "cores": os.cpu_count() or 1, "kind": "port",
            "cpu": cpu_model_name(),
            "sample": "1 x (1 seq x 4096 tokens) layer fwd+bwd at the configs[4] layer, fp32 "
                      "oracle; tokens/s extrapolated to T=32768 (linear cost)"}
    return out


# ---------------------------------------------------------------- GPU arm
def run_cyfa(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from cyclic_flow_attention import CyclicFlowAttention, _lib
    from cyclic_flow_attention.distributed import GradientBuckets
    from cyclic_flow_attention.graphs import GraphedStep

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if args.lm_only:
        # the LM decode leg alone (a smaller model for profiling runs)
        def sync_ranks():
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()

        res = measure_lm_decode(args, rank, world, dev, _peaks()[0], sync_ranks)
        if rank == 0:
            print(json.dumps({"decode_lm": res, "n_gpus": world}), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    B, T, hid = CFG["B"], CFG["T"], CFG["hidden"]
    torch.manual_seed(0)
    layer = CyclicFlowAttention(hid, CFG["heads"], CFG["head_dim"], num_slots=CFG["slots"])
    with torch.no_grad():
        for name, p in layer.named_parameters():
            if p.dim() >= 2 and name != "readout":
                p.normal_(0, 0.02)
    layer = layer.keep_fp32().to(dev)
    params = [p for p in layer.parameters()]
    gen = torch.Generator().manual_seed(1000 + rank)
    x_host = torch.randn(B, T, hid, generator=gen).to(torch.bfloat16).pin_memory()
    dy_host = torch.randn(B, T, hid, generator=gen).to(torch.bfloat16).pin_memory()
    # the layer's input requires grad, as for any layer inside a network: the
    # backward includes dx (the reference's FLOP count is fwd + dgrad + wgrad)
    x = x_host.to(dev).requires_grad_(True)
    dy = dy_host.to(dev)
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)
    peaks, peak_kind = _peaks()

    # gradient averaging over ranks, bucketed and overlapped with the backward
    buckets = None
    if world > 1:
        # one fp32 bucket for the whole layer, completed by the input-side weight
        # gradients, which the fused backward hands over before its dx GEMM: the
        # all-reduce overlaps that GEMM instead of the persistent core kernels;
        # at configs[2] the GEMM leaves 32 SMs to it (cuBLASLt SM-count target),
        # so the collective runs beside the GEMM instead of after it (at
        # configs[4] that measured no faster: the larger GEMM hides it already)
        buckets = GradientBuckets(params, groups=[sum(layer.grad_groups(), [])],
                                  comm_sms=32 if args.workload == "c3" else 0)
        layer.grad_ready = buckets.early

    def allreduce_grads():
        if buckets is not None:
            buckets.finish()

    def step(xin, dyin):
        # training step whose backward is seeded with the cotangent dy (dL/dy = dy,
        # as the reference benchmark seeds its backward: benchmarks/core.py:384-396);
        # the result the host reads back is a checksum of the output's last token
        for p in params:
            p.grad = None
        xin.grad = None
        y, _ = layer(xin)
        y.backward(dyin)
        with torch.no_grad():
            check = y[:, -1].sum(dtype=torch.float32)
        allreduce_grads()
        return check

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # the whole step (forward, backward, gradient all-reduce) as one CUDA graph,
    # captured after W eager warm-up steps; inputs live at fixed device addresses
    graphed = GraphedStep(step, [x, dy], params, warmup=args.warmup)
    for _ in range(3):
        graphed.replay()
    barrier()

    # ---- device-resident timing (value): per-step events, L2 flushed between steps
    sampler = ClockSampler(torch.cuda.current_device() if world == 1 else local_rank)
    sampler.start()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    barrier()
    for a, b in evs:
        flush.fill_(1)
        a.record()
        graphed.replay()
        b.record()
    sampler.poll_until(evs[-1][1])
    barrier()
    launches = graphed.library_launches * args.steps
    clocks = sampler.stop()
    total_ms = sum(a.elapsed_time(b) for a, b in evs)
    t = torch.tensor([total_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = t.item() / args.steps
    value = world * B * T / (ms_per_step / 1000.0)

    # ---- end to end: every step copies its input batch from pinned host memory
    # and reads its result (the output checksum) back.  The cotangent dy is the
    # objective's fixed weight and stays on the device, as the reference
    # benchmark's `do` does (benchmarks/core.py:295-296: one tensor for every
    # step).  The next step's host-to-device copy runs on a side stream into the
    # other of two input buffers while the current step computes, as a data loader
    # would, and the step reads it there: a second capture of the step (sharing
    # the first one's memory pool; the two never run at the same time) takes the
    # other buffer, so steps alternate between the two graphs and no device-side
    # copy is needed.
    x2 = torch.empty_like(x).requires_grad_(True)
    graphed2 = GraphedStep(step, [x2, dy], params, warmup=1, pool=graphed.pool())
    graphs, bufs = [graphed, graphed2], [x, x2]
    copy_stream = torch.cuda.Stream(device=dev)
    copied = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    main = torch.cuda.current_stream(dev)

    def start_copy(i):
        b = i % 2
        copy_stream.wait_event(done[b])
        with torch.cuda.stream(copy_stream), torch.no_grad():
            bufs[b].copy_(x_host, non_blocking=True)
            copied[b].record(copy_stream)

    for b in range(2):
        done[b].record(main)
    # each step's checksum goes to pinned host memory by an asynchronous copy; the
    # host reads step i's value once step i + 1 is enqueued, so the read-back does
    # not leave the GPU idle while the host wakes up
    checks_host = torch.empty(2, dtype=torch.float32).pin_memory()
    read = [torch.cuda.Event() for _ in range(2)]
    checks = []
    e_a, e_b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e_a.record()
    start_copy(0)
    for i in range(args.steps):
        b = i % 2
        main.wait_event(copied[b])
        if i + 1 < args.steps:
            start_copy(i + 1)
        check = graphs[b].replay()
        done[b].record(main)
        checks_host[b].copy_(check, non_blocking=True)
        read[b].record(main)
        if i > 0:
            read[1 - b].synchronize()
            checks.append(checks_host[1 - b].item())
    read[(args.steps - 1) % 2].synchronize()
    checks.append(checks_host[(args.steps - 1) % 2].item())
    e_b.record()
    barrier()
    if len(checks) != args.steps or not all(math.isfinite(c) for c in checks):
        raise RuntimeError(f"e2e: bad step results {checks[:4]}")
    te = torch.tensor([e_a.elapsed_time(e_b)], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_ms = te.item() / args.steps
    e2e = {"value": world * B * T / (e2e_ms / 1000.0), "unit": UNIT,
           "h2d_bytes_per_step": x_host.numel() * 2,
           "d2h_bytes_per_step": 4, "ms_per_step": e2e_ms,
           "note": "H2D of the batch x of step i+1 overlaps step i on a copy stream; the "
                   "cotangent dy stays on the device (the reference benchmark's fixed do); "
                   "each step's output checksum is copied to pinned host memory and read by "
                   "the host once the next step is enqueued"}

    # ---- per-kernel event timing of one step (separate pass) -> dominant kernel
    barrier()
    _lib.profile_enable(True)
    flush.fill_(1)
    step(x, dy)
    torch.cuda.synchronize()
    prof = _lib.profile_report()
    _lib.profile_enable(False)
    tiles = B * CFG["heads"] * math.ceil(T / 128)
    tok_heads = B * T * CFG["heads"]
    flops = _tile_flops(CFG["head_dim"], CFG["head_dim"])
    cbytes = _compulsory_bytes(CFG["head_dim"], CFG["head_dim"])
    roofline = None
    if prof:
        dom = max(prof.items(), key=lambda kv: kv[1][0])
        name, (ms, n) = dom
        traffic = _traffic_from_profiles(name)
        # every core kernel moves more bytes per FLOP than the ridge (peak FLOP/s
        # over peak B/s), so it is bounded by HBM bandwidth: achieved = the
        # compulsory bytes of the operation it implements over its time
        if name in cbytes:
            peak = peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"])
            work = cbytes[name] * tok_heads  # all launches of this kernel in one step
            achieved = work / (ms / 1000.0) / 1e9 if ms > 0 else 0.0
            roofline = {"bound": "hbm", "kernel": name, "achieved": achieved, "peak": peak,
                        "unit": "GB/s", "frac": achieved / peak,
                        "traffic": traffic, "algorithmic_bytes_per_launch": work / n,
                        "algorithmic_bytes_per_tok_head": cbytes[name],
                        "tflops": flops.get(name, 0) * tiles / (ms / 1000.0) / 1e12,
                        "peak_kind": f"{peak_kind} HBM copy (of measured)" if peak_kind ==
                        "measured" else "fallback HBM copy"}
        else:
            peak = peaks.get("bf16_tflops_sustained", PEAKS_FALLBACK["bf16_tflops_sustained"])
            work = flops.get(name, 0) * tiles
            achieved = work / (ms / 1000.0) / 1e12 if ms > 0 else 0.0
            roofline = {"bound": "tensor", "kernel": name, "achieved": achieved, "peak": peak,
                        "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
                        "peak_kind": f"{peak_kind} bf16 sustained"}
        roofline.update({"launches_per_step": n, "ms_per_step": ms,
                         "kernel_ms": {k: round(v[0], 4) for k, v in sorted(prof.items())}})

    # the whole step against the tensor-core peak: the layer's FLOPs (projection
    # GEMMs forward, data and weight gradients, plus the attention core forward and
    # backward) over the measured step time
    hid, H, hd = CFG["hidden"], CFG["heads"], CFG["head_dim"]
    n_used = 3 * H * hd + hd + 3 * H
    gemm_flop = 3 * 2 * B * T * (hid * n_used + hd * H * hd + H * hd * hid)
    core_flop = tok_heads * (OP_FLOPS_FWD + OP_FLOPS_BWD)
    tf_burst = peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"])
    tf_sus = peaks.get("bf16_tflops_sustained", PEAKS_FALLBACK["bf16_tflops_sustained"])
    step_tflops = (gemm_flop + core_flop) / (ms_per_step / 1000.0) / 1e12
    layer_tensor = {"flop_per_step": gemm_flop + core_flop, "gemm_flop": gemm_flop,
                    "core_flop": core_flop, "achieved_tflops": step_tflops,
                    "frac_of_burst": step_tflops / tf_burst,
                    "frac_of_sustained": step_tflops / tf_sus,
                    "peaks": f"{peak_kind} bf16 {tf_burst} (burst) / {tf_sus} (sustained) TFLOP/s"}

    decode = None if args.no_decode else measure_decode(args, rank, world, dev, peaks, barrier)
    op = None if args.no_op else measure_op(args, rank, world, dev, peaks, barrier)
    decode_lm = None if args.no_lm else measure_lm_decode(args, rank, world, dev, peaks, barrier)
    long_ctx = None if (args.no_c5 or args.workload == "c5") else \
        measure_c5(args, rank, world, dev, peaks, barrier)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        tps, cores, sample = cpu_layer_tokens_per_s(min_seconds=args.cpu_seconds)
        cpu = {"value": tps, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample,
               "cpu": cpu_model_name()}
        if decode is not None:
            decode["cpu_baseline"] = cpu_decode_tokens_per_s(DECODE["layers"], DECODE["batch"])

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": ("cyfa_layer_fwd_bwd (BASELINE configs[2])" if args.workload == "c3"
                                    else "cyfa_layer_fwd_bwd long context (BASELINE configs[4])"),
                       **CFG,
                       "global_batch": B * world, "seq_len": T,
                       "parallelism": f"dp{world} (batch x head sharded, grad all-reduce)",
                       "l2": "flushed between timed steps (2x126 MiB write outside the events)",
                       "launch": "whole step (fwd, bwd, grad all-reduce) replayed as one CUDA graph"},
            "roofline": roofline,
            "layer_tensor_frac": layer_tensor["frac_of_burst"],
            "layer_tensor": layer_tensor,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks,
            "decode": decode,
            "decode_lm": decode_lm,
            "op": op,
            "c5": long_ctx,
        }
        print(json.dumps(line), flush=True)
    # a graph that holds NCCL calls must be gone before the process group is
    graphed = graphed2 = graphs = None
    gc.collect()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("cyfa", "reference"), default="cyfa")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode-kernel leg")
    ap.add_argument("--no-lm", action="store_true",
                    help="skip the 24-layer LM decode leg (configs[3] end to end)")
    ap.add_argument("--lm-only", action="store_true",
                    help="run only the LM decode leg and print its result")
    ap.add_argument("--lm-layers", type=int, default=0,
                    help="LM decode leg: layers (default 24, configs[3])")
    ap.add_argument("--lm-batch", type=int, default=0,
                    help="LM decode leg: batch over all ranks (default 256, configs[3])")
    ap.add_argument("--no-op", action="store_true", help="skip the chunk_cyfa op leg (configs[1])")
    ap.add_argument("--no-c5", action="store_true",
                    help="skip the long-context leg (configs[4], one 32768-token sequence per GPU)")
    ap.add_argument("--workload", choices=("c3", "c5"), default="c3",
                    help="layer config: c3 (BASELINE configs[2], default) or c5 (long context, "
                         "configs[4], one 32768-token sequence per GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.workload == "c5":
        CFG.clear()
        CFG.update(C5)
    rank, world, local_rank = _rank_env()
    if world > 1:
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    if args.impl == "reference":
        run_reference(args, rank, world)
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()
        return
    run_cyfa(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
