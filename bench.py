"""Benchmark of the FastDialogueSidon attention hot path on B200.

Headline (BASELINE.json metric, configs[1]): the 13-layer w2v-BERT encoder
relative_key attention of one 120 s window (L=6000, 16 x 64 heads, fp16
operands, fp32 softmax/accumulation), in ms per window (lower is better).

One step = the 13 layer calls of one window, each on its own precomputed QKV
(13 x 36.9 MB = 479 MB of inputs > the 126 MB L2, so no flush is needed
between steps). The QKV of layer i follows the stacking rule: x_{i+1} =
x_i + Attn_i(x_i) W_out^T on an fp32 residual, x_0 ~ N(0,1), weights
~ N(0, 0.02), rel ~ N(0, 0.02) (random init, seeded per window).

Beside the headline, the same line carries (all timed on the device with CUDA
events, max over ranks):
  dit         config 4: the 8-layer DiT RoPE attention of one window;
  config3     config 3: a batch of 8 windows of random length (3.2-120 s),
              bucketed to 10 s, key padding through kv_len; credited FLOPs
              sum_b 13*4*16*64*L_b*kv_len_b (padding not credited);
  throughput  config 5: 64 windows x (13-layer encoder + 8-layer DiT
              attention), windows g, g+N, ... on rank g, windows/s =
              64 / max-over-ranks time of one sweep;
  e2e         the headline through the public API with host buffers, with the
              measured host<->device copy bandwidth of the same pinned buffers
              and the copy-bound time it implies.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
Multi-GPU: launched under torch.distributed.run, one process per GPU; every
rank owns whole windows (weak scaling, no data-path collective); the step time
is the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

L_WINDOW = 6000          # 120 s at 50 Hz
ENC_LAYERS, ENC_HEADS = 13, 16
DIT_LAYERS, DIT_HEADS = 8, 12
HEAD_DIM = 64
FLOP_ENC_LAYER = 4 * ENC_HEADS * L_WINDOW * L_WINDOW * HEAD_DIM   # 147.456 GFLOP (QK^T + PV)
FLOP_DIT_LAYER = 4 * DIT_HEADS * L_WINDOW * L_WINDOW * HEAD_DIM   # 110.592 GFLOP
DATASHEET_DENSE_FP16_TFLOPS = 2250.0
FALLBACK_PEAK_TFLOPS = 1590.0
METRIC = "ms per 120 s window (13-layer rel-bias attn)"
UNIT = "ms/window"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-dit", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own GPU ops (baseline/_ref) beside ours")
    ap.add_argument("--schedule", choices=("auto", "unit"), default="auto",
                    help="auto: the library picks whole units per CTA or the balanced (stream-K) grid; "
                         "unit: always one 256-row unit per CTA")
    ap.add_argument("--case", choices=("enc1", "dit1", "qkv", "ropeqkv", "accum"), default=None,
                    help="profiling case: W + K eager launches of one layer's attention (encoder or DiT), of the "
                         "encoder's QKV projection (qkv), the DiT's QKV projection with RoPE (ropeqkv) or the "
                         "encoder's out-projection into the fp32 residual (accum), at L=6000")
    ap.add_argument("--no-config3", action="store_true")
    ap.add_argument("--no-throughput", action="store_true")
    ap.add_argument("--no-linear", action="store_true")
    return ap.parse_args()


def config_dict(n_gpus: int) -> dict:
    return {
        "workload": "config2: 13-layer encoder relative_key attention, one 120 s window",
        "seq_len": L_WINDOW, "heads": ENC_HEADS, "head_dim": HEAD_DIM, "layers": ENC_LAYERS,
        "windows_per_gpu_per_step": 1, "global_batch": n_gpus,
        "parallelism": f"windows partitioned over {n_gpus} GPU(s), no collectives",
        "l2": "inputs 479 MB per step > 126 MB L2 (no flush)",
        "timing": "13 calls captured in one CUDA graph per step; CUDA events on the launch stream",
    }


def measured_peak():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), "of measured (cuBLAS bf16 burst, MEASURED_PEAKS.json)"
    return FALLBACK_PEAK_TFLOPS, "of fallback (1.59 PFLOP/s bf16, earlier measurement on this pool)"


def ncu_traffic():
    """dram bytes per launch of the encoder kernel from the committed ncu summary."""
    p = REPO / "profiles" / "ncu_traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("flexrel_l6000_bytes_per_launch")
    return None


# ------------------------------------------------------------------ clocks


class ClockSampler:
    """nvidia-smi sampling of SM clocks / throttle reasons while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        self.rows: list[list[str]] = []
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.gpu = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:  # noqa: BLE001
            self.gpu = None

    def __enter__(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"]
        if self.gpu:
            cmd[1:1] = ["-i", self.gpu]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self) -> dict:
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        loaded = [r for r in self.rows if len(r) >= 9 and r[3].isdigit() and int(r[3]) > 0]
        use = loaded or [r for r in self.rows if len(r) >= 9]
        if not use:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[0]) for r in use if r[0].replace(".", "").isdigit()]
        reasons = sorted({names[k] for r in use for k in range(4) if r[5 + k].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(use[0][1]) if use[0][1].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(use),
                "power_w_max": max(float(r[2]) for r in use if r[2].replace(".", "").isdigit())}


# ------------------------------------------------------------------ workload


def make_window(seed: int, device: torch.device, layers: int = ENC_LAYERS, length: int = L_WINDOW,
                heads: int = ENC_HEADS, batch: int = 1, kv_len: torch.Tensor | None = None):
    """Per-layer fp16 QKV [B*L, 3*H*64] and rel [73, 64] for one window (or a
    padded batch of windows with key lengths kv_len), stacked on an fp32
    residual through this library's attention (setup, untimed)."""
    import fastdialoguesidon_b200 as F

    hidden = heads * HEAD_DIM
    gen = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(batch * length, hidden, generator=gen, device=device)
    if kv_len is not None:  # padded frames are zero, as the padded waveform's
        pad = torch.arange(length, device=device)[None, :] >= kv_len.to(device)[:, None].long()
        x[pad.reshape(-1)] = 0.0
    qkvs, rels = [], []
    for _ in range(layers):
        w_qkv = torch.randn(3 * hidden, hidden, generator=gen, device=device) * 0.02
        w_out = torch.randn(hidden, hidden, generator=gen, device=device) * 0.02
        rel = (torch.randn(73, HEAD_DIM, generator=gen, device=device) * 0.02).half()
        qkv = (x @ w_qkv.t()).half()
        ctx = F.flexrel_attention(qkv, batch, heads, rel, kv_len=kv_len)
        x = x + ctx.float() @ w_out.t()
        qkvs.append(qkv)
        rels.append(rel)
    F.check_status(device)
    return qkvs, rels


def config3_lengths(seed: int = 3, batch: int = 8) -> tuple[list[int], list[int]]:
    """Config 3: window lengths drawn uniformly from 3.2-120 s (frames =
    ceil(50 s)), each rounded up to its 10 s bucket (a multiple of 500 frames);
    returns (frames, buckets)."""
    g = torch.Generator().manual_seed(seed)
    secs = 3.2 + (120.0 - 3.2) * torch.rand(batch, generator=g, dtype=torch.float64)
    frames = [min(L_WINDOW, int(math.ceil(float(t) * 50.0))) for t in secs]
    buckets = [min(L_WINDOW, (f + 499) // 500 * 500) for f in frames]
    return frames, buckets


def make_dit_window(seed: int, device: torch.device):
    """Per-layer fp16 DiT QKV [L, 3*12*64] (N(0, 0.55), the scale the DiT's
    projections give) for one window."""
    gen = torch.Generator(device=device).manual_seed(seed)
    return [(torch.randn(L_WINDOW, 3 * DIT_HEADS * HEAD_DIM, generator=gen, device=device) * 0.55).half()
            for _ in range(DIT_LAYERS)]


def time_graph(fn, steps: int, warmup: int, device: torch.device, dist_on: bool, per_step: list | None = None) -> float:
    """Capture fn() once (on the stream its eager warm-up ran on); W untimed
    replays; K timed replays between barrier + synchronize on both sides;
    returns elapsed ms (CUDA events on the replay stream). ``per_step``, if
    given, receives each replay's own event time (for a median)."""
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream(device).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        fn()
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize(device)
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    evs[0].record(stream)
    for k in range(steps):
        g.replay()
        evs[k + 1].record(stream)
    torch.cuda.synchronize(device)
    if dist_on:
        torch.distributed.barrier()
    ms = evs[0].elapsed_time(evs[-1])
    if per_step is not None:
        per_step.extend(evs[k].elapsed_time(evs[k + 1]) for k in range(steps))
    del g
    return ms


def e2e_encoder(qkvs, rels, steps: int, warmup: int, device: torch.device, dist_on: bool, bal: bool = True):
    """The same metric through the public API with host buffers: every step copies
    its 13 QKV + rel tables host->device (pinned) and the 13 contexts back,
    overlapped over a copy-in / compute / copy-out stream pipeline."""
    import fastdialoguesidon_b200 as F

    host_in = [q.cpu().pin_memory() for q in qkvs]
    host_rel = [r.cpu().pin_memory() for r in rels]
    host_out = [torch.empty(q.shape[0], q.shape[1] // 3, dtype=q.dtype).pin_memory() for q in qkvs]
    dev_in = [torch.empty_like(q) for q in qkvs]
    dev_rel = [torch.empty_like(r) for r in rels]
    dev_out = [torch.empty(q.shape[0], q.shape[1] // 3, dtype=q.dtype, device=device) for q in qkvs]
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    comp = torch.cuda.current_stream(device)
    n = len(qkvs)
    h2d = sum(t.numel() * t.element_size() for t in host_in + host_rel)
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    ev_in = [torch.cuda.Event() for _ in range(n)]
    ev_c = [torch.cuda.Event() for _ in range(n)]
    ev_out = [torch.cuda.Event() for _ in range(n)]

    def step():
        for i in range(n):
            with torch.cuda.stream(s_in):
                s_in.wait_event(ev_c[i])  # the previous step's layer i is done with dev_in[i]
                dev_in[i].copy_(host_in[i], non_blocking=True)
                dev_rel[i].copy_(host_rel[i], non_blocking=True)
                ev_in[i].record(s_in)
            comp.wait_event(ev_in[i])
            comp.wait_event(ev_out[i])  # dev_out[i] read back by the previous step
            F.flexrel_attention(dev_in[i], 1, ENC_HEADS, dev_rel[i], out=dev_out[i], balanced=bal)
            ev_c[i].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_c[i])
                host_out[i].copy_(dev_out[i], non_blocking=True)
                ev_out[i].record(s_out)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s_in)
    for _ in range(steps):
        step()
    s_out.wait_stream(comp)
    end.record(s_out)
    torch.cuda.synchronize(device)
    if dist_on:
        torch.distributed.barrier()
    F.check_status(device)
    e2e_ms = start.elapsed_time(end)

    # copy roofline: the same pinned buffers moved with no kernel in between,
    # host->device alone, device->host alone, and both at once (full duplex),
    # every rank at the same time as in the e2e run
    def copies(h2d_on: bool, d2h_on: bool) -> float:
        if dist_on:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(comp)
        s_in.wait_stream(comp)
        s_out.wait_stream(comp)
        for _ in range(steps):
            if h2d_on:
                with torch.cuda.stream(s_in):
                    for i in range(n):
                        dev_in[i].copy_(host_in[i], non_blocking=True)
                        dev_rel[i].copy_(host_rel[i], non_blocking=True)
            if d2h_on:
                with torch.cuda.stream(s_out):
                    for i in range(n):
                        host_out[i].copy_(dev_out[i], non_blocking=True)
        comp.wait_stream(s_in)
        comp.wait_stream(s_out)
        b.record(comp)
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) / steps

    copy = {"h2d_ms": copies(True, False), "d2h_ms": copies(False, True), "both_ms": copies(True, True)}
    return e2e_ms, h2d, d2h, copy


_CPU_INPUTS = None


def _cpu_inputs():
    global _CPU_INPUTS
    if _CPU_INPUTS is None:
        gen = torch.Generator().manual_seed(0)
        shape = (1, ENC_HEADS, L_WINDOW, HEAD_DIM)
        q, k, v = (torch.randn(shape, generator=gen) * 0.64 for _ in range(3))
        rel = torch.randn(73, HEAD_DIM, generator=gen) * 0.02
        _CPU_INPUTS = (q, k, v, rel)
    return _CPU_INPUTS


def reference_cpu_core():
    """The reference's own fp32 CPU path, ``torch_core_chunked``
    (trt/src/fastdialoguesidon/flexrel_triton.py:298-329), imported unmodified
    from baseline/_ref when it is installed there; None otherwise."""
    path = REPO / "baseline" / "_ref"
    if not (path / "fastdialoguesidon" / "flexrel_triton.py").exists():
        return None
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))
    try:
        from fastdialoguesidon.flexrel_triton import torch_core_chunked
    except Exception:  # noqa: BLE001 - fall back to the port, and say so
        return None
    return torch_core_chunked


def cpu_layer_ms_per_window(threads: int | None = None) -> tuple[float, dict]:
    """One full encoder layer of one window (6000 query rows x 16 heads x 6000
    keys, fp32, 512-row chunks) on the host cores, scaled x13 layers to ms per
    window. Runs the reference's own torch_core_chunked when baseline/_ref has
    it ("reference"), else the oracle's restatement of it ("port")."""
    if threads:
        torch.set_num_threads(threads)
    q, k, v, rel = _cpu_inputs()
    core = reference_cpu_core()
    t0 = time.perf_counter()
    if core is not None:
        out = torch.empty_like(q)
        core(q, k, v, rel, out, chunk=512)
        kind, what = "reference", "reference torch_core_chunked (baseline/_ref, unmodified)"
    else:
        from oracle import flexrel_oracle as O

        for start in range(0, L_WINDOW, 512):
            O.flexrel_rows(q, k, v, rel, start, min(start + 512, L_WINDOW))
        kind, what = "port", "oracle restatement of torch_core_chunked"
    dt = time.perf_counter() - t0
    return dt * 1e3 * ENC_LAYERS, {
        "cores": torch.get_num_threads(), "cpu_count": os.cpu_count(), "kind": kind,
        "sample": f"{what}, fp32: one full layer of the window (6000 query rows x 16 heads x 6000 keys, "
                  f"{dt:.2f} s), x13 layers"}


def reference_gpu_leg(qkvs, rels, outs, dit_inputs, device, steps: int = 5) -> dict:
    """The reference's own GPU ops, installed unmodified under baseline/_ref
    (fds_triton.kernels), timed eagerly with CUDA events on the same window
    inputs as our arm: its fused Triton kernel and its split path (two causal
    SDPA calls + band merge, trt/src/fastdialoguesidon/flexrel_triton.py) for the
    encoder, rope_split + SDPA for the DiT (the reference model's pattern).
    Reported beside our numbers; never part of our timed region."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")
    if not os.path.isdir(os.path.join(path, "fds_triton")):
        return {"unavailable": "baseline/_ref/fds_triton not installed"}
    if path not in sys.path:
        sys.path.insert(0, path)
    try:
        import torch.nn.functional as Fn
        from fds_triton import kernels as RK
    except Exception as ex:  # noqa: BLE001 - report, do not fail the bench
        return {"unavailable": f"import failed: {type(ex).__name__}: {str(ex)[:120]}"}

    def timed(fn) -> float:
        for _ in range(3):
            fn()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize(device)
        return e0.elapsed_time(e1) / steps

    res = {"source": "fds_triton.kernels from baseline/_ref (unmodified), eager launches, CUDA events",
           "steps": steps}
    for name, op in (("fused", getattr(RK, "flexrel_attention", None)),
                     ("split", getattr(RK, "flexrel_attention_split", None))):
        if op is None:
            continue
        try:
            diff = (op(qkvs[0], 1, ENC_HEADS, rels[0]).float() - outs[0].float()).abs().max().item()
            ms = timed(lambda: [op(q, 1, ENC_HEADS, r) for q, r in zip(qkvs, rels)])
            res[f"encoder_{name}_ms_per_window"] = round(ms, 4)
            res[f"encoder_{name}_max_abs_diff_vs_ours"] = diff
        except Exception as ex:  # noqa: BLE001
            res[f"encoder_{name}"] = f"failed: {type(ex).__name__}: {str(ex)[:120]}"
    if dit_inputs is not None and hasattr(RK, "rope_split"):
        dq, cos, sin, dout = dit_inputs
        shape = (1, L_WINDOW, DIT_HEADS, HEAD_DIM)

        def ref_dit(q2):
            q, k, v = RK.rope_split(q2, L_WINDOW, DIT_HEADS, cos, sin)
            a = Fn.scaled_dot_product_attention(*(t.view(shape).transpose(1, 2) for t in (q, k, v)))
            return a.transpose(1, 2).reshape(L_WINDOW, DIT_HEADS * HEAD_DIM)

        try:
            diff = (ref_dit(dq[0]).float() - dout[0].float()).abs().max().item()
            res["dit_ms_per_window"] = round(timed(lambda: [ref_dit(q) for q in dq]), 4)
            res["dit_max_abs_diff_vs_ours"] = diff
        except Exception as ex:  # noqa: BLE001
            res["dit"] = f"failed: {type(ex).__name__}: {str(ex)[:120]}"
    return res


# ------------------------------------------------------------------ arms


def run_reference(args, rank: int) -> None:
    """CPU arm: the reference's fp32 path (its own torch_core_chunked from
    baseline/_ref, else the oracle's port of it) on all host cores, each step
    one full layer of the window, reported per window (x13 layers)."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    for _ in range(max(args.warmup, 1)):
        cpu_layer_ms_per_window()
    vals = []
    t0 = time.perf_counter()
    info = {}
    for _ in range(args.steps):
        ms, info = cpu_layer_ms_per_window()
        vals.append(ms)
        if time.perf_counter() - t0 > 150:  # keep the arm within a few minutes
            break
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": len(vals), "warmup": args.warmup, "ms_per_step": round(value, 3),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,0.64) q/k/v, N(0,0.02) rel)", "config": config_dict(args.gpus),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": info["kind"],
                         "sample": info["sample"] + "; median over steps"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def e2e_layer_leg(steps: int, warmup: int, device: torch.device, dist_on: bool) -> dict:
    """The 13 encoder attention layers as the model runs them, end to end
    through the public API with host buffers: per step the fp32 residual x of a
    window (6000 x 1024) is copied in from pinned host memory, each layer runs
    qkv = linear(x16, W_qkv, b) -> flexrel_attention -> accumulate(x, ctx, W_out)
    on the device (weights resident, random-init N(0, 0.02)), and x is copied
    back. The 13 layers of a window are one CUDA graph (as the reference's
    pipeline captures its model); windows alternate between two residual
    buffers so that window k+1's copy in and window k-1's copy out overlap
    window k's layers (copy-in / compute / copy-out streams). Work per window:
    the 13 attention layers plus their QKV and output projections
    (13 x (147.5 + 37.7 + 12.6) GFLOP)."""
    import fastdialoguesidon_b200 as F

    hid = ENC_HEADS * HEAD_DIM
    g = torch.Generator(device=device).manual_seed(4000)
    ws = [((torch.randn(3 * hid, hid, generator=g, device=device) * 0.02).half(),
           (torch.randn(3 * hid, generator=g, device=device) * 0.02).half(),
           (torch.randn(hid, hid, generator=g, device=device) * 0.02).half(),
           (torch.randn(73, HEAD_DIM, generator=g, device=device) * 0.02).half()) for _ in range(ENC_LAYERS)]
    host_x = torch.randn(L_WINDOW, hid, generator=torch.Generator().manual_seed(4001)).pin_memory()
    host_out = [torch.empty_like(host_x).pin_memory() for _ in range(2)]
    xs = [torch.empty(L_WINDOW, hid, device=device) for _ in range(2)]
    x16 = torch.empty(L_WINDOW, hid, dtype=torch.float16, device=device)
    qkv = torch.empty(L_WINDOW, 3 * hid, dtype=torch.float16, device=device)
    ctx = torch.empty(L_WINDOW, hid, dtype=torch.float16, device=device)
    comp = torch.cuda.Stream(device)
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)

    def layers(x):
        for w_qkv, b_qkv, w_out, rel in ws:
            x16.copy_(x)
            F.linear(x16, w_qkv, b_qkv, out=qkv)
            F.flexrel_attention(qkv, 1, ENC_HEADS, rel, out=ctx)
            F.accumulate(x, ctx, w_out)

    comp.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(comp):
        for b in range(2):  # eager warm-up (library state and workspaces are created outside capture)
            xs[b].copy_(host_x)
            layers(xs[b])
    torch.cuda.synchronize(device)
    graphs = []
    for b in range(2):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=comp):
            layers(xs[b])
        graphs.append(gr)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_c = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    for b in range(2):
        ev_c[b].record(comp)
        ev_out[b].record(s_out)
    k = [0]

    def step():
        b = k[0] & 1
        k[0] += 1
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_out[b])  # the previous window in this buffer has been copied out
            xs[b].copy_(host_x, non_blocking=True)
            ev_in[b].record(s_in)
        comp.wait_event(ev_in[b])
        with torch.cuda.stream(comp):  # a graph replays on the current stream
            graphs[b].replay()
        ev_c[b].record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_c[b])
            host_out[b].copy_(xs[b], non_blocking=True)
            ev_out[b].record(s_out)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for _ in range(steps):
        step()
    s_out.wait_stream(comp)
    e1.record(s_out)
    torch.cuda.synchronize(device)
    F.check_status(device)
    for gr in graphs:
        del gr
    graphs.clear()
    # every window starts from the same x: the last one copied out must equal the
    # same 13 layers run eagerly (same kernels, same order: bit for bit)
    last = (k[0] - 1) & 1
    with torch.cuda.stream(comp):
        xs[last].copy_(host_x)
        layers(xs[last])
    torch.cuda.synchronize(device)
    if not torch.equal(xs[last].cpu(), host_out[last]):
        raise RuntimeError("e2e_layer: pipelined windows differ from the eager layers")
    nbytes = host_x.numel() * 4
    return {"ms": e0.elapsed_time(e1), "steps": steps, "h2d": nbytes, "d2h": nbytes}


def linear_leg(device: torch.device, steps: int = 20) -> dict:
    """The projections either side of the attention on this library's tcgen05
    GEMM, at the config-2 / config-4 shapes (L = 6000): the encoder QKV
    projection with bias, the DiT QKV projection with the RoPE epilogue, the
    out-projection accumulated into the fp32 residual. Eight operand sets (more
    bytes than L2 holds) are cycled through one CUDA graph of eight calls; device
    time per call from CUDA events over `steps` replays after 3 warm-up
    replays, with torch (cuBLAS) on the same operands the same way for context.
    Algorithmic FLOPs 2 M N K; frac against the measured cuBLAS bf16 burst peak.
    ``pair`` / ``single``: this library with 256-row tiles over CTA pairs (the
    default) / 128-row tiles on one CTA each."""
    import fastdialoguesidon_b200 as F

    g = torch.Generator(device=device).manual_seed(17)
    peak, _ = measured_peak()
    sets = 8

    def timed(calls) -> float:
        def body():
            for c in calls:
                c()
        return time_graph(body, steps, 3, device, False) / steps / len(calls)

    res = {}
    cases = (("encoder_qkv", 1024, 3072, "store"), ("dit_qkv_rope", 768, 2304, "rope"),
             ("encoder_out_accumulate", 1024, 1024, "accum"))
    cos, sin = F.rope_tables(L_WINDOW, device)
    for name, k, n, kind in cases:
        xs = [torch.randn(L_WINDOW, k, generator=g, device=device).half() for _ in range(sets)]
        ws = [(torch.randn(n, k, generator=g, device=device) * 0.02).half() for _ in range(sets)]
        bs = [(torch.randn(n, generator=g, device=device) * 0.02).half() for _ in range(sets)]
        if kind == "accum":
            outs = [torch.zeros(L_WINDOW, n, device=device) for _ in range(sets)]
        else:
            outs = [torch.empty(L_WINDOW, n, dtype=torch.float16, device=device) for _ in range(sets)]
        flop = 2.0 * L_WINDOW * n * k

        def ours(i, pair):
            x, w, b, o = xs[i], ws[i], bs[i], outs[i]
            if kind == "store":
                return lambda: F.linear(x, w, b, out=o, pair=pair)
            if kind == "rope":
                return lambda: F.linear_rope(x, w, b, cos, sin, L_WINDOW, n // 192, out=o, pair=pair)
            return lambda: F.accumulate(o, x, w, pair=pair)

        def ref(i):
            x, w, b, o = xs[i], ws[i], bs[i], outs[i]
            if kind == "accum":
                return lambda: torch.addmm(o, x, w.t(), out_dtype=torch.float32, out=o)
            return lambda: torch.addmm(b, x, w.t(), out=o)

        pair_ms = timed([ours(i, None) for i in range(sets)])
        single_ms = timed([ours(i, False) for i in range(sets)])
        torch_ms = timed([ref(i) for i in range(sets)])
        tf = flop / (pair_ms * 1e-3) / 1e12
        res[name] = {"m": L_WINDOW, "n": n, "k": k, "ms": round(pair_ms, 4), "tflops": round(tf, 1),
                     "frac": round(tf / peak, 3), "single_cta_ms": round(single_ms, 4),
                     "torch_ms": round(torch_ms, 4), "torch_tflops": round(flop / (torch_ms * 1e-3) / 1e12, 1)}
    F.check_status(device)
    res["note"] = ("tcgen05 GEMM of this library (fds_linear_fwd), 256-row tiles over CTA pairs; single_cta_ms: "
                   "128-row tiles, one CTA each; torch_ms: torch.addmm (cuBLAS) on the same operands, the "
                   "reference's own call at these sites (rope: without the reference's separate rope_split pass); "
                   "device time per call inside a CUDA graph cycling 8 operand sets (> L2)")
    return res


def config3_leg(args, rank: int, device: torch.device, dist_on: bool, bal: bool) -> dict:
    """Config 3: a batch of 8 windows of seeded random length, bucketed to 10 s,
    padded to the longest bucket, keys masked past each window's true length
    (kv_len); 13 layers per step in one graph. Every rank runs its own batch."""
    import fastdialoguesidon_b200 as F

    frames, buckets = config3_lengths()
    B, Lmax = len(frames), max(buckets)
    kv = torch.tensor(frames, dtype=torch.int32, device=device)
    qkvs, rels = make_window(seed=3000 + rank, device=device, length=Lmax, batch=B, kv_len=kv)
    outs = [torch.empty(B * Lmax, ENC_HEADS * HEAD_DIM, dtype=torch.float16, device=device) for _ in qkvs]

    def step():
        for q, r, o in zip(qkvs, rels, outs):
            F.flexrel_attention(q, B, ENC_HEADS, r, out=o, kv_len=kv)

    steps = max(3, args.steps // 4)
    per = []
    ms = time_graph(step, steps, max(3, min(args.warmup, 5)), device, dist_on, per_step=per)
    F.check_status(device)
    credited = sum(ENC_LAYERS * 4 * ENC_HEADS * HEAD_DIM * lb * kb for lb, kb in zip(buckets, frames))
    computed = sum(ENC_LAYERS * 4 * ENC_HEADS * HEAD_DIM * Lmax * ((kb + 127) // 128 * 128) for kb in frames)
    del qkvs, outs
    return {"ms": ms, "steps": steps, "median": statistics.median(per), "credited": credited,
            "computed": computed, "frames": frames, "buckets": buckets, "Lmax": Lmax}


def throughput_leg(args, rank: int, world: int, device: torch.device, dist_on: bool, bal: bool) -> dict:
    """Config 5: 64 windows x (13-layer encoder + 8-layer DiT attention); rank g
    takes windows g, g+N, ...; one sweep over this rank's windows is captured
    in one CUDA graph."""
    import fastdialoguesidon_b200 as F

    mine = list(range(rank, 64, world))
    enc = [make_window(seed=5000 + w, device=device) for w in mine]
    dit = [make_dit_window(seed=6000 + w, device=device) for w in mine]
    cos, sin = F.rope_tables(L_WINDOW, device)
    eout = torch.empty(L_WINDOW, ENC_HEADS * HEAD_DIM, dtype=torch.float16, device=device)
    dout = torch.empty(L_WINDOW, DIT_HEADS * HEAD_DIM, dtype=torch.float16, device=device)
    scratch = torch.empty(L_WINDOW, 2 * DIT_HEADS * HEAD_DIM, dtype=torch.float16, device=device)

    def sweep():
        for (qkvs, rels), dq in zip(enc, dit):
            for q, r in zip(qkvs, rels):
                F.flexrel_attention(q, 1, ENC_HEADS, r, out=eout, balanced=bal)
            for q in dq:
                F.rope_attention(q, 1, DIT_HEADS, cos, sin, out=dout, scratch=scratch, balanced=bal)

    steps = max(2, min(args.steps, 5))
    per = []
    with ClockSampler(device) as clocks:
        ms = time_graph(sweep, steps, 2, device, dist_on, per_step=per)
    F.check_status(device)
    del enc, dit
    return {"ms": ms, "steps": steps, "median": statistics.median(per), "windows_here": len(mine),
            "clocks": clocks.summary()}


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import fastdialoguesidon_b200 as F

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist_on = world > 1
    if dist_on:
        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    bal = args.schedule == "auto"
    qkvs, rels = make_window(seed=1000 + rank, device=device)
    outs = [torch.empty(L_WINDOW, ENC_HEADS * HEAD_DIM, dtype=torch.float16, device=device) for _ in qkvs]

    def enc_step():
        for q, r, o in zip(qkvs, rels, outs):
            F.flexrel_attention(q, 1, ENC_HEADS, r, out=o, balanced=bal)

    per_step: list[float] = []
    with ClockSampler(device) as clocks:
        ms = time_graph(enc_step, args.steps, args.warmup, device, dist_on, per_step=per_step)
    F.check_status(device)
    med = statistics.median(per_step)
    e2e_steps = max(3, min(args.steps, 60))
    e2e_ms, h2d, d2h, copy = e2e_encoder(qkvs, rels, e2e_steps, max(3, min(args.warmup, 5)), device, dist_on,
                                         bal)

    dit = None
    dit_inputs = None
    if not args.no_dit:
        dq = make_dit_window(seed=2000 + rank, device=device)
        cos, sin = F.rope_tables(L_WINDOW, device)
        dout = [torch.empty(L_WINDOW, DIT_HEADS * HEAD_DIM, dtype=torch.float16, device=device) for _ in dq]
        scratch = torch.empty(L_WINDOW, 2 * DIT_HEADS * HEAD_DIM, dtype=torch.float16, device=device)

        def dit_step():
            for q, o in zip(dq, dout):
                F.rope_attention(q, 1, DIT_HEADS, cos, sin, out=o, scratch=scratch, balanced=bal)

        dsteps = max(3, args.steps // 2)
        dper: list[float] = []
        dms = time_graph(dit_step, dsteps, args.warmup, device, dist_on, per_step=dper)
        F.check_status(device)
        # the same 8 layers when the QKV projection's epilogue has applied RoPE
        # (linear_rope): the attention reads q | k rotated, no RoPE pass
        drot = [F.rope_split(q, L_WINDOW, DIT_HEADS, cos, sin) for q in dq]
        drot = [torch.cat([r[0], r[1], r[2]], 1).contiguous() for r in drot]

        def dit_rot_step():
            for q, o in zip(drot, dout):
                F.rotated_attention(q, 1, DIT_HEADS, out=o, balanced=bal)

        rms = time_graph(dit_rot_step, dsteps, args.warmup, device, dist_on)
        F.check_status(device)
        del drot
        dit = (dms, dsteps, statistics.median(dper), rms)
        dit_inputs = (dq, cos, sin, dout)

    el = e2e_layer_leg(max(3, min(args.steps, 30)), 3, device, dist_on)
    c3 = None if args.no_config3 else config3_leg(args, rank, device, dist_on, bal)
    tp = None if args.no_throughput else throughput_leg(args, rank, world, device, dist_on, bal)

    vals = [ms, e2e_ms, copy["h2d_ms"], copy["d2h_ms"], copy["both_ms"], dit[0] if dit else 0.0,
            c3["ms"] if c3 else 0.0, tp["ms"] if tp else 0.0, dit[3] if dit else 0.0, el["ms"]]
    t = torch.tensor(vals, dtype=torch.float64, device=device)
    if dist_on:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms, e2e_ms, h2d_ms, d2h_ms, both_ms, dms, c3_ms, tp_ms, rms, el_ms = (float(x) for x in t.tolist())

    if rank == 0:
        K = args.steps
        windows = K * world
        value = ms / windows                      # whole-job ms per window
        per_launch_ms = ms / (K * ENC_LAYERS)     # each GPU runs its launches back to back
        achieved = FLOP_ENC_LAYER / (per_launch_ms * 1e-3) / 1e12
        peak, peak_note = measured_peak()
        traffic = ncu_traffic()
        e2e_value = e2e_ms / (e2e_steps * world)
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": round(ms / K, 4), "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic (seeded random-init weights / inputs of the config-2 shapes)",
            "config": config_dict(world),
            "median_ms_per_step": round(med, 4),
            "tflops": round(FLOP_ENC_LAYER * ENC_LAYERS * windows / (ms * 1e-3) / 1e12, 1),
            "pct_dense_fp16_peak": round(100 * achieved / DATASHEET_DENSE_FP16_TFLOPS, 1),
            "windows_per_s": round(windows / (ms * 1e-3), 2),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": "fds::attn_fwd_kernel<__half, true> (one encoder layer, 147.456 GFLOP)",
                         "peak_note": peak_note},
            "e2e": {"value": round(e2e_value, 4), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "note": "public API flexrel_attention, pinned host QKV/rel in, context out, per step",
                    "copy_roofline": {
                        "h2d_gbs_per_gpu": round(h2d / (h2d_ms * 1e-3) / 1e9, 1),
                        "d2h_gbs_per_gpu": round(d2h / (d2h_ms * 1e-3) / 1e9, 1),
                        "both_ms_per_step": round(both_ms, 4),
                        "bound_ms_per_window": round(both_ms / world, 4),
                        "frac": round((both_ms / world) / e2e_value, 3),
                        "note": "the same pinned buffers copied with no kernel (h2d alone, d2h alone, both at "
                                "once on every rank); e2e is copy-bound when frac is near 1"}},
            "gpu_launches": K * ENC_LAYERS * world,
            "clocks": clocks.summary(),
            "e2e_layer": {
                "value": round(el_ms / (el["steps"] * world), 4), "unit": UNIT,
                "h2d_bytes_per_step": el["h2d"], "d2h_bytes_per_step": el["d2h"],
                "gpu_launches_per_window": 3 * ENC_LAYERS,
                "note": "the 13 attention layers with their projections on the device (linear -> "
                        "flexrel_attention -> accumulate per layer, weights resident, one CUDA graph per "
                        "window); only the fp32 residual of the window crosses the host link, in and out, "
                        "each step, overlapped with the neighbouring windows' layers; per layer this "
                        "library's QKV GEMM, attention and out-projection GEMM plus torch's fp16 cast of x"},
        }
        if dit:
            dsteps = dit[1]
            dper_ms = dms / (dsteps * DIT_LAYERS)
            line["dit"] = {"workload": "config4: 8-layer DiT RoPE attention, L=6000, 12 x 64 heads",
                           "ms_per_window": round(dms / (dsteps * world), 4),
                           "ms_per_window_per_gpu": round(dms / dsteps, 4),
                           "median_ms_per_window_per_gpu": round(dit[2], 4),
                           "tflops": round(FLOP_DIT_LAYER / (dper_ms * 1e-3) / 1e12, 1),
                           "frac": round(FLOP_DIT_LAYER / (dper_ms * 1e-3) / 1e12 / peak, 4),
                           "steps": dsteps, "launches_per_window": 2 * DIT_LAYERS,
                           "rotated_ms_per_window": round(rms / (dsteps * world), 4),
                           "rotated_note": "q | k rotated by the QKV projection's epilogue (linear_rope): "
                                           "8 attention launches, no RoPE pass"}
        if c3:
            per_batch = c3_ms / c3["steps"]
            line["config3"] = {
                "workload": "config3: batch of 8 windows, lengths U(3.2, 120) s (seed 3), 10 s buckets, "
                            "padded to the longest bucket, kv_len key padding, 13 layers",
                "frames": c3["frames"], "buckets": c3["buckets"], "padded_len": c3["Lmax"],
                "ms_per_batch": round(per_batch, 4), "median_ms_per_batch": round(c3["median"], 4),
                "batches_per_s": round(world / (per_batch * 1e-3), 2),
                "credited_tflops": round(c3["credited"] * world / (per_batch * 1e-3) / 1e12, 1),
                "credited_rule": "sum_b 13*4*16*64*L_b*kv_len_b (L_b the window's own bucket)",
                "computed_tflops": round(c3["computed"] * world / (per_batch * 1e-3) / 1e12, 1),
                "steps": c3["steps"]}
        if tp:
            sweep_ms = tp_ms / tp["steps"]
            line["throughput"] = {
                "workload": "config5: 64 windows x (13-layer encoder rel-bias attention + 8-layer DiT RoPE "
                            "attention), L=6000, windows g, g+N, ... on rank g, no collectives",
                "windows": 64, "windows_per_gpu": tp["windows_here"], "n_gpus": world,
                "ms_per_sweep": round(sweep_ms, 3), "median_ms_per_sweep_rank0": round(tp["median"], 3),
                "windows_per_s": round(64 / (sweep_ms * 1e-3), 2),
                "tflops": round(64 * (ENC_LAYERS * FLOP_ENC_LAYER + DIT_LAYERS * FLOP_DIT_LAYER)
                                / (sweep_ms * 1e-3) / 1e12, 1),
                "steps": tp["steps"], "clocks_rank0": tp["clocks"],
                "timing": "one CUDA graph per rank per sweep; max over ranks of the device time"}
        if world == 1 and not args.no_linear:
            line["linear"] = linear_leg(device)
        if world == 1 and not args.no_cpu_baseline:
            cms, info = cpu_layer_ms_per_window(threads=os.cpu_count())
            line["cpu_baseline"] = {"value": round(cms, 1), "unit": UNIT, "cores": info["cores"],
                                    "kind": info["kind"], "sample": info["sample"]}
        if world == 1 and not args.no_reference_gpu:
            line["reference_gpu"] = reference_gpu_leg(qkvs, rels, outs, dit_inputs, device)
        print(json.dumps(line), flush=True)

    if dist_on:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_case(args) -> None:
    """Small profiling case for ncu: one layer's kernel, W + K eager launches."""
    import fastdialoguesidon_b200 as F

    device = torch.device("cuda", 0)
    bal = args.schedule == "auto"
    gen = torch.Generator(device=device).manual_seed(7)
    if args.case == "qkv":
        x = torch.randn(L_WINDOW, ENC_HEADS * HEAD_DIM, generator=gen, device=device).half()
        w = (torch.randn(3 * ENC_HEADS * HEAD_DIM, ENC_HEADS * HEAD_DIM, generator=gen, device=device) * 0.02).half()
        b = (torch.randn(3 * ENC_HEADS * HEAD_DIM, generator=gen, device=device) * 0.02).half()
        out = torch.empty(L_WINDOW, 3 * ENC_HEADS * HEAD_DIM, dtype=torch.float16, device=device)
        fn, flop = (lambda: F.linear(x, w, b, out=out)), 2.0 * L_WINDOW * x.shape[1] * w.shape[0]
    elif args.case == "ropeqkv":
        hid = DIT_HEADS * HEAD_DIM
        x = torch.randn(L_WINDOW, hid, generator=gen, device=device).half()
        w = (torch.randn(3 * hid, hid, generator=gen, device=device) * 0.02).half()
        b = (torch.randn(3 * hid, generator=gen, device=device) * 0.02).half()
        cos, sin = F.rope_tables(L_WINDOW, device)
        out = torch.empty(L_WINDOW, 3 * hid, dtype=torch.float16, device=device)
        fn = lambda: F.linear_rope(x, w, b, cos, sin, L_WINDOW, DIT_HEADS, out=out)  # noqa: E731
        flop = 2.0 * L_WINDOW * hid * 3 * hid
    elif args.case == "accum":
        hid = ENC_HEADS * HEAD_DIM
        a = torch.randn(L_WINDOW, hid, generator=gen, device=device).half()
        w = (torch.randn(hid, hid, generator=gen, device=device) * 0.02).half()
        x = torch.zeros(L_WINDOW, hid, device=device)
        fn, flop = (lambda: F.accumulate(x, a, w)), 2.0 * L_WINDOW * hid * hid
    elif args.case == "enc1":
        qkv = (torch.randn(L_WINDOW, 3 * ENC_HEADS * HEAD_DIM, generator=gen, device=device) * 0.64).half()
        rel = (torch.randn(73, HEAD_DIM, generator=gen, device=device) * 0.02).half()
        out = torch.empty(L_WINDOW, ENC_HEADS * HEAD_DIM, dtype=torch.float16, device=device)
        fn, flop = (lambda: F.flexrel_attention(qkv, 1, ENC_HEADS, rel, out=out, balanced=bal)), FLOP_ENC_LAYER
    else:
        qkv = (torch.randn(L_WINDOW, 3 * DIT_HEADS * HEAD_DIM, generator=gen, device=device) * 0.55).half()
        cos, sin = F.rope_tables(L_WINDOW, device)
        out = torch.empty(L_WINDOW, DIT_HEADS * HEAD_DIM, dtype=torch.float16, device=device)
        scratch = torch.empty(L_WINDOW, 2 * DIT_HEADS * HEAD_DIM, dtype=torch.float16, device=device)
        fn, flop = (lambda: F.rope_attention(qkv, 1, DIT_HEADS, cos, sin, out=out, scratch=scratch,
                                             balanced=bal)), FLOP_DIT_LAYER
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        fn()
    end.record()
    torch.cuda.synchronize(device)
    F.check_status(device)
    ms = start.elapsed_time(end) / max(args.steps, 1)
    print(json.dumps({"case": args.case, "ms_per_launch": round(ms, 4),
                      "tflops": round(flop / (ms * 1e-3) / 1e12, 1)}), flush=True)


def main():
    args = parse_args()
    if args.case:
        run_case(args)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world == 1 and args.gpus > 1:
        raise SystemExit("for --gpus > 1 launch under torch.distributed.run (one process per GPU)")
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
