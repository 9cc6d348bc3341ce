#!/usr/bin/env python
"""Benchmark of the B200 MoE expert-layer forward (tokens/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N=1: the full single-GPU layer (T=16384 tokens, H=7168, E=256 experts, top-8,
ffn=2048 SwiGLU, Zipf-skewed router logits). N>1 (launched by torchrun, one
rank per GPU): the expert-parallel layer, T=16384 tokens per GPU, experts
split evenly, NCCL all-to-all dispatch/combine. Prints one JSON line on rank 0.

  value  tokens/s of the whole job, inputs resident in HBM, CUDA-event timed
         (max over ranks), weak scaling;
  e2e    the same through the public layer API with host buffers: pinned
         H2D of x and logits and D2H of the output inside every timed step;
  roofline  the dominant kernel (fc1 grouped GEMM, tcgen05) against the
         measured bf16 peak; stages  per-stage device times;
  cpu_baseline  the reference's layer chain restated in torch on the CPU
         (oracle/torch_ref.py: the cases' Model.forward ops) on this host's
         cores over a bounded token sample (rank 0, N=1 only);
  checked  the measured configuration's maps, permuted rows and sampled
         token outputs against a torch reference, after the timed windows.
--impl reference times that CPU restatement alone (the reference's own case
files cannot travel to the GPU host; its ops are restated op for op).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "1188b-reference-kernels_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer fwd tokens/s"
UNIT = "tokens/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def resolve_transport(transport: str, world: int) -> str:
    if transport != "auto":
        return transport
    return "fused_dedup" if world <= 4 else "fused"


def overlap_chunks(a, world: int) -> int:
    return a.overlap_chunks if resolve_transport(a.transport, world) == "fused" else 1


def device_error(layer) -> int:
    return layer.device_error() if hasattr(layer, "device_error") else layer.plan.device_error()


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--tokens", type=int, default=16384, help="tokens per GPU")
    ap.add_argument("--hidden", type=int, default=7168)
    ap.add_argument("--experts", type=int, default=256)
    ap.add_argument("--ffn", type=int, default=2048)
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--routing", choices=["zipf", "uniform"], default="zipf")
    ap.add_argument("--cpu-tokens", type=int, default=4096,
                    help="token sample of the CPU baseline (per step for --impl reference)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-check", action="store_true",
                    help="skip the post-timing correctness check of the expert-parallel layer "
                         "(the single-GPU layer is always checked)")
    ap.add_argument("--settle-s", type=float, default=2.0,
                    help="untimed layer steps after the warm-up, in seconds of GPU time, so "
                         "the timed windows run at the power-capped sustained clock")
    ap.add_argument("--placement", choices=["balanced", "contiguous"], default="balanced",
                    help="EP expert placement: load-balanced (E/G experts per GPU, chosen from "
                         "the routing of the benchmark's own logits) or contiguous id ranges")
    ap.add_argument("--transport", choices=["auto", "fused", "fused_dedup", "fused_pull", "peer",
                                            "nccl"],
                    default="auto",
                    help="EP row exchange: dispatch/combine kernels on peer memory (fused_dedup: "
                         "a token row crosses NVLink once per destination rank), IPC-mapped "
                         "buffers + copy engines, or NCCL all-to-all; auto = fused_dedup up to "
                         "4 GPUs, fused at 8 (where tokens reach 6.8 of 8 ranks and the "
                         "receiver's expansion copy outweighs the saved rows)")
    ap.add_argument("--overlap-chunks", type=int, default=1,
                    help="EP with --transport fused: split the local experts into this many "
                         "chunks and dispatch chunk c+1 over NVLink while chunk c's GEMMs run "
                         "(1 = no overlap)")
    ap.add_argument("--workload", choices=["layer", "router_gemm", "backward", "wgrad",
                                           "rowcopy", "dense_gemm"],
                    default="layer",
                    help="layer: the MoE expert-layer forward (the headline); router_gemm: the "
                         "router gate GEMM that produces its logits; backward: the layer's "
                         "grouped dgrad and wgrad GEMMs; wgrad: the grouped wgrad alone at "
                         "--wgrad-shape; rowcopy: the layer's permute and weighted combine "
                         "alone, with no expert weights on the device (one GPU); dense_gemm: "
                         "the expert GEMMs on one dense group of tokens*topk rows against "
                         "cuBLAS (torch.matmul) on the same operands (one GPU)")
    ap.add_argument("--wgrad-shape", default="40,4096,5120,8192",
                    help="G,T,N,K of --workload wgrad (uniform groups; default: the traced "
                         "shape of kernel_cases/case09_moe_grouped_gemm_fc1_wgrad.py)")
    ap.add_argument("--router-shape", default="16384,8192,320",
                    help="M,K,N of the router GEMM (tokens, hidden, experts)")
    return ap.parse_args()


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def config_dict(a, world):
    return {"workload": "moe_layer_fwd" if world == 1 else "moe_layer_fwd_ep",
            "tokens_per_gpu": a.tokens, "hidden": a.hidden, "experts": a.experts,
            "topk": a.topk, "ffn": a.ffn, "routing": a.routing,
            "parallelism": f"ep{world}" if world > 1 else "single",
            **({"ep_transport": resolve_transport(a.transport, world),
                "ep_placement": a.placement,
                "ep_overlap_chunks": overlap_chunks(a, world)} if world > 1 else {}),
            "l2": "no flush: every step streams >22 GB of expert weights and 0.25 GB of "
                  "activations, both larger than the 126 MB L2"}


def zipf_bias(e, routing):
    import torch
    if routing != "zipf":
        return torch.zeros(e)
    g = torch.Generator().manual_seed(7)
    r = torch.randperm(e, generator=g).float() + 1.0
    return -1.5 * torch.log(r)


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock/throttle sampling (50 ms) around the measurement.

    Samples are time-stamped on the host. Each timed window is marked with a
    label (device-only or e2e); the summary covers the samples inside all
    marked windows (or the whole run when no sample falls inside one) and
    gives the median SM clock of every label separately.
    """
    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, device_index):
        self.device_index = device_index
        self.proc = None
        self.path = None
        self.windows = []  # (label, t0, t1)

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                   "-lms", "50", "-i", str(self.device_index)]
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
            t0 = time.time()
            while time.time() - t0 < 10 and Path(self.path).stat().st_size == 0:
                time.sleep(0.05)
        except Exception:
            self.proc = None

    def mark(self, t0, t1, label="device"):
        self.windows.append((label, t0, t1))

    @staticmethod
    def _num(v):
        try:
            return float(v)
        except ValueError:
            return None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                ts = time.mktime(time.strptime(parts[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                ts += float("0." + parts[0].split(".")[1]) if "." in parts[0] else 0.0
            except Exception:
                ts = None
            rows.append((ts, parts))
        os.unlink(self.path)
        if not rows:
            return None

        def inside(r, w):
            return r[0] is not None and w[1] - 0.05 <= r[0] <= w[2] + 0.05

        per = {}
        for w in self.windows:
            per.setdefault(w[0], []).extend(r for r in rows if inside(r, w))
        timed = [r for r in rows if any(inside(r, w) for w in self.windows)]
        scope = "timed windows"
        if not timed:
            timed, scope = rows, "bench run"
        sm = [v for v in (self._num(p[1]) for _, p in timed) if v is not None]
        mx = [v for v in (self._num(p[2]) for _, p in timed) if v is not None]
        pw = [v for v in (self._num(p[3]) for _, p in timed) if v is not None]
        reasons = sorted({n for _, p in timed for n, v in zip(self.NAMES, p[5:9]) if v == "Active"})
        out = {"sm_mhz": statistics.median(sm) if sm else None,
               "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
               "samples": len(timed), "scope": scope,
               "power_w_max": max(pw) if pw else None}
        wins = {}
        for label, rs in per.items():
            v = [x for x in (self._num(p[1]) for _, p in rs) if x is not None]
            wins[label] = {"sm_mhz": statistics.median(v) if v else None, "samples": len(v)}
        if wins:
            out["windows"] = wins
        return out


class EnergyMeter:
    """The GPU's cumulative energy counter (NVML, millijoules), read around each
    timed window: joules per step is the figure that decides speed when the
    step runs at the board's power cap. Reading the counter changes nothing."""

    def __init__(self, device_index):
        self.h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(int(device_index))
            self.read()
        except Exception:
            self.h = None

    def read(self):
        if self.h is None:
            return None
        try:
            return float(self._nvml.nvmlDeviceGetTotalEnergyConsumption(self.h))
        except Exception:
            self.h = None
            return None


# --------------------------------------------------------------------------- CPU port
def cpu_layer_setup(a, tokens, seed=0):
    """Inputs of one bounded CPU sample of the layer: `tokens` tokens with the
    bench's shapes and Zipf routing, and bf16 weights for the experts those
    tokens reach (the others are never read). Each expert's weights are a
    distinct window of one seeded N(0,1) pool scaled by 0.02: generating
    ~90 x 88 MB of fresh normals per run would take longer than the sample,
    and the values do not change the work."""
    import torch
    from oracle import torch_ref as tr
    h, e, f, k = a.hidden, a.experts, a.ffn, a.topk
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(tokens, h, generator=g).to(torch.bfloat16)
    lg = torch.randn(tokens, e, generator=g)
    bias = zipf_bias(e, a.routing)
    rmap, _ = tr.route(lg, bias, k)
    hit = rmap.any(dim=0).nonzero().flatten().tolist()
    torch.manual_seed(seed)
    pool = torch.randn(1 << 26)
    n1, n2 = 2 * f * h, h * f

    def window(i, n):
        off = (i * 1000003) % (pool.numel() - n // 2)
        return pool[off:off + n // 2].repeat(2)[:n].mul(0.02).to(torch.bfloat16)

    w1 = {i: window(2 * i, n1).view(2 * f, h) for i in hit}
    w2 = {i: window(2 * i + 1, n2).view(h, f) for i in hit}
    return x, lg, bias, w1, w2


def cpu_layer_time(a, setup):
    """Seconds for one forward of the torch CPU restatement of the
    reference's layer chain (oracle/torch_ref.py) on one sample."""
    from oracle import torch_ref as tr
    x, lg, bias, w1, w2 = setup
    t0 = time.perf_counter()
    tr.layer(x, lg, bias, w1.__getitem__, w2.__getitem__, a.topk)
    return time.perf_counter() - t0


def cpu_sample_desc(a):
    return (f"{a.cpu_tokens} tokens per step of the {a.tokens}-token layer (same H/E/F/top-k, "
            f"{a.routing} routing): the reference's torch chain restated on the CPU "
            f"(sort top-k, case12 cumsum row_id_map, case17 index_copy_ permute, case03/case04 "
            f"bf16 torch.mm per expert, SwiGLU, weighted case15 index_add_ combine), bf16 "
            f"weights of every expert the sample reaches")


def use_all_cores():
    """Lets the CPU legs use every host core (torchrun sets OMP_NUM_THREADS=1)."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    import numpy  # noqa: F401  (load BLAS so its pool can be resized)
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=n)
    except Exception:
        pass
    import torch
    torch.set_num_threads(n)
    return n


def cpu_threads():
    import torch
    return torch.get_num_threads()


def cpu_baseline_sample(a):
    """The cpu_baseline object of the GPU arm's line: the reference's layer
    chain on this host's cores, one warm-up and two timed runs of one sample."""
    use_all_cores()
    setup = cpu_layer_setup(a, a.cpu_tokens)
    cpu_layer_time(a, setup)
    dt = min(cpu_layer_time(a, setup) for _ in range(2))
    return {"value": a.cpu_tokens / dt, "unit": UNIT, "cores": cpu_threads(), "kind": "port",
            "sample": cpu_sample_desc(a)}


def check_ep(layer, x, logits, bias, w, k, placement, world, rank, dev):
    """Expert-parallel check (outside the timed windows): every rank's EP output
    equals, bit for bit, the single-GPU layer run on that rank with all
    experts' weights (gathered from the ranks, slot order) and the same
    placement; the single-GPU forward also passes check_layer. Collective:
    every rank calls it."""
    import torch
    import torch.distributed as dist
    import moe_b200
    out_ep = layer(x, logits)
    el = w.w1.shape[0]
    w1_all = torch.empty((world * el,) + tuple(w.w1.shape[1:]), dtype=w.w1.dtype, device=dev)
    w2_all = torch.empty((world * el,) + tuple(w.w2.shape[1:]), dtype=w.w2.dtype, device=dev)
    dist.all_gather_into_tensor(w1_all, w.w1.contiguous())
    dist.all_gather_into_tensor(w2_all, w.w2.contiguous())
    full = moe_b200.MoELayer(moe_b200.MoEWeights(w1_all, w2_all), topk=k, expert_bias=bias,
                             placement=placement)
    out, mid = full.forward(x, logits, return_intermediates=True)
    torch.cuda.synchronize()
    same = bool(torch.equal(out, out_ep))
    chk = check_layer(out, mid, x, logits, bias, w1_all, w2_all, k, placement)
    derr = {"ep": device_error(layer), "single": full.plan.device_error(),
            "permute": moe_b200.permute_device_error(dev)}
    mine = {"rank": rank, "ep_equals_single_gpu": same, "checks_ok": bool(chk["ok"]),
            "failed": [k for k, v in chk.items() if v is False],
            "max_abs_err": chk.get("max_abs_err"),
            "device_errors": {k: v for k, v in derr.items() if v}}
    mine["ok"] = same and chk["ok"] and not mine["device_errors"]
    every = [None] * world
    dist.all_gather_object(every, mine)
    del out, mid, full, w1_all, w2_all, out_ep
    torch.cuda.empty_cache()
    chk.update({"ok": all(r["ok"] for r in every), "ranks": every,
                "scope": "every rank's tokens vs the single-GPU layer bit for bit, and the "
                         "torch reference on the single-GPU forward (ok = all ranks); rank "
                         "0's details shown"})
    return chk


def run_reference_arm(a, world, rank):
    if rank != 0:
        return
    use_all_cores()
    setup = cpu_layer_setup(a, a.cpu_tokens, seed=1)
    for _ in range(a.warmup):
        cpu_layer_time(a, setup)
    times = [cpu_layer_time(a, setup) for _ in range(a.steps)]
    total = sum(times)
    value = a.cpu_tokens * a.steps / total
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": 1e3 * total / a.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "impl": "reference", "config": config_dict(a, world),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu_threads(), "kind": "port",
                             "sample": cpu_sample_desc(a)},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- router GEMM
def run_router_gemm(a):
    """Router gate GEMM, logits [M,N] fp32 = x [M,K] bf16 @ w [N,K] bf16 ^T, at the
    traced shape of kernel_cases/case38_ref_musa_asm_bf16_ssgemm_nt_320x256.py
    (M=16384, K=8192, N=320). One GPU; x (268 MB) is larger than L2, so no flush."""
    m, kk, n = (int(v) for v in a.router_shape.split(","))
    flops = 2.0 * m * n * kk
    nbytes = m * kk * 2 + n * kk * 2 + m * n * 4
    cfg = {"workload": "router_gemm", "tokens": m, "hidden": kk, "experts": n,
           "l2": "no flush: x is larger than the 126 MB L2"}
    metric, unit = "router GEMM tokens/s", "tokens/s"
    if a.impl == "reference":
        use_all_cores()
        import numpy as np
        sys.path.insert(0, str(ROOT))
        from oracle import moe_oracle as orc
        rows = 256
        rng = np.random.default_rng(0)
        xs = rng.standard_normal((rows, kk), dtype=np.float32)
        ws = rng.standard_normal((n, kk), dtype=np.float32)
        xu, wu = orc.f32_to_bf16(xs), orc.f32_to_bf16(ws)
        for _ in range(a.warmup):
            orc.router_logits(xu, wu)
        t0 = time.perf_counter()
        for _ in range(a.steps):
            orc.router_logits(xu, wu)
        dt = (time.perf_counter() - t0) / a.steps
        value = rows / dt
        line = {"metric": metric, "value": value, "unit": unit, "n_gpus": 1, "steps": a.steps,
                "warmup": a.warmup, "ms_per_step": 1e3 * dt * m / rows, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "impl": "reference", "config": cfg,
                "cpu_baseline": {"value": value, "unit": unit, "cores": cpu_threads(),
                                 "kind": "port", "sample": f"{rows} of {m} rows, numpy fp32"},
                "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    import torch
    import moe_b200
    from moe_b200 import _lib
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    moe_b200.load_library()
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    x = torch.randn(m, kk, device=dev, generator=g).to(torch.bfloat16)
    w = torch.randn(n, kk, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(m, n, dtype=torch.float32, device=dev)
    sampler = ClockSampler(os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0])
    sampler.start()
    for _ in range(a.warmup):
        moe_b200.router_logits(x, w, out=out)
    torch.cuda.synchronize()
    launches0 = _lib.launch_count
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    wall0 = time.time()
    ev[0].record()
    for _ in range(a.steps):
        moe_b200.router_logits(x, w, out=out)
    ev[1].record()
    torch.cuda.synchronize()
    sampler.mark(wall0, time.time())
    launches = _lib.launch_count - launches0
    t = ev[0].elapsed_time(ev[1]) / 1e3 / a.steps

    def timed(fn):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / a.steps * 1e3  # us

    # The whole router (gate GEMM + softmax/top-8/renorm -> routing map + probs):
    # one fused kernel vs the GEMM followed by the standalone router kernel.
    fused = {}
    if n % 32 == 0 and n <= 512:
        fused["router_us"] = round(timed(lambda: moe_b200.router_gemm_topk(
            x, w, 8, "softmax", True, None, outputs="maps")), 2)
        fused["gemm_logits_only_us"] = round(timed(lambda: moe_b200.router_gemm_topk(
            x, w, 8, outputs="none", return_logits=True)), 2)
        fused["unfused_router_us"] = round(timed(lambda: moe_b200.router_topk(
            moe_b200.router_logits(x, w, out=out), 8, "softmax", True, outputs="maps")), 2)
        fused["device_error"] = moe_b200.router_device_error(dev)
    # cuBLAS on the same operands (torch.matmul, bf16 out; fp32 out where
    # this torch build offers it), for the GEMM alone
    cb = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    fused["cublas_bf16_out_us"] = round(timed(lambda: torch.matmul(x, w.t(), out=cb)), 2)
    try:
        fused["cublas_fp32_out_us"] = round(timed(
            lambda: torch.mm(x, w.t(), out_dtype=torch.float32)), 2)
    except (TypeError, RuntimeError):
        pass
    clocks = sampler.stop()
    peaks, peak_kind = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    achieved = flops / t / 1e12
    line = {"metric": metric, "value": m / t, "unit": unit, "n_gpus": 1, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (N(0,1))",
            "config": cfg,
            "roofline": {"bound": "tensor", "kernel": "grouped_gemm, one group, fp32 epilogue",
                         "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4), "traffic": None},
            "hbm": {"achieved_gbs": round(nbytes / t / 1e9, 1), "peak_gbs": hbm,
                    "frac": round(nbytes / t / 1e9 / hbm, 4), "bytes": nbytes},
            "peak_kind": f"bf16 burst, of {peak_kind}",
            "cpu_baseline": None, "e2e": None, "gpu_launches": launches, "clocks": clocks,
            "fused_router": fused}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- grouped backward
def run_backward(a):
    """The layer's grouped-GEMM backward at the bench workload, group sizes from
    the layer's own routing: fc2 dgrad dh = dy @ W2[e] ([R,H] x [H,F]), fc2
    wgrad dW2[e] = dy[seg]^T @ h[seg], fc1 dgrad dx = dz @ W1[e] ([R,2F] x
    [2F,H]) and fc1 wgrad dW1[e] = dz[seg]^T @ x[seg]. dgrad uses the weights
    as stored (staged MN-major); wgrad writes every expert's gradient."""
    import torch
    import moe_b200
    from moe_b200 import _lib
    t, h, e, f, k = a.tokens, a.hidden, a.experts, a.ffn, a.topk
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    moe_b200.load_library()
    g = torch.Generator(device=dev)
    g.manual_seed(1000)
    logits = torch.randn(t, e, device=dev, generator=g)
    r = moe_b200.router_topk(logits, k, "softmax", True, zipf_bias(e, a.routing).to(dev),
                             outputs="maps")
    counts = moe_b200.row_id_map(r.routing_map, want_et=False).counts
    rows = t * k
    w = moe_b200.MoEWeights.random(e, h, f, dev, seed=77)
    dy = torch.randn(rows, h, device=dev, generator=g).to(torch.bfloat16)
    dz = torch.randn(rows, 2 * f, device=dev, generator=g).to(torch.bfloat16)
    xp = torch.randn(rows, h, device=dev, generator=g).to(torch.bfloat16)
    hm = torch.randn(rows, f, device=dev, generator=g).to(torch.bfloat16)
    plan = moe_b200.GroupedGemmPlan(e, dev).from_splits(counts)
    dh = torch.empty(rows, f, dtype=torch.bfloat16, device=dev)
    dx = torch.empty(rows, h, dtype=torch.bfloat16, device=dev)
    dw2 = torch.empty(e, h, f, dtype=torch.bfloat16, device=dev)
    dw1 = torch.empty(e, 2 * f, h, dtype=torch.bfloat16, device=dev)
    names = ["fc2_dgrad", "fc2_wgrad", "fc1_dgrad", "fc1_wgrad"]
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]

    def step():
        ev[0].record()
        moe_b200.grouped_gemm(dy, w.w2, plan=plan, out=dh, w_layout="KN")
        ev[1].record()
        moe_b200.grouped_wgrad(dy, hm, counts, out=dw2)
        ev[2].record()
        moe_b200.grouped_gemm(dz, w.w1, plan=plan, out=dx, w_layout="KN")
        ev[3].record()
        moe_b200.grouped_wgrad(dz, xp, counts, out=dw1)
        ev[4].record()

    sampler = ClockSampler(os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0])
    sampler.start()
    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    assert plan.device_error() == 0
    launches0 = _lib.launch_count
    wall0 = time.time()
    tot = [0.0] * len(names)
    for _ in range(a.steps):
        step()
        torch.cuda.synchronize()
        for i in range(len(names)):
            tot[i] += ev[i].elapsed_time(ev[i + 1]) / 1e3
    sampler.mark(wall0, time.time())
    launches = _lib.launch_count - launches0
    clocks = sampler.stop()
    # The whole layer backward (MoELayer.backward: combine backward, the four
    # GEMMs, SwiGLU backward, permute backward) on the same routing.
    del dy, dz, xp, hm, dh, dx, dw2, dw1
    layer = moe_b200.MoELayer(w, topk=k, expert_bias=zipf_bias(e, a.routing).to(dev))
    x = torch.randn(t, h, device=dev, generator=g).to(torch.bfloat16)
    go = torch.randn(t, h, device=dev, generator=g).to(torch.bfloat16)
    _, ctx = layer.forward(x, logits, save_for_backward=True)
    for _ in range(max(a.warmup, 1)):
        layer.backward(go, ctx)
    torch.cuda.synchronize()
    lb0, lb1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    lb0.record()
    for _ in range(a.steps):
        layer.backward(go, ctx)
    lb1.record()
    torch.cuda.synchronize()
    assert layer.plan.device_error() == 0
    layer_bwd_ms = lb0.elapsed_time(lb1) / a.steps
    sec = {n: v / a.steps for n, v in zip(names, tot)}
    flops = {"fc2_dgrad": 2.0 * rows * h * f, "fc2_wgrad": 2.0 * rows * h * f,
             "fc1_dgrad": 2.0 * rows * 2 * f * h, "fc1_wgrad": 2.0 * rows * 2 * f * h}
    step_s = sum(sec.values())
    peaks, peak_kind = load_peaks()
    peak = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    ach = sum(flops.values()) / step_s / 1e12
    wg_bytes = (e * h * f + e * 2 * f * h) * 2  # every expert's gradient is written
    line = {"metric": "grouped GEMM backward tokens/s", "value": t / step_s, "unit": "tokens/s",
            "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": step_s * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (N(0,1) activations/gradients, N(0,0.02) weights, Zipf routing)",
            "config": {"workload": "grouped_gemm_backward", "tokens": t, "hidden": h,
                       "experts": e, "topk": k, "ffn": f, "routing": a.routing,
                       "l2": "no flush: every step streams >22 GB of weights and gradients"},
            "roofline": {"bound": "tensor", "kernel": "grouped dgrad + wgrad (fc1 + fc2)",
                         "achieved": round(ach, 2), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(ach / peak, 4), "traffic": None},
            "stages_ms": {n: round(v * 1e3, 4) for n, v in sec.items()},
            "stage_tflops": {n: round(flops[n] / sec[n] / 1e12, 1) for n in names},
            "wgrad_write_gbs": round(wg_bytes / (sec["fc1_wgrad"] + sec["fc2_wgrad"]) / 1e9, 1),
            "layer_backward_ms": round(layer_bwd_ms, 3),
            "hbm_peak_gbs": hbm, "peak_kind": f"bf16 sustained, of {peak_kind}",
            "cpu_baseline": None, "e2e": None, "gpu_launches": launches, "clocks": clocks}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- grouped wgrad alone
def run_rowcopy(a):
    """The layer's two row kernels at the bench shape without the GEMMs: the
    permute of x [T,H] into T*k expert-major rows and the gate-weighted
    combine of T*k rows back to [T,H], routing from the bench's own logits.
    Only x, the permuted rows, the maps and the output are on the device
    (about 4.3 GB), so the kernels can be profiled at the layer's size.
    Inputs (1.9 GB of rows) are larger than L2."""
    import torch
    import moe_b200
    from moe_b200 import _lib
    t, h, e, k = a.tokens, a.hidden, a.experts, a.topk
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    moe_b200.load_library()
    g = torch.Generator(device=dev)
    g.manual_seed(1000)
    x = torch.randn(t, h, device=dev, generator=g).to(torch.bfloat16)
    logits = torch.randn(t, e, device=dev, generator=g)
    r = moe_b200.router_topk(logits, k, "softmax", True, zipf_bias(e, a.routing).to(dev),
                             outputs="all")
    rim = moe_b200.row_id_map(r.routing_map, want_et=False)
    rows = t * k
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]

    def step():
        ev[0].record()
        xp_, _ = moe_b200.permute(x, rim.map_te, None, num_out=rows)
        ev[1].record()
        moe_b200.unpermute(xp_, rim.map_te, r.probs, probs_mode="dense", token_major=True)
        ev[2].record()
        xl, _ = moe_b200.permute(x, rim.map_te, None, num_out=rows, experts=r.topk_idx)
        ev[3].record()
        return xp_, xl

    sampler = ClockSampler(os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0])
    sampler.start()
    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    launches0 = _lib.launch_count
    wall0 = time.time()
    tp = tc = tl = 0.0
    for _ in range(a.steps):
        xa, xb = step()
        torch.cuda.synchronize()
        tp += ev[0].elapsed_time(ev[1]) / 1e3
        tc += ev[1].elapsed_time(ev[2]) / 1e3
        tl += ev[2].elapsed_time(ev[3]) / 1e3
    same = bool(torch.equal(xa, xb))
    sampler.mark(wall0, time.time())
    launches = _lib.launch_count - launches0
    clocks = sampler.stop()
    tp, tc, tl = tp / a.steps, tc / a.steps, tl / a.steps
    perm_bytes = t * h * 2 + rows * h * 2 + t * e * 8
    comb_bytes = rows * h * 2 + t * h * 2 + t * e * 8 + t * e * 4
    peaks, peak_kind = load_peaks()
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    pg, cg = perm_bytes / tp / 1e9, comb_bytes / tc / 1e9
    line = {"metric": "permute + combine tokens/s", "value": t / (tp + tc), "unit": "tokens/s",
            "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": (tp + tc) * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) activations/logits, Zipf expert bias)",
            "config": {"workload": "rowcopy", "tokens": t, "hidden": h, "experts": e, "topk": k,
                       "routing": a.routing, "l2": "no flush: rows (1.9 GB) exceed L2"},
            "roofline": {"bound": "hbm", "kernel": "permute_kernel", "achieved": round(pg, 1),
                         "peak": hbm, "unit": "GB/s", "frac": round(pg / hbm, 4),
                         "traffic": None},
            "permute_ms": round(tp * 1e3, 4), "combine_ms": round(tc * 1e3, 4),
            "permute_from_expert_list": {"ms": round(tl * 1e3, 4),
                                         "gbs": round(perm_bytes / tl / 1e9, 1),
                                         "frac": round(perm_bytes / tl / 1e9 / hbm, 4),
                                         "same_rows": same},
            "permute_gbs": round(pg, 1), "combine_gbs": round(cg, 1),
            "combine_frac": round(cg / hbm, 4), "peak_kind": f"hbm copy, of {peak_kind}",
            "cpu_baseline": None, "e2e": None, "gpu_launches": launches, "clocks": clocks}
    print(json.dumps(line), flush=True)


def run_wgrad(a):
    """dW[g] = dy[seg]^T @ x[seg] over G uniform groups of T rows (N(0,1)
    inputs), timed over --steps calls of the public op."""
    import torch
    import moe_b200
    from moe_b200 import _lib
    gsz, t, n, k = (int(v) for v in a.wgrad_shape.split(","))
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    moe_b200.load_library()
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    dy = torch.randn(t, n, device=dev, generator=g).to(torch.bfloat16)
    x = torch.randn(t, k, device=dev, generator=g).to(torch.bfloat16)
    base, rem = divmod(t, gsz)
    splits = [base + (1 if i < rem else 0) for i in range(gsz)]
    out = torch.empty(gsz, n, k, dtype=torch.bfloat16, device=dev)
    sampler = ClockSampler(os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0])
    sampler.start()
    for _ in range(a.warmup):
        moe_b200.grouped_wgrad(dy, x, splits, out=out)
    torch.cuda.synchronize()
    launches0 = _lib.launch_count
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    wall0 = time.time()
    ev[0].record()
    for _ in range(a.steps):
        moe_b200.grouped_wgrad(dy, x, splits, out=out)
    ev[1].record()
    torch.cuda.synchronize()
    sampler.mark(wall0, time.time())
    launches = _lib.launch_count - launches0
    clocks = sampler.stop()
    sec = ev[0].elapsed_time(ev[1]) / 1e3 / a.steps
    flops = 2.0 * t * n * k
    nbytes = gsz * n * k * 2 + t * (n + k) * 2
    peaks, peak_kind = load_peaks()
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    line = {"metric": "grouped wgrad TFLOP/s", "value": flops / sec / 1e12, "unit": "TFLOP/s",
            "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": sec * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (N(0,1))",
            "config": {"workload": "grouped_wgrad", "groups": gsz, "rows": t, "n": n, "k": k,
                       "l2": "no flush: dW is larger than L2"},
            "roofline": {"bound": "hbm", "kernel": "grouped_wgrad_kernel",
                         "achieved": round(nbytes / sec / 1e9, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(nbytes / sec / 1e9 / hbm, 4), "traffic": None},
            "peak_kind": f"hbm copy, of {peak_kind}",
            "cpu_baseline": None, "e2e": None, "gpu_launches": launches, "clocks": clocks}
    print(json.dumps(line), flush=True)


def run_dense_gemm(a):
    """The expert GEMMs' kernel against cuBLAS on the same dense problems: one
    group of T*k rows through moe_b200.grouped_gemm (fc1 [rows,H]x[2F,H]^T
    with the SwiGLU and the plain epilogue, fc2 [rows,F]x[H,F]^T) and
    torch.matmul on the same operands (cuBLAS), in interleaved windows so both
    see the same power-capped clock. Per arm: median ms per call, TFLOP/s,
    median SM clock of its windows and flops per SM cycle; the outputs of the
    plain fc1 and fc2 are compared bit for bit with cuBLAS's."""
    import statistics
    import torch
    import moe_b200
    from moe_b200 import _lib, ops
    t, h, f, k = a.tokens, a.hidden, a.ffn, a.topk
    rows = t * k
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    moe_b200.load_library()
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    x = torch.randn(rows, h, device=dev, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(1, 2 * f, h, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(1, h, f, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    hm = torch.randn(rows, f, device=dev, generator=g).to(torch.bfloat16)
    plan = ops.GroupedGemmPlan(1, dev).from_splits(torch.tensor([rows], dtype=torch.int32))
    o_sw = torch.empty(rows, f, dtype=torch.bfloat16, device=dev)
    o1, c1 = (torch.empty(rows, 2 * f, dtype=torch.bfloat16, device=dev) for _ in range(2))
    o2, c2 = (torch.empty(rows, h, dtype=torch.bfloat16, device=dev) for _ in range(2))
    arms = {
        "fc1_swiglu": lambda: ops.grouped_gemm(x, w1, epilogue="swiglu", plan=plan, out=o_sw),
        "fc1": lambda: ops.grouped_gemm(x, w1, plan=plan, out=o1),
        "fc1_cublas": lambda: torch.matmul(x, w1[0].t(), out=c1),
        "fc2": lambda: ops.grouped_gemm(hm, w2, plan=plan, out=o2),
        "fc2_cublas": lambda: torch.matmul(hm, w2[0].t(), out=c2),
    }
    flops = {"fc1_swiglu": 2.0 * rows * 2 * f * h, "fc1": 2.0 * rows * 2 * f * h,
             "fc1_cublas": 2.0 * rows * 2 * f * h, "fc2": 2.0 * rows * h * f,
             "fc2_cublas": 2.0 * rows * h * f}
    sampler = ClockSampler(os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0])
    sampler.start()
    for _ in range(a.warmup):
        for fn in arms.values():
            fn()
    t_end = time.time() + a.settle_s  # run into the power-capped clock first
    while time.time() < t_end:
        for fn in arms.values():
            fn()
        torch.cuda.synchronize()
    times = {n: [] for n in arms}
    launches0 = _lib.launch_count
    per = max(1, a.steps // 4)
    for _ in range(4):
        for n, fn in arms.items():
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(per + 1)]
            torch.cuda.synchronize()
            w0 = time.time()
            evs[0].record()
            for i in range(per):
                fn()
                evs[i + 1].record()
            torch.cuda.synchronize()
            sampler.mark(w0, time.time(), n)
            times[n] += [evs[i].elapsed_time(evs[i + 1]) for i in range(per)]
    launches = _lib.launch_count - launches0
    clocks = sampler.stop() or {}
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    res = {}
    for n in arms:
        ms = statistics.median(times[n])
        mhz = clocks.get("windows", {}).get(n, {}).get("sm_mhz")
        tf = flops[n] / (ms / 1e3) / 1e12
        res[n] = {"ms": round(ms, 4), "tflops": round(tf, 1), "sm_mhz": mhz,
                  "flop_per_sm_cycle": round(tf * 1e12 / (mhz * 1e6) / sms) if mhz else None}
    same = {"fc1": bool(torch.equal(o1, c1)), "fc2": bool(torch.equal(o2, c2))}
    peaks, peak_kind = load_peaks()
    peak = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    line = {"metric": "dense expert GEMM TFLOP/s (fc1 with SwiGLU)", "value": res["fc1_swiglu"]["tflops"],
            "unit": "TFLOP/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": res["fc1_swiglu"]["ms"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (N(0,1))",
            "config": {"workload": "dense_gemm", "rows": rows, "hidden": h, "ffn": f,
                       "l2": "no flush: operands larger than L2"},
            "arms": res, "vs_cublas": {"fc1": round(res["fc1_cublas"]["ms"] / res["fc1"]["ms"], 4),
                                       "fc2": round(res["fc2_cublas"]["ms"] / res["fc2"]["ms"], 4)},
            "bit_equal_to_cublas": same,
            "roofline": {"bound": "tensor", "kernel": "grouped_gemm_pair_kernel (fc1, SwiGLU)",
                         "achieved": res["fc1_swiglu"]["tflops"], "peak": peak, "unit": "TFLOP/s",
                         "frac": round(res["fc1_swiglu"]["tflops"] / peak, 4), "traffic": None},
            "peak_kind": f"sustained bf16, of {peak_kind}",
            "cpu_baseline": None, "e2e": None, "gpu_launches": launches, "clocks": clocks}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU arm
def read_traffic():
    p = ROOT / "profiles" / "grouped_gemm_fc1_layer.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_fc1_stage:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def layer_inputs(t, h, e, f, routing, dev, rank=0, num_w=None):
    """The benchmark's seeded synthetic layer inputs on `dev` for rank `rank`:
    x [t,h] bf16 ~N(0,1), router logits [t,e] fp32 ~N(0,1) (device generator,
    seed 1000+rank), the Zipf expert bias and num_w experts' weights ~N(0,0.02)
    (seed 77+rank). The full-size parity test builds the same inputs."""
    import torch
    import moe_b200
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    x = torch.randn(t, h, device=dev, generator=g).to(torch.bfloat16)
    logits = torch.randn(t, e, device=dev, generator=g)
    bias = zipf_bias(e, routing).to(dev)
    w = moe_b200.MoEWeights.random(e if num_w is None else num_w, h, f, dev, seed=77 + rank)
    return x, logits, bias, w


def sample_tokens(counts, map_te, n_random=12, seed=0):
    """Tokens whose outputs the check recomputes: the first and last token, a
    token of the busiest expert, a token of the least-used expert that has
    rows, and n_random seeded others."""
    import torch
    t = map_te.shape[0]
    c = counts.to(torch.int64)
    busiest = int(torch.argmax(c))
    pos = torch.where(c > 0, c, torch.full_like(c, 1 << 40))
    rarest = int(torch.argmin(pos))
    picks = [0, t - 1]
    for e_ in (busiest, rarest):
        ts = torch.nonzero(map_te[:, e_] >= 0).flatten()
        picks.append(int(ts[len(ts) // 2]))
    g = torch.Generator().manual_seed(seed)
    picks += torch.randint(0, t, (n_random,), generator=g).tolist()
    return sorted(set(picks))


def check_layer(out, mid, x, logits, bias, w1, w2, k, placement=None):
    """Checks one layer forward against a plain torch reference computed on the
    device (outside every timed region): the routing map (top-k of logits +
    bias), the row_id_map (per-expert cumsum + exclusive offsets) and every
    permuted row exactly; the gates within rtol 1e-5; and the outputs of
    sampled tokens, recomputed in fp32 from their own rows with the chain's
    bf16 roundings, within rtol 2e-2 / atol 1e-2. Returns a summary dict."""
    import torch
    import torch.nn.functional as F
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        r, rim, xp = mid["routing"], mid["rim"], mid["xp"]
        lb = logits + bias[None, :]
        if placement is not None:
            lb = lb[:, placement.long()]
        idx = torch.topk(lb, k, dim=1).indices
        ref_map = torch.zeros_like(r.routing_map)
        ref_map.scatter_(1, idx, True)
        maps_ok = bool(torch.equal(ref_map, r.routing_map))
        p = torch.softmax(lb, dim=1).gather(1, idx)
        p = p / p.sum(dim=1, keepdim=True)
        ref_probs = torch.zeros_like(r.probs).scatter_(1, idx, p)
        probs_ok = bool(torch.allclose(r.probs, ref_probs, rtol=1e-5, atol=1e-7))
        m = ref_map.to(torch.int64)
        cnt = m.sum(dim=0)
        ref_te = torch.where(m > 0, torch.cumsum(m, dim=0) - 1 + (torch.cumsum(cnt, 0) - cnt)[None, :],
                             torch.full_like(m, -1))
        rim_ok = bool(torch.equal(ref_te, rim.map_te))
        ti, ei = torch.nonzero(ref_te >= 0, as_tuple=True)
        dst = ref_te[ti, ei]
        perm_ok = True
        for c0 in range(0, dst.numel(), 16384):  # chunks keep the gathers small
            sl = slice(c0, c0 + 16384)
            perm_ok &= bool(torch.equal(xp[dst[sl]], x[ti[sl]]))
        tokens = sample_tokens(cnt, ref_te)
        fdim = w2.shape[2]
        hk, yk = mid["h"], mid["y"]  # the kernel's fc1 (SwiGLU) and fc2 rows
        worst = {"fc1": 0.0, "fc2": 0.0, "layer": 0.0}
        stage_ok = {"fc1": True, "fc2": True, "combine_exact": True, "layer": True}

        def within(name, got, ref, scale):
            d = (got.float() - ref).abs()
            worst[name] = max(worst[name], float(d.max()))
            return bool(torch.all(d <= 1e-2 + 2e-2 * scale))

        for tok in tokens:
            acc_k = torch.zeros(x.shape[1], dtype=torch.float32, device=x.device)
            acc_r = torch.zeros_like(acc_k)
            mag = torch.zeros_like(acc_k)
            for e_ in sorted(int(v) for v in torch.nonzero(ref_map[tok]).flatten()):
                row = int(ref_te[tok, e_])
                y1 = (x[tok].float() @ w1[e_].float().t()).to(torch.bfloat16).float()
                hm = F.silu(y1[:fdim]) * y1[fdim:]
                stage_ok["fc1"] &= within("fc1", hk[row], hm, hm.abs())
                y_ref = hk[row].float() @ w2[e_].float().t()  # fc2 on the kernel's own fc1 row
                stage_ok["fc2"] &= within("fc2", yk[row], y_ref, y_ref.abs())
                p = r.probs[tok, e_]
                acc_k = acc_k + p * yk[row].float()  # the combine's order and roundings
                yr = (hm.to(torch.bfloat16).float() @ w2[e_].float().t()).to(torch.bfloat16).float()
                acc_r = acc_r + p * yr
                mag = mag + (p * yr).abs()
            stage_ok["combine_exact"] &= bool(torch.equal(out[tok], acc_k.to(torch.bfloat16)))
            # end to end against the all-fp32 chain: each fc2 row may differ by its own
            # bf16 rounding, so the bound scales with the summed magnitude of the terms
            stage_ok["layer"] &= within("layer", out[tok], acc_r.to(torch.bfloat16).float(), mag)
        out_ok = all(stage_ok.values())
        ok = maps_ok and probs_ok and rim_ok and perm_ok and out_ok
        return {"ok": ok, "routing_map": maps_ok, "gates_rtol_1e-5": probs_ok,
                "row_id_map": rim_ok, "permuted_rows": perm_ok, "rows": int(dst.numel()),
                "tokens": len(tokens), "outputs_ok": out_ok,
                "fc1_rows_ok": stage_ok["fc1"], "fc2_rows_ok": stage_ok["fc2"],
                "combine_bit_exact": stage_ok["combine_exact"], "layer_ok": stage_ok["layer"],
                "max_abs_err": {k: round(v, 6) for k, v in worst.items()},
                "tolerance": "rtol 2e-2, atol 1e-2; fc1/fc2 rows relative to the element, "
                             "the layer output relative to the sum of |gate x row| of its terms",
                "reference": "torch on the device: top-k/softmax/cumsum/gather for the maps and "
                             "rows; per sampled token, fp32 fc1+SwiGLU and fc2 from its own rows "
                             "(fc2 also fed the kernel's fc1 row), the combine of the kernel's "
                             "fc2 rows in ascending expert order, and the all-fp32 chain"}
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32


def split_blocks(steps, nblk):
    base, rem = divmod(steps, nblk)
    return [base + (1 if i < rem else 0) for i in range(nblk)]


def main():
    a = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if a.workload == "router_gemm":
        if rank == 0:
            run_router_gemm(a)
        return
    if a.workload == "backward":
        if rank == 0 and a.impl != "reference":
            run_backward(a)
        return
    if a.workload == "wgrad":
        if rank == 0 and a.impl != "reference":
            run_wgrad(a)
        return
    if a.workload == "rowcopy":
        if rank == 0 and a.impl != "reference":
            run_rowcopy(a)
        return
    if a.workload == "dense_gemm":
        if rank == 0 and a.impl != "reference":
            run_dense_gemm(a)
        return
    if a.impl == "reference":
        run_reference_arm(a, world, rank)
        return

    import torch
    import torch.distributed as dist
    import moe_b200
    from moe_b200 import _lib

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    moe_b200.load_library()

    t, h, e, f, k = a.tokens, a.hidden, a.experts, a.ffn, a.topk
    e_loc = e // world
    x, logits, bias, w = layer_inputs(t, h, e, f, a.routing, dev, rank, num_w=e_loc)
    placement = None
    if world == 1:
        layer = moe_b200.MoELayer(w, topk=k, expert_bias=bias)
        stage_names = ["start", "routing", "permute", "fc1", "fc2", "combine"]
    else:
        from moe_b200.ep import MoELayerEP, balanced_placement
        if a.placement == "balanced":
            # Calibration (untimed): expert loads of this job's routing, summed over ranks.
            r0 = moe_b200.router_topk(logits, k, "softmax", True, bias, outputs="maps")
            load = r0.routing_map.sum(0, dtype=torch.int64)
            dist.all_reduce(load)
            placement = torch.tensor(balanced_placement(load.cpu().tolist(), world),
                                     dtype=torch.int32, device=dev)
        layer = MoELayerEP(w, e, topk=k, expert_bias=bias,
                           transport=resolve_transport(a.transport, world), tokens=t,
                           placement=placement, overlap_chunks=overlap_chunks(a, world))
        stage_names = ["start", "local_dispatch", "a2a_dispatch", "fc1", "fc2", "a2a_combine",
                       "combine"]

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def agree_max(v):
        if world == 1:
            return v
        tv = torch.tensor([float(v)], device=dev)
        dist.all_reduce(tv, op=dist.ReduceOp.MAX)
        return float(tv.item())

    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    smi_index = vis.split(",")[local_rank] if vis else str(local_rank)
    sampler = ClockSampler(smi_index)
    sampler.start()
    meter = EnergyMeter(smi_index)
    energy_mj = {"device": 0.0, "e2e": 0.0}
    for _ in range(a.warmup):
        layer(x, logits)
    torch.cuda.synchronize()
    assert device_error(layer) == 0, "grouped GEMM reported a device error"

    # Host-buffer copies of the inputs for the end-to-end windows.
    pipe = None
    if not a.no_e2e:
        x_h = x.cpu().pin_memory()
        lg_h = logits.cpu().pin_memory()
        outs_h = [torch.empty((t, h), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        pipe = moe_b200.HostPipeline(layer, t, h, e, dev, depth=2)
        for i in range(3):
            pipe.submit(x_h, lg_h, outs_h[i % 2])
        pipe.synchronize()

    # Settle (untimed): keep stepping until the GPU has run the layer for
    # --settle-s seconds, so the timed windows see the clock the power cap
    # holds under sustained load rather than the first seconds' boost.
    settle_steps = 0
    if a.settle_s > 0:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        layer(x, logits)
        e1.record()
        torch.cuda.synchronize()
        per = max(e0.elapsed_time(e1), 0.1)
        settle_steps = int(agree_max(min(2000, max(0, int(a.settle_s * 1e3 / per)))))
        for _ in range(settle_steps):
            layer(x, logits)
        torch.cuda.synchronize()

    # ---- timed windows. K device-only steps (inputs resident in HBM) and K
    # end-to-end steps (public API with host buffers) run in interleaved
    # blocks so both see the same clock; each block is bracketed by a barrier
    # and a synchronize on both sides.
    events = [{n: torch.cuda.Event(enable_timing=True) for n in stage_names}
              for _ in range(a.steps)]
    nblk = 2 if (pipe is not None and a.steps >= 8) else 1
    dev_ms = e2e_ms = 0.0
    launches = 0
    step_i = 0
    for nb in split_blocks(a.steps, nblk):
        barrier()
        torch.cuda.synchronize()
        l0 = _lib.launch_count
        j0 = meter.read()
        w0 = time.time()
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record()
        for _ in range(nb):
            layer.events = events[step_i]
            step_i += 1
            layer(x, logits)
        t_end.record()
        torch.cuda.synchronize()
        j1 = meter.read()
        sampler.mark(w0, time.time(), "device")
        if j0 is not None and j1 is not None:
            energy_mj["device"] += j1 - j0
        barrier()
        launches += _lib.launch_count - l0
        layer.events = None
        dev_ms += t_start.elapsed_time(t_end)
        if pipe is not None:
            barrier()
            torch.cuda.synchronize()
            q0 = torch.cuda.Event(enable_timing=True)
            q1 = torch.cuda.Event(enable_timing=True)
            j0 = meter.read()
            w0 = time.time()
            q0.record(pipe.up)
            pipe.run([(x_h, lg_h, outs_h[i % 2]) for i in range(nb)])
            q1.record(pipe.down)
            torch.cuda.synchronize()
            j1 = meter.read()
            sampler.mark(w0, time.time(), "e2e")
            if j0 is not None and j1 is not None:
                energy_mj["e2e"] += j1 - j0
            barrier()
            e2e_ms += q0.elapsed_time(q1)
    stage_ms = {}
    for i in range(1, len(stage_names)):
        n0, n1 = stage_names[i - 1], stage_names[i]
        stage_ms[n1] = sum(ev[n0].elapsed_time(ev[n1]) for ev in events) / a.steps
    fc1_ms = stage_ms["fc1"]
    fc1_rows = t * k if world == 1 else int(layer.last_recv_rows)
    fc2_ms = stage_ms["fc2"]

    ms_step = agree_max(dev_ms / a.steps)
    value = world * t / (ms_step / 1e3)
    e2e = None
    if pipe is not None:
        e2e_step = agree_max(e2e_ms / a.steps)
        e2e = {"value": world * t / (e2e_step / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": x.numel() * 2 + logits.numel() * 4,
               "d2h_bytes_per_step": t * h * 2, "ms_per_step": e2e_step,
               "api": "moe_b200.HostPipeline.run (copies overlapped with compute)"}
    clocks = sampler.stop()

    # ---- correctness of the measured configuration (outside the timed windows)
    check = None
    if world == 1:
        out, mid = layer.forward(x, logits, return_intermediates=True)
        torch.cuda.synchronize()
        check = check_layer(out, mid, x, logits, bias, w.w1, w.w2, k)
        check["device_error"] = layer.plan.device_error() + moe_b200.permute_device_error(dev)
        check["ok"] = check["ok"] and check["device_error"] == 0
        del out, mid
    elif not a.no_check:
        check = check_ep(layer, x, logits, bias, w, k, placement, world, rank, dev)

    peaks, peak_kind = load_peaks()
    fc1_flops = 2.0 * fc1_rows * (2 * f) * h
    fc2_flops = 2.0 * fc1_rows * h * f
    achieved = fc1_flops / (fc1_ms / 1e3) / 1e12
    peak = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    traffic = read_traffic() if world == 1 else None  # captured at the single-GPU workload
    rows = fc1_rows
    perm_bytes = t * h * 2 + rows * h * 2 + t * e * 8
    comb_bytes = rows * h * 2 + t * h * 2 + t * e * 8 + t * e * 4
    stages = {n: round(ms, 4) for n, ms in stage_ms.items()}
    extra = {
        "stages_ms": stages,
        "fc1_tflops": round(achieved, 1),
        "fc2_tflops": round(fc2_flops / (fc2_ms / 1e3) / 1e12, 1),
        "gemm_frac_of_peak": round((fc1_flops + fc2_flops) / ((fc1_ms + fc2_ms) / 1e3) / 1e12 / peak, 4),
        "peak_kind": f"bf16 sustained, of {peak_kind}",
        "hbm_peak_gbs": hbm,
        "settle_steps": settle_steps,
        "timed_blocks": nblk,
    }
    if world == 1:
        extra["permute_gbs"] = round(perm_bytes / (stage_ms["permute"] / 1e3) / 1e9, 1)
        extra["combine_gbs"] = round(comb_bytes / (stage_ms["combine"] / 1e3) / 1e9, 1)
    if clocks and clocks.get("windows"):
        # Clock-normalised step cost: ms per step x median SM MHz of its window
        # (millions of SM cycles per step), comparable across power-capped runs.
        wn = clocks["windows"]
        norm = {}
        if wn.get("device", {}).get("sm_mhz"):
            norm["value_mcycles_per_step"] = round(ms_step * wn["device"]["sm_mhz"] / 1e3, 3)
        if e2e and wn.get("e2e", {}).get("sm_mhz"):
            norm["e2e_mcycles_per_step"] = round(e2e["ms_per_step"] * wn["e2e"]["sm_mhz"] / 1e3, 3)
        extra["clock_normalised"] = norm
    if meter.h is not None and energy_mj["device"] > 0:
        # This GPU's energy (rank 0's at N > 1): the timed device-only and e2e
        # windows, from the board's counter, which includes the idle host gaps.
        extra["energy"] = {"j_per_step": round(energy_mj["device"] / 1e3 / a.steps, 4),
                           "e2e_j_per_step": round(energy_mj["e2e"] / 1e3 / a.steps, 4)
                           if energy_mj["e2e"] > 0 else None,
                           "tokens_per_joule": round(t * a.steps / (energy_mj["device"] / 1e3), 1),
                           "source": "NVML total energy counter, timed windows"}

    cpu = None
    if world == 1 and rank == 0 and not a.no_cpu_baseline:
        cpu = cpu_baseline_sample(a)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms_step,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (seeded N(0,1) activations/logits, "
                "N(0,0.02) weights, Zipf expert bias)",
                "config": config_dict(a, world),
                "roofline": {"bound": "tensor", "kernel": "grouped_gemm fc1 stage (tcgen05 pair kernel + remainder kernel, fused SwiGLU)",
                             "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                             "frac": round(achieved / peak, 4), "traffic": traffic},
                "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches, "clocks": clocks,
                "checked": None if check is None else bool(check["ok"]), "check": check}
        line.update(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        if hasattr(layer, "close"):
            layer.close()
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
