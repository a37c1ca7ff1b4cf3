"""Benchmark: the KSDraft INT8 training step (benchmark config 4 by default).

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]
                    [--workload config4|config2]

config4 (the metric's "train tokens/sec"): the full 24-layer KSDraft model at
d_model=1536 (5888 KS3 charts, 512 Rosa streams, vocab 150144 with the head
tied to the embedding), batch 16 x 2048 tokens of Zipf(1.1) ids with repeated
spans plus bf16 N(0,1) teacher states (teacher_dim 384), weights N(0,0.02).
One step = forward, CE + transfer-space loss, backward, the data-parallel
gradient mean (NCCL, N > 1), clip_grad_norm_(1.0) and AdamW.  The global batch
is fixed at 16 sequences, 16/N per GPU ("scaling": "strong");
--per-gpu-batch K runs K sequences on every rank instead ("scaling": "weak").

config2: one KS3 decoder layer INT8 fwd+bwd (+ DP all-reduce + AdamW) at 4096
tokens per GPU (weak scaling), kept as a second workload.

config5: draft serving -- 64 contexts of 8192 Zipf(1.1) tokens prefilled (not
timed), then each step appends a block of 8 positions to every context through
the 24 layers and returns the top-8 candidates of the W8A8 head (contexts split
over the GPUs, vocabulary sharded); value = 512 tokens per step / step time.

`value`  tokens/s of the whole job with inputs resident in HBM, device-timed
         with CUDA events per step (L2 flushed between steps), max over ranks.
`e2e`    the same step through the public API with pinned host inputs copied
         in and the loss read back inside the timed region.
`roofline` the W8A8 GEMM (the dominant kernel): algorithmic ops of every GEMM
         launch / their summed CUDA-event durations inside the timed steps,
         against 2x the measured dense bf16 peak (int8 = 2x the bf16 rate).
`cpu_baseline` / `--impl reference`: the reference's own torch CPU tier
         (installed unmodified in baseline/_ref) on the same step, timed on the
         host cores for the steps that fit a time budget (the count is printed).
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
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

D_MODEL, CHARTS, TOKENS, BATCH, SEQ = 1536, 5888, 4096, 8, 512
C4_BATCH, C4_SEQ, C4_TEACHER = 16, 2048, 384
C5_CONTEXTS, C5_CONTEXT_LEN, C5_BLOCK, C5_TOPK = 64, 8192, 8, 8
REF_C4_TOKENS = int(os.environ.get("KSD8_REF_TOKENS", "128"))
METRIC = "W8A8 GS128 GEMM TOPS; KSDraft INT8 train tokens/sec at 1/2/4/8 B200"
DITHER = 0.5


def config4(n: int, per_gpu: int | None = None) -> dict:
    per_gpu = C4_BATCH // n if per_gpu is None else per_gpu
    return {"workload": "benchmark config 4: full KSDraft INT8 training step, 24 layers, "
                        "d_model=1536, vocab=150144, 512 Rosa streams, 5888 KS3 charts, "
                        + (f"batch {per_gpu} x 2048 tokens per GPU" if per_gpu * n != C4_BATCH
                           else f"global batch {C4_BATCH} x 2048 tokens ({per_gpu} per GPU)")
                        + ", DP over the GPUs",
            "model": "KSDraft 24 x (Rosa + DSpine + KS3) d_model=1536 vocab=150144",
            "global_batch": per_gpu * n, "seq_len": C4_SEQ,
            "tokens_per_step": per_gpu * n * C4_SEQ,
            "sequences_per_gpu": per_gpu, "parallelism": f"dp{n}",
            "teacher_dim": C4_TEACHER, "activations": "bf16 residual stream",
            "l2": "flushed between timed steps (256 MiB write); step working set > L2"}


def config(n: int) -> dict:
    return {"workload": "benchmark config 2: one KS3 decoder layer INT8 fwd+bwd (+DP all-reduce "
                        "+ AdamW), d_model=1536, charts=5888, 4096 tokens/GPU",
            "model": "KSDraft KS3 decoder layer (d_model=1536, charts=5888)",
            "global_batch": BATCH * n, "seq_len": SEQ, "tokens_per_gpu": TOKENS,
            "parallelism": f"dp{n}", "ptqr_dither": DITHER,
            "l2": "flushed between timed steps (256 MiB write); step working set > L2"}


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"bf16": float(d["bf16_tflops"]), "hbm": float(d["hbm_gbs"]), "src": "measured",
                "bf16_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"]))}
    return {"bf16": 1590.0, "hbm": 6650.0, "src": "fallback", "bf16_sustained": 1400.0}


def gemm_traffic() -> float | None:
    p = ROOT / "profiles" / "w8a8_gemm_traffic.json"
    if p.exists():
        return float(json.loads(p.read_text())["bytes_per_launch"])
    return None


# ---------------------------------------------------------------- CPU side
#
# The reference (curvedinf/ksdraft) is a pure-torch package; its own fp32/bf16
# CPU tier is what the CPU figures time.  It is installed (unmodified) into
# baseline/_ref, which travels with the repository; only when that install is
# missing does the oracle port (oracle/, C + numpy) stand in, labelled "port".

REF_DIR = ROOT / "baseline" / "_ref"
REF_BUDGET_S = float(os.environ.get("KSD8_REF_BUDGET_S", "150"))


def import_reference():
    """The reference package from baseline/_ref, or None when it is not installed."""
    if not (REF_DIR / "ksdraft" / "__init__.py").exists():
        return None
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import ksdraft
    if not str(Path(ksdraft.__file__).resolve()).startswith(str(REF_DIR.resolve())):
        raise RuntimeError(f"ksdraft imported from {ksdraft.__file__}, not {REF_DIR}")
    return ksdraft


def _timed_steps(step, steps: int, warmup: int, budget_s: float):
    """Run `warmup` untimed and then up to `steps` timed calls of step(), stopping
    early once the timed calls would exceed budget_s.  Returns the per-step
    seconds actually measured (never extrapolated)."""
    for _ in range(warmup):
        step()
    times = []
    t_start = time.perf_counter()
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        elapsed = time.perf_counter() - t_start
        if elapsed + statistics.mean(times) > budget_s:
            break
    return times


def reference_layer_step(tokens: int = TOKENS):
    """The reference's own config-2 step on the host cores: KS3Int8Cell(trainable)
    forward + backward (ksdraft/kernels/ks3_int8.py:317-429) on `tokens` bf16
    tokens, then the trainer's clip_grad_norm_(1.0) and AdamW step
    (ksdraft/train/__init__.py:163-166) over the cell's fp32 masters."""
    import torch
    ref = import_reference()
    from ksdraft.kernels.ks3_int8 import KS3Int8Cell
    from ksdraft.model.ks3 import KS3
    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator().manual_seed(1234)
    cell = KS3(D_MODEL, CHARTS)
    with torch.no_grad():
        cell.down.weight.copy_(torch.randn(CHARTS, D_MODEL, generator=gen) * 0.02)
        cell.up.weight.copy_(torch.randn(D_MODEL, CHARTS, generator=gen) * 0.02)
    q = KS3Int8Cell(cell, 128, "int8", trainable=True)
    params = [p for p in q.parameters() if p.requires_grad]
    opt = torch.optim.AdamW(params, lr=3e-4, weight_decay=0.01)
    x = torch.randn(tokens, D_MODEL, generator=gen).to(torch.bfloat16)
    g = (torch.randn(tokens, D_MODEL, generator=gen) * 1e-2).to(torch.bfloat16)

    def step():
        opt.zero_grad(set_to_none=True)
        xr = x.detach().requires_grad_(True)
        q(xr).backward(g)
        torch.nn.utils.clip_grad_norm_(params, 1.0)
        opt.step()
    return step, ref.__file__


def reference_draft_step(tokens: int = REF_C4_TOKENS):
    """The reference's own config-4 step on the host cores, on one sequence of
    `tokens` tokens: KSDraftModel (24 layers, d_model 1536, vocab 150144, 512
    streams, 5888 charts, teacher_dim 384) converted by to_int8 with trainable
    KS3 cells, in training mode (the CPU hard Rosa path, rosa.py:150-165), then
    distillation_losses, backward, clip_grad_norm_(1.0) and AdamW
    (ksdraft/train/__init__.py:145-166)."""
    import torch
    ref = import_reference()
    from ksdraft.config import KSDraftConfig
    from ksdraft.kernels.ks3_int8 import KS3Int8Cell
    from ksdraft.model import KSDraftModel
    from ksdraft.model.int8_convert import to_int8
    from ksdraft.train import distillation_losses
    torch.set_num_threads(os.cpu_count() or 1)
    torch.manual_seed(0)
    cfg = KSDraftConfig(d_model=D_MODEL, layers=24, rosa_streams=512, ks3_charts=CHARTS)
    model = KSDraftModel(cfg, teacher_dim=C4_TEACHER)
    q = to_int8(model)
    for blk, src in zip(q.blocks, model.blocks):
        blk.ffn = KS3Int8Cell(src.ffn, 128, "int8", trainable=True)
    del model
    q.train()
    opt = torch.optim.AdamW(q.parameters(), lr=3e-4, weight_decay=0.01)
    ids = torch.from_numpy(rosa_ids(1, tokens + 1, seed=7))
    states = torch.randn(1, tokens, C4_TEACHER).to(torch.bfloat16)

    def step():
        logits, feats = q(ids[:, :-1], teacher_states=states)
        loss, _ = distillation_losses(logits, ids, feats, q.embedding.weight, None, None,
                                      0.5, 0.0)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(q.parameters(), 1.0)
        opt.step()
    return step, ref.__file__


def port_layer_step(tokens: int = 128):
    """Stand-in when the reference is not installed: the oracle port of the same
    layer step (oracle/, C + numpy with OpenMP) on `tokens` tokens."""
    from oracle import oracle
    args = cpu_layer_inputs(tokens)
    return lambda: oracle.ks3_layer(*args)


def cpu_layer_inputs(tokens: int, seed: int = 0):
    rng = np.random.default_rng(seed)
    import torch
    x = torch.from_numpy(rng.standard_normal((tokens, D_MODEL)).astype(np.float32)) \
        .to(torch.bfloat16).float().numpy()
    g = torch.from_numpy((rng.standard_normal((tokens, D_MODEL)) * 1e-2).astype(np.float32)) \
        .to(torch.bfloat16).float().numpy()
    down = (rng.standard_normal((CHARTS, D_MODEL)) * 0.02).astype(np.float32)
    up = (rng.standard_normal((D_MODEL, CHARTS)) * 0.02).astype(np.float32)
    coeffs = (rng.standard_normal((CHARTS, 6)) * 0.05).astype(np.float32)
    rs = np.full(CHARTS, 0.75, np.float32)
    rh = np.zeros(CHARTS, np.float32)
    return x, down, up, coeffs, rs, rh, g


def cpu_measure(steps: int, warmup: int, budget_s: float, workload: str = "config2") -> dict:
    """The reference's CPU tier on the workload's step, timed on all host cores for
    as many of `steps` as fit in budget_s.  config2: the full 4096-token layer
    step; config4: the full 24-layer model step on one sequence of
    REF_C4_TOKENS tokens (a full 32768-token CPU step would take hours)."""
    import torch
    if workload == "config4":
        if import_reference() is None:
            raise RuntimeError("the config-4 reference arm needs the reference installed in "
                               "baseline/_ref")
        step, where = reference_draft_step(REF_C4_TOKENS)
        times = _timed_steps(step, steps, warmup, budget_s)
        sec = statistics.median(times)
        return {"value": REF_C4_TOKENS / sec, "unit": "tokens/s",
                "cores": torch.get_num_threads(), "kind": "reference",
                "sample": f"the reference's own 24-layer KSDraftModel int8 tier (to_int8, "
                          f"trainable KS3, CPU hard Rosa path, float head) training step "
                          f"(fwd, CE+transfer loss, bwd, clip, AdamW) on 1 x {REF_C4_TOKENS} "
                          f"tokens, torch CPU tier from baseline/_ref; median of "
                          f"{len(times)} timed steps",
                "sec_per_step": sec, "steps_timed": len(times), "tokens_per_step": REF_C4_TOKENS}
    if import_reference() is not None:
        step, where = reference_layer_step(TOKENS)
        tokens, kind = TOKENS, "reference"
        what = (f"the reference's own KS3Int8Cell(trainable) fwd+bwd + clip_grad_norm_ + "
                f"AdamW at the full config-2 step ({TOKENS} tokens), torch CPU tier "
                f"imported from baseline/_ref")
    else:
        step, tokens, kind = port_layer_step(), 128, "port"
        what = ("oracle port of the config-2 layer step on 128 tokens (the reference is not "
                "installed in baseline/_ref)")
    times = _timed_steps(step, steps, warmup, budget_s)
    sec = statistics.median(times)
    return {"value": tokens / sec, "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": kind, "sample": f"{what}; median of {len(times)} timed steps",
            "sec_per_step": sec, "steps_timed": len(times), "tokens_per_step": tokens}


def cpu_baseline(workload: str = "config2") -> dict:
    m = cpu_measure(steps=2, warmup=1, budget_s=60, workload=workload)
    return {k: m[k] for k in ("value", "unit", "cores", "kind", "sample")}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload == "config5":
        print(json.dumps({"impl": "reference", "unavailable":
                          "the reference has no incremental decode or proposal API (only "
                          "whole-sequence forwards, ksdraft/model/draft.py:58-82)"}), flush=True)
        return
    m = cpu_measure(steps=max(1, args.steps), warmup=max(1, min(args.warmup, 1)),
                    budget_s=REF_BUDGET_S, workload=args.workload)
    c4 = args.workload == "config4"
    line = {"impl": "reference", "metric": METRIC, "value": m["value"], "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": m["steps_timed"], "steps_requested": args.steps,
            "warmup": 1, "ms_per_step": m["sec_per_step"] * 1e3,
            "higher_is_better": True,
            "scaling": "strong" if (c4 and args.per_gpu_batch is None) else "weak",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": (config4(args.gpus, args.per_gpu_batch or C4_BATCH // args.gpus)
                       if c4 else config(1)),
            "cpu_baseline": {k: m[k] for k in ("kind", "cores", "sample", "value", "unit")},
            "e2e": {"value": m["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU side

class ClockSampler:
    """SM clock and clock-event reasons during the timed region, read every 5 ms
    through NVML on a background thread (nvidia-smi -lms as the fallback).
    Only reads: no clock, power or mode of the GPU is changed."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
               ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []       # (sm_mhz, reason bits)
        self.max_mhz = None
        self.stop = None
        self.thread = None
        self.proc = None
        self.path = None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.index)
        try:
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:  # noqa: BLE001 - fall back to the visible index
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def __enter__(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self.stop = threading.Event()

            def poll():
                while not self.stop.is_set():
                    try:
                        self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                             int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))))
                    except Exception:  # noqa: BLE001
                        break
                    self.stop.wait(0.005)
            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return self
        except Exception:  # noqa: BLE001 - no NVML: nvidia-smi
            pass
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.thread is not None:
            if not self.samples:
                return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
            sm = [s for s, _ in self.samples]
            loaded = [s for s in sm if s > 500] or sm
            reasons = sorted({name for _, bits in self.samples for name, bit in self.REASONS
                              if bits & bit})
            return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": self.max_mhz,
                    "reasons": reasons, "samples": len(self.samples), "source": "nvml"}
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except (OSError, TypeError):
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        loaded = [s for s in sm if s > 500] or sm
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            for name, val in zip(names, r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit()
                else None, "reasons": sorted(reasons), "samples": len(rows),
                "source": "nvidia-smi"}


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from ksdraft_b200 import _lib
    from ksdraft_b200.kernels.gemm import GemmTimer
    from ksdraft_b200.kernels.ks3_int8 import KS3Int8Cell, init_ks3_weights
    from ksdraft_b200.train.dp import KS3DataParallelStep, init_distributed

    rank, world, local = init_distributed(timeout_s=300)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    # same weights on every rank
    cell = init_ks3_weights(D_MODEL, CHARTS, generator=torch.Generator().manual_seed(1234),
                            device=dev)
    q = KS3Int8Cell(cell, nonlinear="int8", trainable=True)
    q._dither = DITHER
    q._dither_seed = 20260101
    # gradient clipping as the reference trainer (max norm 1.0); KSD8_GRAD_CLIP=0 disables it
    clip = float(os.environ.get("KSD8_GRAD_CLIP", "1.0"))
    step = KS3DataParallelStep(q, grad_clip=clip if clip > 0 else None)

    gen = torch.Generator().manual_seed(1000 + rank)  # each rank its own tokens
    x_host = torch.randn(TOKENS, D_MODEL, generator=gen).to(torch.bfloat16).pin_memory()
    g_host = (torch.randn(TOKENS, D_MODEL, generator=gen) * 1e-2).to(torch.bfloat16) \
        .pin_memory()
    y_host = torch.empty(TOKENS, D_MODEL, dtype=torch.bfloat16).pin_memory()
    x_dev, g_dev = x_host.to(dev), g_host.to(dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(x_dev, g_dev)
    barrier()

    # ---- device-resident timing (value) + per-GEMM events (roofline)
    times = []
    launches0 = _lib.LAUNCHES
    with ClockSampler(local) as clocks, GemmTimer() as gt:
        for _ in range(args.steps):
            flush.zero_()
            barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            step(x_dev, g_dev)
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
    launches = _lib.LAUNCHES - launches0
    gemm = gt.durations_ms()
    total_ms = torch.tensor([sum(times)], device=dev)
    if world > 1:
        dist.all_reduce(total_ms, op=dist.ReduceOp.MAX)
    total_ms = float(total_ms.item())

    # ---- end to end through the public API with host buffers
    e2e_times = []
    for _ in range(args.steps):
        flush.zero_()
        barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        # host tensors in and out: the step copies x before the forward, the
        # upstream gradient during the forward and y back during the backward
        step(x_host, g_host, y_out=y_host)
        e.record()
        torch.cuda.synchronize()
        e2e_times.append(s.elapsed_time(e))
    e2e_ms = torch.tensor([sum(e2e_times)], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())

    if rank == 0:
        tokens_total = TOKENS * world * args.steps
        value = tokens_total / (total_ms / 1e3)
        peaks = load_peaks()
        gemm_ms = [d for d, _ in gemm]
        ops = gemm[0][1] if gemm else 0
        avg_gemm_ms = statistics.mean(gemm_ms) if gemm_ms else float("nan")
        achieved = ops / (avg_gemm_ms / 1e3) / 1e12 if gemm_ms else None
        peak_int8 = 2.0 * peaks["bf16"]
        traffic = gemm_traffic()
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic", "config": config(world),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_int8,
                         "unit": "TFLOP/s", "frac": achieved / peak_int8 if achieved else None,
                         "traffic": traffic,
                         "kernel": "w8a8_gemm_kernel (tcgen05 kind::i8), 6 launches/step of "
                                   "2*4096*5888*1536 = 74.09 GOP each",
                         "peak_note": f"2 x {peaks['src']} dense bf16 TF/s (int8 rate = 2x bf16)"
                         },
            "gemm": {"launches": len(gemm_ms), "avg_ms": avg_gemm_ms,
                     "tops": achieved, "ops_per_launch": ops,
                     "share_of_step": sum(gemm_ms) / sum(times) if times else None},
            "e2e": {"value": TOKENS * world * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": x_host.numel() * 2 + g_host.numel() * 2,
                    "d2h_bytes_per_step": y_host.numel() * 2},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_side:
            del flush, x_dev, g_dev
            line["side"] = side_measurements(dev)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _roofline_from_gemms(gemm, peaks) -> tuple[dict, dict]:
    """Aggregate W8A8 GEMM figures: total algorithmic ops / total event time."""
    gemm_ms = [d for d, _ in gemm]
    ops = [o for _, o in gemm]
    total_ms = sum(gemm_ms)
    achieved = sum(ops) / (total_ms / 1e3) / 1e12 if total_ms > 0 else None
    peak_int8 = 2.0 * peaks["bf16"]
    traffic = gemm_traffic()
    roof = {"bound": "tensor", "achieved": achieved, "peak": peak_int8, "unit": "TFLOP/s",
            "frac": achieved / peak_int8 if achieved else None, "traffic": traffic,
            "kernel": "w8a8_gemm_kernel (tcgen05 kind::i8): sum of 2*M*N*K over every GEMM "
                      "launch in the timed steps / sum of their CUDA-event durations",
            "peak_note": f"2 x {peaks['src']} dense bf16 TF/s (int8 rate = 2x bf16), the burst "
                         "figure: the step's sampled SM clock stays at its maximum",
            "frac_vs_sustained_peak": (achieved / (2.0 * peaks["bf16_sustained"])
                                       if achieved else None)}
    info = {"launches": len(gemm_ms), "total_ms": total_ms,
            "avg_ms": statistics.mean(gemm_ms) if gemm_ms else None, "tops": achieved}
    return roof, info


def run_config4(args) -> None:
    """benchmark config 4 on N GPUs (one process each): the full training step."""
    import torch
    import torch.distributed as dist

    from ksdraft_b200 import _lib
    from ksdraft_b200.kernels.gemm import GemmTimer
    from ksdraft_b200.train.dp import init_distributed
    from ksdraft_b200.train.draft_step import DRAFT_SM_RESERVE, DraftShape, DraftTrainStep

    rank, world, local = init_distributed(timeout_s=600, nccl_max_ctas=DRAFT_SM_RESERVE)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    strong = args.per_gpu_batch is None
    if strong:
        if C4_BATCH % world:
            raise SystemExit(f"global batch {C4_BATCH} does not split over {world} GPUs")
        B = C4_BATCH // world
    else:
        B = args.per_gpu_batch
    group = dist.group.WORLD if world > 1 else None
    step = DraftTrainStep(DraftShape(), dev, seed=1234, group=group)   # same weights on every rank
    # this rank's sequences: Zipf(1.1) ids with repeated spans (as config 3), teacher states
    ids = rosa_ids(B * world, C4_SEQ + 1, seed=4)[rank * B:(rank + 1) * B]
    tok_host = torch.from_numpy(ids).pin_memory()
    gen = torch.Generator().manual_seed(100 + rank)
    ts_host = torch.randn(B, C4_SEQ, C4_TEACHER, generator=gen).to(torch.bfloat16).pin_memory()
    tok_dev, ts_dev = tok_host.to(dev), ts_host.to(dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(tok_dev, ts_dev)
    barrier()

    # forward + backward (with the gradient collectives) replay as one CUDA
    # graph (no per-kernel host work); the GEMM events are recorded inside it
    use_graph = not args.no_graph
    gt = GemmTimer(external=True)
    if use_graph:
        with gt:
            step.capture(tok_dev, ts_dev, phase_marks=True)
        captured = step.captured_launches

        def run(tok, ts):
            return step.replay(tok, ts)
    else:
        run = step

    times = []
    gemm = []
    launches0 = _lib.LAUNCHES
    with ClockSampler(local) as clocks:
        for _ in range(args.steps):
            flush.zero_()
            barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if not use_graph:
                gt = GemmTimer().__enter__()
            s.record()
            with torch.cuda.nvtx.range("c4_step"):    # launch-list filter for ncu --nvtx
                run(tok_dev, ts_dev)
            e.record()
            torch.cuda.synchronize()
            if not use_graph:
                gt.__exit__()
            times.append(s.elapsed_time(e))
            gemm += gt.durations_ms()
    launches = (_lib.LAUNCHES - launches0) // max(1, args.steps)
    if use_graph:
        launches += captured
    total_ms = torch.tensor([sum(times)], device=dev)
    if world > 1:
        dist.all_reduce(total_ms, op=dist.ReduceOp.MAX)
    total_ms = float(total_ms.item())

    # where the time goes: the phase events of the last timed step (inside the
    # graph) or of one more eager step (outside the timed region)
    if use_graph:
        phases = step.graph_phases()
    else:
        marks = []
        step.phase_marks = marks
        step(tok_dev, ts_dev)
        torch.cuda.synchronize()
        step.phase_marks = None
        phases = {}
        for (name, ev), (_, nxt) in zip(marks, marks[1:]):
            phases[name] = phases.get(name, 0.0) + ev.elapsed_time(nxt)

    # end to end: host ids and teacher states copied in, the loss read back
    loss_host = torch.empty(1, dtype=torch.float32).pin_memory()
    e2e_times = []
    for _ in range(args.steps):
        flush.zero_()
        barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        loss = run(tok_host, ts_host)
        loss_host.copy_(loss.detach().reshape(1), non_blocking=True)
        e.record()
        torch.cuda.synchronize()
        e2e_times.append(s.elapsed_time(e))
    e2e_ms = torch.tensor([sum(e2e_times)], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())
    gn = float(step.last_grad_norm)

    if rank == 0:
        tokens_total = B * world * C4_SEQ * args.steps
        peaks = load_peaks()
        roof, ginfo = _roofline_from_gemms(gemm, peaks)
        ginfo["share_of_step"] = ginfo["total_ms"] / sum(times) if times else None
        line = {
            "metric": METRIC, "value": tokens_total / (total_ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if strong else "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic", "config": config4(world, B),
            "roofline": roof, "gemm": ginfo,
            "e2e": {"value": tokens_total / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": world * (tok_host.numel() * 8 + ts_host.numel() * 2),
                    "d2h_bytes_per_step": world * 4},
            "gpu_launches": launches, "loss": float(loss_host.item()), "grad_norm": gn,
            "phases_ms": {k: round(v, 3) for k, v in phases.items()},
            "cuda_graph": use_graph,
            "clocks": clocks.summary(),
        }
    step.release()
    torch.cuda.synchronize()
    if rank == 0:
        if world == 1 and not args.no_side:
            del step, tok_dev, ts_dev, flush
            torch.cuda.empty_cache()
            line["side"] = side_measurements(dev)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline("config4")
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def config5(n: int) -> dict:
    return {"workload": "benchmark config 5: KSDraft INT8 draft serving, 64 concurrent contexts "
                        "of 8192 Zipf(1.1) tokens with bf16 N(0,1) teacher states, blocks of 8 "
                        "appended positions per context per step through 24 layers at "
                        "d_model=1536, top-8 candidates from the W8A8 GS128 LM head (vocab "
                        "150144) sharded by vocab over the GPUs",
            "model": "KSDraft 24 x (Rosa + DSpine + KS3) d_model=1536 vocab=150144",
            "contexts": C5_CONTEXTS, "context_len": C5_CONTEXT_LEN, "block": C5_BLOCK,
            "topk": C5_TOPK, "tokens_per_step": C5_CONTEXTS * C5_BLOCK,
            "contexts_per_gpu": C5_CONTEXTS // n,
            "parallelism": f"contexts split over {n} GPU(s), head sharded by vocab",
            "activations": "bf16", "l2": "step working set (decode state, weights) > L2"}


def run_config5(args) -> None:
    """benchmark config 5 on N GPUs: prefill the contexts (untimed), then time
    `steps` propose() calls of one 8-position block per context."""
    import torch
    import torch.distributed as dist

    from ksdraft_b200 import _lib
    from ksdraft_b200.kernels.gemm import GemmTimer
    from ksdraft_b200.model.drafter import KSDraftDrafter
    from ksdraft_b200.train.dp import init_distributed
    from ksdraft_b200.train.draft_step import DraftShape, init_draft_params

    rank, world, local = init_distributed(timeout_s=600)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if C5_CONTEXTS % world:
        raise SystemExit(f"{C5_CONTEXTS} contexts do not split over {world} GPUs")
    shape = DraftShape()
    flat, frozen = init_draft_params(shape, dev, seed=1234)   # same weights on every rank
    state = {n: flat.p(n) for n in flat.names}
    state.update(frozen)
    group = dist.group.WORLD if world > 1 else None
    # the delta keys the step kernel compares directly grow from 0 to ~2000
    # between two main-run rebuilds: untimed blocks after the warm-up bring the
    # timed ones to the middle of that cycle, whose step time is the average
    advance = max(0, KSDraftDrafter.steps_per_rebuild(C5_BLOCK) // 2 - args.warmup
                  - args.steps // 2)
    n_steps = args.warmup + advance + 2 * args.steps
    cap = C5_CONTEXT_LEN + n_steps * C5_BLOCK
    drafter = KSDraftDrafter(state, shape, dev, contexts=C5_CONTEXTS, capacity=cap,
                             group=group)
    del flat, frozen, state
    torch.cuda.empty_cache()
    T = cap
    ids = torch.from_numpy(rosa_ids(C5_CONTEXTS, T, seed=5))
    gen = torch.Generator().manual_seed(55)
    # teacher states of every position, generated in context blocks (bf16 N(0, 1))
    states = torch.empty(C5_CONTEXTS, T, C4_TEACHER, dtype=torch.bfloat16)
    for c in range(C5_CONTEXTS):
        states[c] = torch.randn(T, C4_TEACHER, generator=gen).to(torch.bfloat16)
    ids_pin, states_pin = ids.pin_memory(), states.pin_memory()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    t_pre = time.perf_counter()
    drafter.prefill(ids[:, :C5_CONTEXT_LEN], states[:, :C5_CONTEXT_LEN], topk=C5_TOPK)
    barrier()
    prefill_s = time.perf_counter() - t_pre
    pos = C5_CONTEXT_LEN

    def block(p, host=False):
        sl = slice(p, p + C5_BLOCK)
        if host:
            return states_pin[:, sl], ids_pin[:, sl]
        return states_dev[:, sl], ids_dev[:, sl]

    # device-resident inputs of the timed device-side steps
    ids_dev = ids.to(dev)
    states_dev = states.to(dev)
    for _ in range(args.warmup):
        drafter.propose(*block(pos), topk=C5_TOPK)
        pos += C5_BLOCK
    for _ in range(advance):
        drafter.propose(*block(pos), topk=C5_TOPK)
        pos += C5_BLOCK
    # the block's ~750 small launches replay as one CUDA graph (position read on
    # the device; main-run rebuilds, when due, run before the replay)
    use_graph = not args.no_graph
    gt = GemmTimer(external=True)
    captured = 0
    if use_graph:
        with gt:
            drafter.capture(C5_BLOCK, C5_TOPK, phase_marks=True)
        captured = drafter.captured_launches
    barrier()
    times, gemm = [], []
    launches0 = _lib.LAUNCHES
    with ClockSampler(local) as clocks:
        for _ in range(args.steps):
            barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if not use_graph:
                gt = GemmTimer().__enter__()
            s.record()
            with torch.cuda.nvtx.range("c5_step"):
                drafter.propose(*block(pos), topk=C5_TOPK)
            e.record()
            torch.cuda.synchronize()
            if not use_graph:
                gt.__exit__()
            gemm += gt.durations_ms()
            times.append(s.elapsed_time(e))
            pos += C5_BLOCK
    launches = (_lib.LAUNCHES - launches0) // max(1, args.steps) + captured
    total = torch.tensor([sum(times)], device=dev)
    if world > 1:
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
    total_ms = float(total.item())
    # end to end: host ids and teacher states in, the candidate ids back to the host
    out_host = torch.empty(C5_CONTEXTS, C5_BLOCK, C5_TOPK, dtype=torch.int64).pin_memory()
    e2e = []
    for _ in range(args.steps):
        barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        cand, _, _ = drafter.propose(*block(pos, host=True), topk=C5_TOPK)
        out_host.copy_(cand, non_blocking=True)
        e.record()
        torch.cuda.synchronize()
        e2e.append(s.elapsed_time(e))
        pos += C5_BLOCK
    # a main-run rebuild (every layer's keys re-sorted) comes every
    # steps_per_rebuild blocks; its cost is reported beside the step time
    barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    drafter.rebuild()
    e.record()
    torch.cuda.synchronize()
    rebuild_ms = s.elapsed_time(e)
    e2e_t = torch.tensor([sum(e2e)], device=dev)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    tok = C5_CONTEXTS * C5_BLOCK * args.steps
    if rank == 0:
        roof, ginfo = _roofline_from_gemms(gemm, load_peaks())
        line = {
            "metric": METRIC, "value": tok / (total_ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": config5(world), "roofline": roof, "gemm": ginfo,
            "e2e": {"value": tok / (float(e2e_t.item()) / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": C5_CONTEXTS * C5_BLOCK * (8 + C4_TEACHER * 2),
                    "d2h_bytes_per_step": C5_CONTEXTS * C5_BLOCK * C5_TOPK * 8},
            "gpu_launches": launches, "prefill_s": prefill_s, "cuda_graph": use_graph,
            "rebuild": {"ms": rebuild_ms, "every_steps": drafter.steps_per_rebuild(C5_BLOCK),
                        "timed_blocks_after_build": args.warmup + advance,
                        "value_amortized": tok / ((total_ms + rebuild_ms * args.steps
                                                   / drafter.steps_per_rebuild(C5_BLOCK))
                                                  / 1e3)},
            "phases_ms": ({k: round(v, 3) for k, v in drafter.phases().items()}
                          if use_graph else None),
            "clocks": clocks.summary()}
        print(json.dumps(line), flush=True)
    drafter.release()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def rosa_ids(B: int, T: int, seed: int = 0, vocab: int = 150144):
    """Config-3 token ids: Zipf(1.1) over the vocabulary, then repeated spans of
    length 8-64 copied from earlier positions until 10% of positions are covered."""
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    p = ranks ** -1.1
    p /= p.sum()
    ids = rng.choice(vocab, size=(B, T), p=p).astype(np.int64)
    for b in range(B):
        covered = 0
        while covered < T // 10:
            L = int(rng.integers(8, 65))
            dst = int(rng.integers(L, T - L))
            src = int(rng.integers(0, dst - L + 1))
            ids[b, dst:dst + L] = ids[b, src:src + L]
            covered += L
    return ids


def profile_case_fn(case: str, dev):
    """The callable of one profile case on `dev` (built once, inputs resident)."""
    import torch

    from ksdraft_b200.kernels.gemm import gemm_out
    from ksdraft_b200.kernels.quant import quantize_cols, quantize_last_dim
    g = torch.Generator(device=dev).manual_seed(0)
    if case == "gemm_config1":
        # benchmark config 1: A (256, 1536) N(0,1), W (1536, 1536) N(0,0.02), GS128, fp32 out
        a = torch.randn(256, D_MODEL, device=dev, generator=g)
        w = torch.randn(D_MODEL, D_MODEL, device=dev, generator=g) * 0.02
        ac, as_ = quantize_last_dim(a)
        wc, ws = quantize_last_dim(w)
        out = torch.empty(256, D_MODEL, device=dev)
        fn = lambda: gemm_out(ac, as_, wc, ws, out=out)  # noqa: E731
    elif case == "gemm":
        a = torch.randint(-127, 128, (TOKENS, D_MODEL), dtype=torch.int8, device=dev, generator=g)
        w = torch.randint(-127, 128, (CHARTS, D_MODEL), dtype=torch.int8, device=dev, generator=g)
        sa = (torch.rand(TOKENS, D_MODEL // 128, device=dev, generator=g) * 0.01).half()
        sw = (torch.rand(CHARTS, D_MODEL // 128, device=dev, generator=g) * 0.01).half()
        out = torch.empty(TOKENS, CHARTS, dtype=torch.float16, device=dev)
        fn = lambda: gemm_out(a, sa, w, sw, out=out, clamp_f16=True)  # noqa: E731
    elif case == "quant":
        x = torch.randn(TOKENS, CHARTS, device=dev, generator=g)
        fn = lambda: quantize_last_dim(x)  # noqa: E731
    elif case == "quant_dither":
        # the master weight of the down projection, PTQR dither 0.5 (forward re-pack)
        from ksdraft_b200.kernels.quant import quantize_rows_into
        w = torch.randn(CHARTS, D_MODEL, device=dev, generator=g) * 0.02
        wc = torch.empty(CHARTS, D_MODEL, dtype=torch.int8, device=dev)
        ws = torch.empty(CHARTS, D_MODEL // 128, dtype=torch.float16, device=dev)
        fn = lambda: quantize_rows_into(w, wc, ws, dither=0.5, seed=1)  # noqa: E731
    elif case == "quant_cols":
        x = torch.randn(TOKENS, CHARTS, device=dev, generator=g).to(torch.bfloat16)
        fn = lambda: quantize_cols(x)  # noqa: E731
    elif case == "requant_t":
        hq = torch.randint(-127, 128, (TOKENS, CHARTS), dtype=torch.int8, device=dev,
                           generator=g)
        hs = (torch.rand(TOKENS, CHARTS // 128, device=dev, generator=g) * 0.01).half()
        fn = lambda: quantize_cols(hq, x_scales=hs)  # noqa: E731
    elif case in ("spine", "vjp"):
        from ksdraft_b200 import _lib
        from ksdraft_b200.kernels.ks3_int8 import make_tanh_lut, pack_small, spine_quant
        coeffs = torch.randn(CHARTS, 6, device=dev, generator=g) * 0.05
        rs = torch.full((CHARTS,), 0.75, device=dev)
        rh = torch.zeros(CHARTS, device=dev)
        p = pack_small(coeffs, rs, rh)
        coords = (torch.randn(TOKENS, CHARTS, device=dev, generator=g) * 0.5).half()
        if case == "spine":
            lut = make_tanh_lut(dev)
            fn = lambda: spine_quant(coords, *p, lut, "int8")  # noqa: E731
        else:
            value = (torch.randn(TOKENS, CHARTS, device=dev, generator=g) * 1e-3).half()
            nt = TOKENS // 128
            outs = [torch.empty(TOKENS, CHARTS, dtype=torch.int8, device=dev),
                    torch.empty(TOKENS, CHARTS // 128, dtype=torch.float16, device=dev),
                    torch.empty(CHARTS, TOKENS, dtype=torch.int8, device=dev),
                    torch.empty(CHARTS, nt, dtype=torch.float16, device=dev),
                    torch.empty(nt, 8, CHARTS, device=dev)]

            def fn():
                rc = _lib.lib().ksd8_ks3_vjp(value.data_ptr(), coords.data_ptr(), TOKENS, CHARTS,
                                             *(t.data_ptr() for t in p),
                                             *(o.data_ptr() for o in outs), None,
                                             _lib.stream_ptr(dev))
                _lib.check(rc, "vjp")
    elif case == "head":
        # LM head of one vocab shard: 4096 tokens x d 1536 x V 150144 (one GPU
        # holds the whole vocabulary), W8A8 logits + CE partials + gradient +
        # dgrad / wgrad, forward and backward
        from ksdraft_b200.model.head import VocabParallelHead
        V = 150144
        w = torch.randn(V, D_MODEL, device=dev, generator=g) * 0.02
        head = VocabParallelHead(w)
        x = torch.randn(TOKENS, D_MODEL, device=dev, generator=g).to(torch.bfloat16)
        tg = torch.randint(0, V, (TOKENS,), device=dev, generator=g)

        def fn():
            xd = x.detach().requires_grad_(True)
            head.weight.grad = None
            head.cross_entropy(xd, tg).backward()
    elif case in ("rosa_layer", "rosa_runs"):
        # config-4 layer shape, 16 x 2048 positions x 512 streams: independent fair
        # bits (rosa_layer; the chunked matcher keeps every stream) or bits that
        # flip with probability 0.1 per position (rosa_runs; long runs as deep-layer
        # projections give them, most streams handed to the sorted-key matcher)
        from ksdraft_b200.model.rosa import match_words, pack_bits
        B, T, S = 16, 2048, 512
        if case == "rosa_layer":
            bits = [(torch.rand(B, T, S, device=dev, generator=g) > 0.5).to(torch.int8)
                    for _ in range(3)]
        else:
            bits = []
            for _ in range(3):
                flips = (torch.rand(B, T, S, device=dev, generator=g) < 0.1).to(torch.int32)
                bits.append((torch.cumsum(flips, 1) & 1).to(torch.int8))
        words = [pack_bits(b, B, T, S, T * S, S, 1) for b in bits]
        del bits
        out = torch.empty(B, T, S, dtype=torch.bfloat16, device=dev)
        fn = lambda: match_words(*words, B, S, T, 62, out=out,  # noqa: E731
                                 strides=(T * S, S, 1))
    elif case in ("decode_step", "decode_step_delta"):
        # config 5's incremental match of one layer: 64 contexts x 512 streams
        # matched up to 8192 positions (fair bits), then blocks of 8 appended;
        # decode_step_delta: the main run ends 1024 positions earlier (the
        # middle of a rebuild cycle: 1024 delta keys compared directly)
        from ksdraft_b200.model.drafter import RosaDecodeState
        from ksdraft_b200.model.rosa import pack_bits
        C, S, T0, k = 64, 512, 8192, 8
        bits = [(torch.rand(C, T0, S, device=dev, generator=g) > 0.5).to(torch.int8)
                for _ in range(3)]
        st = RosaDecodeState(C, S, T0 + 512, dev)
        st.load_words([pack_bits(b, C, T0, S, T0 * S, S, 1) for b in bits], T0)
        del bits
        st.build(T0 - 1024 if case == "decode_step_delta" else T0)
        projs = [torch.randn(C, k, S, device=dev, generator=g) for _ in range(3)]
        pay = torch.ones(S, device=dev)
        out = torch.empty(C, k, S, dtype=torch.bfloat16, device=dev)
        fn = lambda: st.step(projs, T0, pay, out)  # noqa: E731  (re-appends the same block)
    elif case == "rosa_mixer":
        # config 3 end to end: RosaMixer(1536, 512) after to_int8 (Int8Linear q/k/v/out
        # projections N(0, 0.02)), evaluation forward on x = E[ids], E bf16 N(0, 1)
        # over the vocabulary, ids Zipf(1.1) with repeated spans, B 4 x T 4096
        from ksdraft_b200.kernels.linear import Int8Linear
        from ksdraft_b200.model.rosa import RosaMixer
        B, T, S = 4, 4096, 512
        torch.manual_seed(0)
        m = RosaMixer(D_MODEL, S).to(dev)
        with torch.no_grad():
            for n in ("q_proj", "k_proj", "v_proj", "out_proj"):
                getattr(m, n).weight.normal_(0, 0.02)
                getattr(m, n).bias.zero_()
        for n in ("q_proj", "k_proj", "v_proj", "out_proj"):
            setattr(m, n, Int8Linear.from_float(getattr(m, n)))
        m.eval()
        E = torch.randn(150144, D_MODEL, device=dev, generator=g).to(torch.bfloat16)
        x = E[torch.from_numpy(rosa_ids(B, T, seed=0)).to(dev)]
        del E

        def fn():
            with torch.no_grad():
                m(x)
    elif case == "rosa":
        # config 3: batch 4 x seq 4096, 512 streams (2048 stream sequences); bits
        # from Zipf(1.1) ids with repeated spans (length 8-64, 10% of positions)
        from ksdraft_b200.model.rosa import match_words, pack_bits
        B, T, S = 4, 4096, 512
        ids = rosa_ids(B, T, seed=0)
        idt = torch.from_numpy(ids).to(dev)
        salt = torch.arange(S, device=dev, dtype=torch.int64)
        bits = []
        for tag in (1, 2, 3):  # q, k, v: stand-ins for sign(proj(E[ids])) per stream
            h = (idt[:, :, None] * 0x9E3779B1 + salt[None, None, :] * 0x85EBCA77 + tag * 0xC2B2AE3D)
            h = (h ^ (h >> 15)) * 0x2C1B3C6D
            bits.append(((h >> 17) & 1).to(torch.int8).contiguous())   # (B, T, S)
        words = [pack_bits(b, B, T, S, T * S, S, 1) for b in bits]
        out = torch.empty(B, T, S, dtype=torch.float32, device=dev)
        fn = lambda: match_words(*words, B, S, T, 62, out=out,  # noqa: E731
                                 strides=(T * S, S, 1))
    else:
        raise SystemExit(f"unknown profile case {case}")
    return fn


def time_on_device(fn, iters: int) -> float:
    """ms per call of fn over `iters` back-to-back calls, CUDA events on the
    current stream.  The GPU is held by a spin kernel while the CPU enqueues,
    so host launch overhead does not enter the figure."""
    import torch
    fn()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(int(2e6) + iters * int(2e5))  # covers the enqueue of `iters` calls
    ev0.record()
    for _ in range(iters):
        fn()
    ev1.record()
    torch.cuda.synchronize()
    return ev0.elapsed_time(ev1) / iters


def side_measurements(dev) -> dict:
    """1-GPU figures of the other benchmark configurations, measured after the
    main line (outside its timed region): config 1 (W8A8 GEMM fwd), config 3
    (Rosa stream matcher, B 4 x T 4096 x 512 streams) and the LM head
    (4096 tokens x vocab 150144 on one GPU, forward + backward)."""
    out = {}
    ms = time_on_device(profile_case_fn("gemm_config1", dev), 200)
    ops = 2 * 256 * D_MODEL * D_MODEL
    out["config1_gemm"] = {"shape": [256, D_MODEL, D_MODEL], "ms": ms,
                           "tops": ops / (ms / 1e3) / 1e12, "unit": "TOP/s",
                           "note": "operands L2-resident (the whole problem is 2.8 MB)"}
    ms = time_on_device(profile_case_fn("rosa", dev), 5)
    out["config3_rosa_match"] = {"shape": [4, 4096, 512], "ms": ms,
                                 "positions_per_s": 4 * 4096 * 512 / (ms / 1e3),
                                 "note": "matcher alone on hash bits of the ids"}
    ms = time_on_device(profile_case_fn("rosa_mixer", dev), 5)
    out["config3_rosa_mixer"] = {"shape": [4, 4096, 512, D_MODEL], "ms": ms,
                                 "tokens_per_s": 4 * 4096 / (ms / 1e3),
                                 "gemm_gop": 4 * 2 * 4 * 4096 * D_MODEL * 512 / 1e9,
                                 "note": "RosaMixer int8 eval forward on E[Zipf ids]: time-mix "
                                         "+ quantise, 3 W8A8 GEMMs, bits, match, out_proj"}
    ms = time_on_device(profile_case_fn("head", dev), 3)
    out["lm_head_fwd_bwd"] = {"tokens": TOKENS, "vocab": 150144, "ms": ms,
                              "tokens_per_s": TOKENS / (ms / 1e3)}
    return out


def run_profile_case(case: str, iters: int) -> None:
    """One kernel of the layer step at its config-2 shape, `iters` launches after
    one warm-up (for ncu captures: small, single-kernel, ends by itself)."""
    import torch
    dev = torch.device("cuda", 0)
    fn = profile_case_fn(case, dev)
    fn()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(iters):
        fn()
    ev1.record()
    torch.cuda.synchronize()
    print(f"profile case {case}: {iters + 1} launches done, "
          f"{ev0.elapsed_time(ev1) / max(iters, 1):.4f} ms per launch (CUDA events)")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("config4", "config2", "config5"), default="config4")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--per-gpu-batch", type=int, default=None,
                    help="config4: this many sequences on every rank (weak scaling) "
                         "instead of the global batch of 16 split over the ranks")
    ap.add_argument("--no-graph", action="store_true",
                    help="config4 on one GPU: run the step eagerly instead of as a CUDA graph")
    ap.add_argument("--no-side", action="store_true",
                    help="skip the 1-GPU side figures (configs 1 and 3, LM head)")
    ap.add_argument("--profile-case", default=None,
                    help="run one kernel (gemm | gemm_config1 | quant | quant_dither | quant_cols | "
                         "requant_t | spine | vjp | head | rosa | rosa_mixer) a few times, "
                         "for ncu")
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()
    if args.profile_case:
        run_profile_case(args.profile_case, args.iters)
        return
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "config4":
        run_config4(args)
    elif args.workload == "config5":
        run_config5(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
