#!/usr/bin/env python
"""MoE-layer forward benchmark on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c5_ep|c3_prefill|c4_skewed|c2_decode]

A step is one MoE FFN layer forward (router -> dispatch -> gate/up GEMM with ERA -> down
GEMM -> combine -> aux loss) over one batch of synthetic tokens per GPU.  The default
workload is the expert-parallel layer quoted at 1/2/4/8 GPUs: 65,536 tokens per GPU,
d_model 4096, expert d_ff 2048, 64 experts, top-4, bf16; x ~ N(0,1), weights ~ N(0,0.02),
zero biases, FlyLoRA off.

* ``value``  tokens/s of the whole job, inputs resident in HBM, CUDA events around
  exactly K steps bracketed by barrier + synchronize, max over ranks.  Inputs (x: 512 MiB,
  weights: 3.2 GiB) are larger than the 126 MB L2, so no flush is needed between steps.
* ``e2e``    the same metric through the public API with x in pinned host memory and the
  output copied back to pinned host memory inside the timed region: on one GPU
  ``MoELayer.forward_host`` (token chunks whose copies overlap the layer), on N GPUs
  ``ExpertParallelMoE.forward_host`` (each rank's token chunks copied in and out while the
  other chunks exchange rows and run their GEMMs).
* ``workloads`` (one GPU) the other configurations -- decode, prefill, skewed with
  FlyLoRA, fp32 -- each timed after the headline region with its stage table, roofline and
  the CPU restatement beside it.
* ``ep_parity`` (N GPUs) every rank's output against a single-GPU forward of its tokens
  with all experts, after the timed regions.
* ``roofline`` the dominant kernel (the gate/up grouped GEMM) from CUDA events recorded
  around every launch of the timed region; algorithmic FLOPs = 4 * T * K * H * I.
* ``cpu_baseline`` the CPU restatement of the reference algorithm (the oracle, numpy fp32)
  on a bounded token sample of the same workload on this host's cores.
* ``--impl reference`` times that CPU implementation alone (no GPU work).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

# name -> (tokens per GPU, batch, hidden, inter, experts, top_k, lora_on, zipf_alpha)
WORKLOADS = {
    "c5_ep": dict(tokens=65536, batch=16, hidden=4096, inter=2048, experts=64, top_k=4),
    "c3_prefill": dict(tokens=32768, batch=8, hidden=2048, inter=8192, experts=8, top_k=2),
    "c4_skewed": dict(tokens=32768, batch=8, hidden=2048, inter=1024, experts=64, top_k=8,
                      lora_on=True, zipf_alpha=1.2),
    "c2_decode": dict(tokens=64, batch=64, hidden=2048, inter=8192, experts=8, top_k=2),
    # the fp32 correctness configuration (the reference's own CPU-runnable case): CUDA-core
    # GEMMs, fp32 end to end
    "c1_fp32": dict(tokens=512, batch=2, hidden=768, inter=3072, experts=8, top_k=2,
                    dtype="f32"),
    # the per-expert shape of c5_ep (4,096 rows per expert, d_model 4096, d_ff 2048) on 8
    # experts: small enough (a few GB on the device) for full profiler captures
    "c5_profile_e8": dict(tokens=16384, batch=4, hidden=4096, inter=2048, experts=8, top_k=2),
}
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of the gate|up
# GEMM, measured with ncu on the 8-expert slice of the c5_ep layer (c5_profile_e8: the same
# 4,096 rows per expert, d_model 4096, d_ff 2048) and scaled to the 64-expert launch by 8
GEMM1_TRAFFIC = {"c5_ep": {"bytes": 8 * 806_619_392,
                           "source": "ncu dram bytes of the 8-expert slice (c5_profile_e8) x 8"},
                 "c5_profile_e8": {"bytes": 806_619_392, "source": "ncu dram bytes"}}


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=list(WORKLOADS), default="c5_ep")
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="target CPU time of the cpu_baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-workloads", action="store_true",
                   help="on one GPU, skip timing the other configurations after the headline one")
    p.add_argument("--no-ep-parity", action="store_true",
                   help="on N GPUs, skip the bit-identity check of the expert-parallel output "
                        "against a single-GPU forward (run after the timed regions)")
    p.add_argument("--ep-chunks", type=int, default=0,
                   help="token chunks of the fused expert-parallel forward (overlap); "
                        "0 = 1 chunk up to 2 GPUs, 4 beyond (the measured best)")
    p.add_argument("--prenorm", action="store_true",
                   help="time the fused pre-norm block x + MoE(LayerNorm(x)) "
                        "(MoELayer.forward_residual) on one GPU, and beside it the unfused "
                        "torch LayerNorm -> MoELayer.forward -> torch add")
    p.add_argument("--backward", action="store_true",
                   help="time the training step instead: vmoe_forward_train + vmoe_backward "
                        "(dx, router / expert weight and bias gradients) on one GPU")
    p.add_argument("--ffn", action="store_true",
                   help="time the dense FeedForward (non-MoE layers) on the same GEMMs at the "
                        "workload's tokens / d_model / d_ff instead of the MoE layer")
    p.add_argument("--no-numa-bind", action="store_true",
                   help="leave the e2e host buffers wherever the process runs (default: bind "
                        "to the GPU's NUMA node before allocating them)")
    p.add_argument("--graph", action="store_true",
                   help="replay the single-GPU layer forward as a captured CUDA graph")
    p.add_argument("--host-chunks", type=int, default=0,
                   help="token chunks of the single-GPU host-buffer forward timed as e2e "
                        "(0 = automatic)")
    return p.parse_args()


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS, source="fallback")


def algorithmic(w, elt=2, logits=False):
    """Algorithmic work per forward: FLOPs of the expert GEMMs, bytes of the data stages.

    Router bytes are the ones the timed forward moves: x and W_r read, top-K indices and
    weights written, the per-128-token expert histograms and probability sums written;
    the T*E*4 bytes of router logits only when the forward returns them (``logits``).
    Expert weight bytes (read once per forward, every expert assumed to receive tokens)
    bound the decode-sized layer."""
    T, H, I, E, K = w["tokens"], w["hidden"], w["inter"], w["experts"], w["top_k"]
    nblk = -(-T // 128)
    return {
        "gemm1_flop": 4.0 * T * K * H * I,
        "gemm2_flop": 2.0 * T * K * H * I,
        "router_bytes": T * H * elt + E * H * elt + T * K * 8 + nblk * E * 8
                        + (T * E * 4 if logits else 0),
        "dispatch_bytes": T * H * elt + T * K * H * elt + T * K * 4,
        "combine_bytes": T * K * H * elt + T * K * 4 + T * H * elt,
        "gemm1_weight_bytes": E * 2 * I * H * elt,
        "gemm2_weight_bytes": E * H * I * elt,
    }


def cpu_model() -> str | None:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or None


# --------------------------------------------------------------------------------------
# clocks during the timed region
# --------------------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu_id: str):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-i", gpu_id, "-lms", "100"], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        for line in out.strip().splitlines():
            parts = [s.strip() for s in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, v in zip(self.NAMES, parts[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons)}


# --------------------------------------------------------------------------------------
# our implementation
# --------------------------------------------------------------------------------------
def build_layer(w, device, seed=0):
    import torch
    from velvetoptimizer_b200 import MoEConfig, MoELayer

    cfg = MoEConfig(hidden_size=w["hidden"], intermediate_size=w["inter"],
                    moe_num_experts=w["experts"], moe_top_k=w["top_k"], flylora_rank=16,
                    flylora_alpha=32.0, era_gamma=0.1)
    with torch.device(device):
        layer = MoELayer(cfg)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    with torch.no_grad():
        # VesperLM._init_weights: N(0, 0.02) weights, zero biases (model.py:456-467)
        for m in layer.modules():
            if isinstance(m, torch.nn.Linear):
                m.weight.normal_(0.0, 0.02, generator=g)
                m.bias.zero_()
        for e in layer.experts:
            for proj in (e.gate_proj, e.up_proj):
                if not w.get("lora_on"):
                    proj.lora_up.weight.zero_()  # FlyLoRA off
        if w.get("zipf_alpha"):
            ranks = torch.arange(1, w["experts"] + 1, dtype=torch.float64)
            pmf = ranks ** (-w["zipf_alpha"])
            layer.router.bias.copy_(torch.log(pmf / pmf.sum()).float())
    return layer


def global_weights(w, device, seed=0):
    """Stacked weights of all E experts (bf16), drawn like build_layer's, on `device`."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    E, H, I, r = w["experts"], w["hidden"], w["inter"], 16
    n = lambda *s: (torch.randn(*s, generator=g, device=device) * 0.02).to(torch.bfloat16)  # noqa: E731
    z = lambda *s: torch.zeros(*s, dtype=torch.bfloat16, device=device)  # noqa: E731
    out = {"router_w": n(E, H), "router_b": z(E), "down_w": n(E, H, I), "down_b": z(E, H)}
    for p in ("gate", "up"):
        out[f"{p}_w"], out[f"{p}_b"] = n(E, I, H), z(E, I)
        out[f"{p}_lora_down_w"], out[f"{p}_lora_down_b"] = n(E, r, H), z(E, r)
        out[f"{p}_lora_up_w"] = n(E, I, r) if w.get("lora_on") else z(E, I, r)
        out[f"{p}_lora_up_b"] = z(E, I)
    if w.get("zipf_alpha"):
        ranks = torch.arange(1, E + 1, dtype=torch.float64)
        pmf = ranks ** (-w["zipf_alpha"])
        out["router_b"] = torch.log(pmf / pmf.sum()).to(device=device, dtype=torch.bfloat16)
    return out


def cpu_baseline(layer, x_dev, w, seconds):
    """Time the oracle (CPU restatement of the reference, numpy fp32) on a token sample."""
    import numpy as np
    import torch
    from oracle import moe_oracle as O
    from oracle.inputs import MoECase

    st = layer.stacked_weights(torch.float32)
    names = {"router_w": "w_r", "router_b": "b_r", "gate_w": "w_g", "gate_b": "b_g",
             "up_w": "w_u", "up_b": "b_u", "down_w": "w_d", "down_b": "b_d",
             "gate_lora_down_w": "a_g", "gate_lora_down_b": "ba_g", "gate_lora_up_w": "l_g",
             "gate_lora_up_b": "bl_g", "up_lora_down_w": "a_u", "up_lora_down_b": "ba_u",
             "up_lora_up_w": "l_u", "up_lora_up_b": "bl_u"}
    p = {names[k]: v.cpu().numpy() for k, v in st.items()}
    del st
    case = MoECase(tokens=1, hidden=w["hidden"], inter=w["inter"], experts=w["experts"],
                   top_k=w["top_k"])
    xs = x_dev.float().cpu().numpy()

    def run(n):
        case.tokens = n
        p["x"] = xs[:n]
        t0 = time.perf_counter()
        O.moe_forward(p, case)
        return time.perf_counter() - t0

    n = min(256, xs.shape[0])
    t = run(n)
    n2 = int(min(xs.shape[0], max(n, n * seconds / max(t, 1e-3))))
    if n2 > n:
        n, t = n2, run(n2)
    return {"value": n / t, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "cpu_model": cpu_model(),
            "sample": f"{n} of {xs.shape[0]} tokens, numpy fp32 oracle (CPU restatement of "
                      f"python/vesper/model.py:317-385), {t:.1f} s"}


# what the expert-parallel forward's profiled stages hold (rank 0, its first token chunk)
EP_STAGE_NAMES = {"plan": "plan_publish_counts", "dispatch": "dispatch_nvlink_wait_rows",
                  "gemm2_down": "gemm2_down_push_rows", "combine": "signal_wait_combine"}


def stage_table(stages, alg, pk, scale=1.0, weight_bound=False, fp32=False, ep=False):
    """Per-stage ms, share, achieved rate and fraction of the measured peak.

    GEMM stages are FLOP-rated against the bf16 peak, except in a weight-bound
    (decode-sized) layer, where their weight bytes are rated against HBM; fp32 CUDA-core
    GEMMs have no measured peak.  ``scale`` is the share of the workload's tokens the
    profiled stages processed (the first token chunk of an expert-parallel forward)."""
    total = max(sum(stages.values()), 1e-9)
    rep = {}
    # a decode batch runs both expert GEMMs in one launch: its "gemm1" stage holds both
    merged = weight_bound and stages.get("gemm2_down", 0.0) < 0.01 * stages.get("gemm1_gate_up_era", 1.0)
    for name, t_ms in stages.items():
        rec = {"ms": round(t_ms, 4), "share": round(t_ms / total, 4)}
        sec = max(t_ms, 1e-9) * 1e-3
        if name.startswith(("gemm1", "gemm2")):
            key = name[:5]
            tf = alg[f"{key}_flop"] * scale / sec / 1e12
            if fp32:
                rec.update(achieved=round(tf, 2), unit="TFLOP/s", frac=None,
                           bound="fp32 CUDA cores (no measured peak)")
            elif weight_bound:
                if merged and key == "gemm2":
                    rec["note"] = "runs inside the gemm1 stage's launch"
                    rep[name] = rec
                    continue
                wbytes = alg[f"{key}_weight_bytes"]
                if merged:
                    wbytes += alg["gemm2_weight_bytes"]
                    tf = (alg["gemm1_flop"] + alg["gemm2_flop"]) * scale / sec / 1e12
                    rec["note"] = "gate|up and down GEMMs in one launch"
                gbs = wbytes / sec / 1e9
                rec.update(achieved=round(gbs, 1), unit="GB/s", frac=round(gbs / pk["hbm_gbs"], 4),
                           bound="hbm (expert weights read once)", tflops=round(tf, 2))
            else:
                rec.update(achieved=round(tf, 1), unit="TFLOP/s",
                           frac=round(tf / pk["bf16_tflops"], 4))
        elif name in ("router", "dispatch", "combine"):
            gbs = alg[f"{name}_bytes"] * scale / sec / 1e9
            rec.update(achieved=round(gbs, 1), unit="GB/s", frac=round(gbs / pk["hbm_gbs"], 4))
        rep[EP_STAGE_NAMES.get(name, name) if ep else name] = rec
    return rep


def time_workload(name, steps, warmup, dev, cpu_seconds, graph=False):
    """Tokens/s, stage table and roofline of one single-GPU workload (after the headline
    timed region, in the same process), with the CPU restatement timed beside it."""
    import torch
    w = dict(WORKLOADS[name])
    T, H, E, K = w["tokens"], w["hidden"], w["experts"], w["top_k"]
    f32 = w.get("dtype") == "f32"
    tdt = torch.float32 if f32 else torch.bfloat16
    layer = build_layer(w, dev, seed=0)
    packed = layer.packed_for(dev, tdt)
    g = torch.Generator(device=dev)
    g.manual_seed(1000)
    x = torch.randn(T, H, generator=g, device=dev).to(tdt).reshape(w["batch"], T // w["batch"], H)
    for _ in range(warmup):
        layer(x)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    e0.record(stream)
    for _ in range(steps):
        layer(x)
        launches += packed.handle.last_launch_count()
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    # the stage table from a second, profiled loop (stage events between kernels would end
    # their launch overlap inside the timed one)
    packed.handle.set_profiling(steps)
    for _ in range(steps):
        layer(x)
    torch.cuda.synchronize()
    stages, nprof = packed.handle.stage_times()
    packed.handle.set_profiling(0)
    pk = peaks()
    elt = 4 if f32 else 2
    alg = algorithmic(w, elt)
    weight_bound = name == "c2_decode"
    table = stage_table(stages, alg, pk, weight_bound=weight_bound, fp32=f32)
    top = max((k for k in table if k.startswith("gemm")), key=lambda k: table[k]["ms"])
    rec = {"ms_per_step": round(ms, 4), "tokens_per_s": round(T / (ms * 1e-3), 1),
           "dtype": "f32" if f32 else "bf16", "steps": steps, "warmup": warmup,
           "gpu_launches": launches,
           "config": f"{T} tokens, d_model {H}, expert d_ff {w['inter']}, {E} experts, top-{K}"
                     + (", FlyLoRA r16 on, Zipf(1.2) router bias" if w.get("lora_on") else ""),
           "stages": table,
           "roofline": dict(table[top], kernel=top, avg_launch_ms=table[top]["ms"],
                            launches_timed=nprof,
                            peak=None if f32 else (pk["hbm_gbs"] if weight_bound else pk["bf16_tflops"]),
                            peak_source=None if f32 else pk["source"] + (" HBM copy" if weight_bound
                                                                         else " bf16 burst"))}
    if graph:
        # the same forward replayed as one CUDA graph (it allocates nothing and never
        # synchronises the host, so it captures as is)
        cg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(cg):
            layer(x)
        for _ in range(warmup):
            cg.replay()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(steps):
            cg.replay()
        e1.record(stream)
        e1.synchronize()
        rec["graph_ms_per_step"] = round(e0.elapsed_time(e1) / steps, 4)
        del cg
    rec["cpu_baseline"] = cpu_baseline(layer, x.reshape(T, H), w, cpu_seconds)
    layer.close()
    del layer, packed, x
    torch.cuda.empty_cache()
    return rec


def check_ep_parity(layer, x2d, w, dev, world):
    """Outside the timed regions: this rank's tokens through the expert-parallel layer and
    through a single-GPU handle holding all E experts; the outputs must be bit-identical
    (the same kernels compute every row and the combine order is fixed)."""
    import ctypes

    import torch
    import torch.distributed as dist

    from velvetoptimizer_b200 import _lib
    out_ep, aux_ep = layer(x2d)  # every rank takes part
    torch.cuda.synchronize()
    status = layer.device_status()
    gw = global_weights(w, dev, seed=0)
    c = layer.cfg
    abi = _lib.VmoeConfig(hidden=c.hidden_size, inter=c.intermediate_size,
                          num_experts=c.moe_num_experts, top_k=c.moe_top_k,
                          lora_rank=c.flylora_rank, lora_scaling=c.lora_scaling,
                          era_gamma=c.era_gamma, dtype=_lib.VMOE_BF16, capacity=0)
    h = _lib.Handle(abi, dev.index)
    stream = torch.cuda.current_stream(dev).cuda_stream
    h.set_weights(_lib.VmoeWeights(**{k: ctypes.c_void_p(v.data_ptr()) for k, v in gw.items()}),
                  stream)
    T = x2d.shape[0]
    ws = torch.empty(h.workspace_size(T), dtype=torch.uint8, device=dev)
    out = torch.empty_like(x2d)
    aux = torch.empty((), dtype=torch.float32, device=dev)
    h.forward(x2d.data_ptr(), T, out.data_ptr(), None, None, None, None, aux.data_ptr(),
              ws.data_ptr(), ws.numel(), stream)
    torch.cuda.synchronize()
    same = bool(torch.equal(out, out_ep))
    aux_err = abs(aux.item() - aux_ep.item()) / max(abs(aux.item()), 1e-30)
    h.close()
    del gw, ws, out, out_ep
    torch.cuda.empty_cache()
    flags = torch.tensor([0.0 if same else 1.0, 1.0 if status else 0.0, aux_err], device=dev)
    dist.all_reduce(flags, op=dist.ReduceOp.MAX)
    return {"bit_identical": bool(flags[0].item() == 0.0), "tokens_checked": T * world,
            "device_status_clean": bool(flags[1].item() == 0.0),
            "aux_max_rel_err": float(flags[2].item()),
            "reference": "each rank's tokens through a single-GPU handle with all "
                         f"{c.moe_num_experts} experts (torch.equal of the outputs)"}


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    torch.set_grad_enabled(False)  # the forward (inference) step; --backward times training

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    w = dict(WORKLOADS[args.workload])
    T, H, E, K = w["tokens"], w["hidden"], w["experts"], w["top_k"]
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    f32 = w.get("dtype") == "f32"
    x = torch.randn(T, H, generator=g, device=dev).to(torch.float32 if f32 else torch.bfloat16).reshape(
        w["batch"], T // w["batch"], H)

    if args.ep_chunks <= 0:
        args.ep_chunks = 1 if world <= 2 else 4
    if world == 1:
        # the drop-in module (python/vesper/model.py MoELayer interface) on one GPU
        layer = build_layer(w, dev, seed=0)
        packed = layer.packed_for(dev, x.dtype)

        if args.prenorm:
            # the layer's ffn_norm (model.py:399) as _init_weights leaves it: ones, zeros
            norm = torch.nn.LayerNorm(H, eps=1e-6, device=dev, dtype=torch.bfloat16)

            def fwd(inp):
                return layer.forward_residual(inp, norm)
        else:
            def fwd(inp):
                return layer(inp)

        def start_profile():
            packed.handle.set_profiling(args.steps)

        def read_profile():
            return packed.handle.stage_times()

        def launches_of_last():
            return packed.handle.last_launch_count()
    else:
        # experts sharded over the ranks, rows exchanged with NCCL all-to-all-v
        from velvetoptimizer_b200 import MoEConfig
        from velvetoptimizer_b200.ep import ExpertParallelMoE
        cfg = MoEConfig(hidden_size=H, intermediate_size=w["inter"], moe_num_experts=E,
                        moe_top_k=K, flylora_rank=16, flylora_alpha=32.0, era_gamma=0.1)
        gw = global_weights(w, dev, seed=0)
        layer = ExpertParallelMoE(cfg, gw, dev, torch.bfloat16, transport="p2p", max_tokens=T,
                                  chunks=args.ep_chunks)
        del gw
        torch.cuda.empty_cache()

        def fwd(inp):
            out, aux = layer(inp.reshape(-1, H))
            return out.reshape(inp.shape), aux

        def start_profile():
            layer.set_profiling(args.steps)

        def read_profile():
            return layer.stage_times()

        def launches_of_last():
            return layer.launches

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up
    for _ in range(args.warmup):
        out, aux = fwd(x)
    torch.cuda.synchronize()
    graph_stages = None
    if args.graph and world == 1:
        # per-stage times from eager forwards first (a replayed graph records no new stage
        # events), then the whole layer forward captured once as a CUDA graph and replayed
        # every step (it allocates nothing and never synchronises the host, so it captures
        # as is)
        start_profile()
        for _ in range(args.steps):
            fwd(x)
        graph_stages = read_profile()
        packed.handle.set_profiling(0)  # no stage events inside the captured graph
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out, aux = fwd(x)
        graph_launches = launches_of_last()
        torch.cuda.synchronize()

        def fwd(inp):  # noqa: F811 - replays the captured forward on the same input buffer
            graph.replay()
            return out, aux

        def launches_of_last():  # noqa: F811
            return graph_launches

    # ---- device-resident timed region ----
    props = torch.cuda.get_device_properties(dev)
    gpu_id = str(getattr(props, "uuid", "") or local_rank)
    if gpu_id and not gpu_id.startswith("GPU-") and len(gpu_id) > 8:
        gpu_id = "GPU-" + gpu_id
    stream = torch.cuda.current_stream(dev)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(gpu_id)
    time.sleep(0.3)
    launches = 0
    t_start.record(stream)
    for _ in range(args.steps):
        out, aux = fwd(x)
        launches += launches_of_last()
    t_end.record(stream)
    t_end.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = t_start.elapsed_time(t_end) / args.steps
    if graph_stages is None:
        # the stage table from as many forwards again, each stage bracketed by CUDA events
        # (kept out of the timed loop: events between kernels end their launch overlap)
        start_profile()
        for _ in range(args.steps):
            fwd(x)
        torch.cuda.synchronize()
        stages, nprof = read_profile()
    else:
        stages, nprof = graph_stages
    ms_t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    value = world * T / (ms_max * 1e-3)

    prenorm_report = None
    if args.prenorm and world == 1:
        # the same block unfused: torch LayerNorm, the MoE layer, torch residual add
        def unfused(inp):
            o, a = layer(norm(inp))
            return inp + o, a
        for _ in range(args.warmup):
            unfused(x)
        torch.cuda.synchronize()
        u0 = torch.cuda.Event(enable_timing=True)
        u1 = torch.cuda.Event(enable_timing=True)
        u0.record(stream)
        for _ in range(args.steps):
            unfused(x)
        u1.record(stream)
        u1.synchronize()
        ms_u = u0.elapsed_time(u1) / args.steps
        elt = x.element_size()
        prenorm_report = {
            "fused_ms": round(ms, 4), "unfused_ms": round(ms_u, 4),
            "unfused": "torch LayerNorm -> MoELayer.forward -> torch residual add",
            "bytes_saved_per_step": 4 * T * H * elt,
            "note": "fused: LayerNorm folded into the router (row statistics from MMAs on the x "
                    "tile, folded weights) and the dispatch read, residual add in the combine"}

    # ---- end-to-end through the public module, host buffers in/out ----
    numa = None
    if not args.no_numa_bind:
        # pinned buffers next to the GPU's PCIe root (first touch on its NUMA node)
        from velvetoptimizer_b200.host import bind_to_device_node, device_numa_node
        numa = device_numa_node(local_rank)
        bind_to_device_node(local_rank)
    x_host = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    x_host.copy_(x)
    out_host = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    aux_host = torch.empty((), dtype=torch.float32, pin_memory=True)
    e2e_layer = None
    if world == 1 and not args.prenorm:
        # the layer's host-buffer forward: token chunks whose copies overlap the layer
        def e2e_step():
            _, a = layer.forward_host(x_host, device=dev, chunks=args.host_chunks, out=out_host)
            aux_host.copy_(a)
    elif world > 1:
        # the expert-parallel host-buffer forward: each token chunk's copies overlap the other
        # chunks' exchange and GEMMs, so it needs 2+ chunks; with a 1-chunk device layer it
        # gets its own 4-chunk layer
        e2e_layer = layer
        if layer.chunks < 2:
            gw = global_weights(w, dev, seed=0)
            e2e_layer = ExpertParallelMoE(cfg, gw, dev, torch.bfloat16, transport="p2p",
                                          max_tokens=T, chunks=4)
            del gw
            torch.cuda.empty_cache()
        x_host2d, out_host2d = x_host.reshape(-1, H), out_host.reshape(-1, H)

        def e2e_step():
            _, a = e2e_layer.forward_host(x_host2d, out=out_host2d)
            aux_host.copy_(a)
    else:
        def e2e_step():
            xd = x_host.to(dev, non_blocking=True)
            o, a = fwd(xd)
            out_host.copy_(o, non_blocking=True)
            aux_host.copy_(a, non_blocking=True)
    for _ in range(2):
        e2e_step()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    e1.synchronize()
    barrier()
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_value = world * T / (float(e2e_ms.item()) * 1e-3)

    e2e_chunks = e2e_layer.chunks if e2e_layer is not None else None
    if e2e_layer is not None and e2e_layer is not layer:
        e2e_layer.close()
    ep_parity = None
    if world > 1 and not args.no_ep_parity:
        ep_parity = check_ep_parity(layer, x.reshape(-1, H), w, dev, world)

    if rank != 0:
        return None

    pk = peaks()
    alg = algorithmic(w, x.element_size())
    g1 = stages.get("gemm1_gate_up_era", float("nan"))
    if world == 1:
        scale = 1.0
        roof_kernel = "gemm1_gate_up_era (tcgen05 grouped GEMM, fused ERA*up)"
    else:
        # rank 0's stages of its first token chunk; its local experts received the mean
        # t0*K rows for the t0 chunk tokens
        t0 = min(T, -(-(-(-T // args.ep_chunks)) // 128) * 128)
        scale = t0 / T
        roof_kernel = (f"gemm1_gate_up_era on rank 0's local experts, first of {args.ep_chunks} "
                       f"token chunks ({t0} tokens; FLOPs of the mean {t0}*K received rows)")
    roof_flop = alg["gemm1_flop"] * scale
    achieved = roof_flop / (g1 * 1e-3) / 1e12
    stage_report = stage_table(stages, alg, pk, scale=scale, fp32=f32, ep=world > 1)

    line = {
        "metric": "MoE-layer fwd tokens/s",
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_max, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32" if f32 else "bf16",
        "data": "synthetic: x~N(0,1), weights~N(0,0.02), zero bias, FlyLoRA off, seed 0",
        "config": {"workload": f"{args.workload}: MoE FFN layer fwd, {T} tokens/GPU, d_model {H}, "
                               f"expert d_ff {w['inter']}, {E} experts, top-{K}",
                   "tokens_per_gpu": T, "hidden": H, "inter": w["inter"], "experts": E,
                   "top_k": K,
                   "parallelism": "single GPU" if world == 1 else
                   f"expert parallel ep{world}: {E // world} experts/GPU, dispatch/combine "
                   f"over NVLink peer memory, {args.ep_chunks} overlapped token chunks",
                   "l2": "inputs larger than L2 (x 512 MiB, weights 3.2 GiB); no flush",
                   "cuda_graph": bool(args.graph and world == 1)},
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "host_numa_node": numa,
                "h2d_bytes_per_step": int(x.numel() * x.element_size()),
                "d2h_bytes_per_step": int(x.numel() * x.element_size() + 4),
                "api": "velvetoptimizer_b200.MoELayer.forward_host (vmoe_forward_host: "
                       "pinned host x/out, copies overlapped with the layer in token chunks)"
                       if world == 1 and not args.prenorm else
                       "velvetoptimizer_b200.MoELayer.forward_residual after a host copy"
                       if world == 1 else
                       "velvetoptimizer_b200.ep.ExpertParallelMoE.forward_host "
                       f"(vmoe_ep_p2p_forward_host: pinned host x/out, {e2e_chunks} token chunks "
                       "whose copies overlap the other chunks' exchange and GEMMs)"},
        "roofline": {"kernel": roof_kernel,
                     "bound": "tensor", "achieved": round(achieved, 1),
                     "peak": pk["bf16_tflops"], "peak_source": pk["source"] + " bf16 burst",
                     "unit": "TFLOP/s", "frac": round(achieved / pk["bf16_tflops"], 4),
                     "traffic": (GEMM1_TRAFFIC[args.workload]["bytes"]
                                 if world == 1 and args.workload in GEMM1_TRAFFIC else None),
                     "traffic_source": (GEMM1_TRAFFIC[args.workload]["source"]
                                        if world == 1 and args.workload in GEMM1_TRAFFIC else None),
                     "flop_per_launch": roof_flop,
                     "avg_launch_ms": round(g1, 4), "launches_timed": nprof},
        "stages": stage_report,
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if world > 1:
        line["stages_note"] = ("rank 0's first token chunk: plan includes publishing the counts "
                               "to every rank, dispatch the wait for every rank's rows, gemm2 the "
                               "NVLink push of the outputs when pushing, combine the signal and "
                               "wait for every rank's outputs")
    if ep_parity is not None:
        line["ep_parity"] = ep_parity
    if prenorm_report:
        line["prenorm"] = prenorm_report
        line["config"]["workload"] += "; fused pre-norm block x + MoE(LayerNorm(x))"
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(layer, x.reshape(T, H), w, args.cpu_seconds)
    if world == 1 and not args.no_workloads and not args.prenorm and not args.graph:
        # the other configurations, each timed after the headline region in this process
        layer.close()
        del layer, packed, x, x_host, out_host
        torch.cuda.empty_cache()
        extra = {}
        for name in ("c2_decode", "c3_prefill", "c4_skewed", "c1_fp32"):
            if name == args.workload:
                continue
            extra[name] = time_workload(name, min(args.steps, 20), max(3, min(args.warmup, 5)),
                                        dev, cpu_seconds=min(args.cpu_seconds, 4.0),
                                        graph=name == "c2_decode")
        line["workloads"] = extra
    return line


# --------------------------------------------------------------------------------------
# training step: forward that keeps its intermediates + backward
# --------------------------------------------------------------------------------------
def run_backward(args, rank, world, local_rank):
    import ctypes

    import torch

    from velvetoptimizer_b200 import _lib

    torch.set_grad_enabled(False)
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    w = dict(WORKLOADS[args.workload])
    T, H, I, E, K = w["tokens"], w["hidden"], w["inter"], w["experts"], w["top_k"]
    layer = build_layer(w, dev, seed=0)
    h = layer.packed_for(dev, torch.bfloat16).handle
    stream = torch.cuda.current_stream(dev)
    h.set_training(True, stream.cuda_stream)
    g = torch.Generator(device=dev)
    g.manual_seed(2000 + rank)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    dout = (torch.randn(T, H, generator=g, device=dev) * 1e-2).to(torch.bfloat16)
    daux = torch.full((1,), 0.01, device=dev)  # the reference's moe_aux_loss_weight
    saved_b, scratch_b = h.train_workspace_size(T)
    saved = torch.empty(saved_b, dtype=torch.uint8, device=dev)
    scratch = torch.empty(scratch_b, dtype=torch.uint8, device=dev)
    out = torch.empty_like(x)
    aux = torch.empty(1, device=dev)
    dx = torch.empty_like(x)
    f = dict(device=dev, dtype=torch.float32)
    grads = {"router_w": torch.empty(E, H, **f), "router_b": torch.empty(E, **f),
             "gate_w": torch.empty(E, I, H, **f), "gate_b": torch.empty(E, I, **f),
             "up_w": torch.empty(E, I, H, **f), "up_b": torch.empty(E, I, **f),
             "down_w": torch.empty(E, H, I, **f), "down_b": torch.empty(E, H, **f)}
    vg = _lib.VmoeGrads(**{k: ctypes.c_void_p(v.data_ptr()) for k, v in grads.items()})
    ev_mid = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    launches = [0]

    def step(i=None, e0=None):
        h.forward_train(x.data_ptr(), T, out.data_ptr(), None, aux.data_ptr(), saved.data_ptr(),
                        saved_b, stream.cuda_stream)
        n = h.last_launch_count()
        if i is not None:
            ev_mid[i].record(stream)
        h.backward(x.data_ptr(), dout.data_ptr(), T, daux.data_ptr(), dx.data_ptr(), vg,
                   saved.data_ptr(), saved_b, scratch.data_ptr(), scratch_b, stream.cuda_stream)
        launches[0] += n + h.last_launch_count()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert h.device_status(stream.cuda_stream) == 0
    props = torch.cuda.get_device_properties(dev)
    gpu_id = str(getattr(props, "uuid", "") or local_rank)
    if gpu_id and not gpu_id.startswith("GPU-") and len(gpu_id) > 8:
        gpu_id = "GPU-" + gpu_id
    h.set_profiling(args.steps)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    torch.cuda.synchronize()
    sampler = ClockSampler(gpu_id)
    time.sleep(0.3)
    launches[0] = 0
    for i in range(args.steps):
        starts[i].record(stream)
        step(i)
    starts[args.steps].record(stream)
    starts[args.steps].synchronize()
    clocks = sampler.stop()
    ms = starts[0].elapsed_time(starts[args.steps]) / args.steps
    fwd_ms = statistics.mean(starts[i].elapsed_time(ev_mid[i]) for i in range(args.steps))
    bwd_ms = statistics.mean(ev_mid[i].elapsed_time(starts[i + 1]) for i in range(args.steps))
    stages, nprof = h.backward_stage_times()
    assert h.device_status(stream.cuda_stream) == 0
    pk = peaks()
    flop = {"dh_glu_bwd_gemm": 2.0 * T * K * H * I, "dx_gemm": 4.0 * T * K * H * I,
            "wgrad_down": 2.0 * T * K * H * I, "wgrad_gate_up": 4.0 * T * K * H * I,
            "router_dx_gemm": 2.0 * T * E * H}
    e = 2
    byts = {"combine_bwd": T * H * e + 2 * T * K * H * e + T * K * 4,
            "dx_gather": T * K * H * e + 2 * T * H * e,
            "transposes": 2 * e * (T * K * (2 * H + 3 * I) + T * H + T * E)}
    rep = {}
    for name, t_ms in stages.items():
        rec = {"ms": round(t_ms, 4), "share": round(t_ms / max(sum(stages.values()), 1e-9), 4)}
        if name in flop:
            a = flop[name] / (t_ms * 1e-3) / 1e12
            rec.update(achieved=round(a, 1), unit="TFLOP/s", frac=round(a / pk["bf16_tflops"], 4))
        elif name in byts:
            a = byts[name] / (t_ms * 1e-3) / 1e9
            rec.update(achieved=round(a, 1), unit="GB/s", frac=round(a / pk["hbm_gbs"], 4))
        rep[name] = rec
    top = max(flop, key=lambda k: stages.get(k, 0.0))  # the backward kernel that takes longest
    top_ms = stages[top]
    achieved = flop[top] / (top_ms * 1e-3) / 1e12
    return {
        "metric": "MoE-layer training step (fwd + bwd) tokens/s",
        "value": round(T / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "fwd_ms": round(fwd_ms, 4), "bwd_ms": round(bwd_ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: x~N(0,1), dout~N(0,1e-4), weights~N(0,0.02), zero bias, FlyLoRA off",
        "config": {"workload": f"{args.workload}: MoE FFN layer training step, {T} tokens, "
                               f"d_model {H}, expert d_ff {I}, {E} experts, top-{K}; outputs dx and "
                               f"fp32 router / expert weight and bias gradients",
                   "l2": "inputs larger than L2; no flush"},
        "e2e": None,
        "roofline": {"kernel": top, "bound": "tensor", "achieved": round(achieved, 1),
                     "peak": pk["bf16_tflops"], "peak_source": pk["source"] + " bf16 burst",
                     "unit": "TFLOP/s", "frac": round(achieved / pk["bf16_tflops"], 4),
                     "traffic": None, "flop_per_launch": flop[top], "avg_launch_ms": round(top_ms, 4),
                     "launches_timed": nprof},
        "stages": rep,
        "gpu_launches": launches[0],
        "clocks": clocks,
    }


# --------------------------------------------------------------------------------------
# dense FeedForward (python/vesper/model.py:249-270) on the same grouped GEMMs
# --------------------------------------------------------------------------------------
def run_ffn(args, rank, world, local_rank):
    import torch

    from velvetoptimizer_b200 import FeedForward, MoEConfig

    torch.set_grad_enabled(False)
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    w = dict(WORKLOADS[args.workload])
    T, H, I = w["tokens"], w["hidden"], w["inter"]
    cfg = MoEConfig(hidden_size=H, intermediate_size=I, flylora_rank=16, flylora_alpha=32.0,
                    era_gamma=0.1)
    with torch.device(dev):
        ffn = FeedForward(cfg)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    for m in ffn.modules():
        if isinstance(m, torch.nn.Linear):
            m.weight.normal_(0.0, 0.02, generator=g)
            m.bias.zero_()
    for proj in (ffn.gate_proj, ffn.up_proj):
        proj.lora_up.weight.zero_()
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16).reshape(w["batch"], -1, H)
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        ffn(x)
    torch.cuda.synchronize()
    props = torch.cuda.get_device_properties(dev)
    gpu_id = str(getattr(props, "uuid", "") or local_rank)
    if gpu_id and not gpu_id.startswith("GPU-") and len(gpu_id) > 8:
        gpu_id = "GPU-" + gpu_id
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(gpu_id)
    time.sleep(0.3)
    e0.record(stream)
    for _ in range(args.steps):
        ffn(x)
    e1.record(stream)
    e1.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    pk = peaks()
    flop = 6.0 * T * H * I
    achieved = flop / (ms * 1e-3) / 1e12
    return {
        "metric": "dense FeedForward fwd tokens/s", "value": round(T / (ms * 1e-3), 1),
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: x~N(0,1), weights~N(0,0.02), zero bias, FlyLoRA off",
        "config": {"workload": f"{args.workload} shape, dense FeedForward (non-MoE layer): "
                               f"{T} tokens, d_model {H}, d_ff {I}",
                   "l2": "inputs larger than L2; no flush"},
        "e2e": None,
        "roofline": {"kernel": "gate|up GEMM + down GEMM (whole layer)", "bound": "tensor",
                     "achieved": round(achieved, 1), "peak": pk["bf16_tflops"],
                     "peak_source": pk["source"] + " bf16 burst", "unit": "TFLOP/s",
                     "frac": round(achieved / pk["bf16_tflops"], 4), "traffic": None,
                     "flop_per_launch": flop},
        "gpu_launches": 3 * args.steps,
        "clocks": clocks,
    }


# --------------------------------------------------------------------------------------
# reference arm: the CPU implementation of the path (the oracle port) on host cores
# --------------------------------------------------------------------------------------
def run_reference(args):
    import numpy as np
    import torch
    from oracle import moe_oracle as O
    from oracle.inputs import MoECase

    w = dict(WORKLOADS[args.workload])
    T, H, I, E, K = w["tokens"], w["hidden"], w["inter"], w["experts"], w["top_k"]
    r = 16
    torch.manual_seed(0)
    gen = lambda *s: torch.empty(*s).normal_(0.0, 0.02).numpy()  # noqa: E731
    z = lambda *s: np.zeros(s, dtype=np.float32)  # noqa: E731
    p = {"w_r": gen(E, H), "b_r": z(E), "w_d": gen(E, H, I), "b_d": z(E, H)}
    for q in ("g", "u"):
        p[f"w_{q}"], p[f"b_{q}"] = gen(E, I, H), z(E, I)
        p[f"a_{q}"], p[f"ba_{q}"] = gen(E, r, H), z(E, r)
        p[f"l_{q}"] = gen(E, I, r) if w.get("lora_on") else z(E, I, r)
        p[f"bl_{q}"] = z(E, I)
    if w.get("zipf_alpha"):
        from oracle.inputs import zipf_router_bias
        p["b_r"] = zipf_router_bias(E, w["zipf_alpha"])
    xs = torch.randn(min(T, 8192), H).numpy()
    case = MoECase(tokens=1, hidden=H, inter=I, experts=E, top_k=K)

    def step(n):
        case.tokens = n
        p["x"] = xs[:n]
        t0 = time.perf_counter()
        O.moe_forward(p, case)
        return time.perf_counter() - t0

    # size the per-step sample so warm-up + steps take about two minutes
    n = 128
    t = step(n)
    budget = 120.0 / max(1, args.steps + args.warmup)
    n = int(min(xs.shape[0], max(64, n * budget / max(t, 1e-3))))
    for _ in range(args.warmup):
        step(n)
    times = [step(n) for _ in range(args.steps)]
    med = statistics.median(times)
    value = n / med
    return {
        "metric": "MoE-layer fwd tokens/s", "impl": "reference", "value": round(value, 2),
        "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(med * 1e3, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (same shapes and distributions)",
        "config": {"workload": args.workload, "tokens_per_step": n, "hidden": H, "inter": I,
                   "experts": E, "top_k": K},
        "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": os.cpu_count(),
                         "kind": "port", "cpu_model": cpu_model(),
                         "sample": f"{n} tokens per step of the {T}-token workload, numpy fp32 "
                                   "oracle (CPU restatement of python/vesper/model.py:317-385)"},
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return 0
    import torch
    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    if args.backward or args.ffn:
        if world > 1:
            raise SystemExit("--backward / --ffn run on one GPU")
        run = run_backward if args.backward else run_ffn
        print(json.dumps(run(args, rank, world, local_rank)), flush=True)
        return 0
    try:
        line = run_ours(args, rank, world, local_rank)
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
