#!/usr/bin/env python
"""Benchmark: RWKV-v7 L12 D768 GPT-mode prefill tok/s on B200 (one process per GPU).

Default workload (the one BASELINE.json's metric is quoted on, configs[1]): a randomly
initialised L12 D768 model (12 heads x 64, ChannelMix hidden 3072, vocab 65568;
fp16 weights with fp32 decay bias w0, orthogonal init as rwkv_mlx/train.py:209-310),
prefill of a global batch of B=8 sequences x T=4096 uniform-random tokens, split
over the GPUs by sequence (8/4/2/1 per GPU at 1/2/4/8 GPUs; strong scaling, no
collective on the data path).  `value` is the tokens of all ranks per second over the
max-over-ranks step time.  The same JSON line carries `secondary` measurements taken
in the same run: the weak-scaled prefill (B=8 per GPU), the WKV-7 forward and
backward kernels at B=8 T=4096 H=12 with their HBM roofline fractions, the LoRA-MoE
ChannelMix layer of configs[3] (and its expert-parallel form over NCCL at N>1), and
the batched decode of configs[2].

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload prefill|wkv_fwd|wkv_bwd|decode|moe|moe_full|head_loss|config5]

Multi-GPU: launched by torch.distributed.run (RANK/LOCAL_RANK/WORLD_SIZE from the
environment).  `--impl reference` times the CPU restatement of the reference
path (the reference itself is MLX/Metal and cannot run here) on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CFG_L12 = dict(n_layer=12, n_embd=768, vocab_size=65568, dim_ffn=3072)


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------
def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d.get("bf16_tflops"), "measured"
    return 6650.0, 1590.0, "fallback"


def dist_setup():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([float(x)], device="cuda", dtype=torch.float64)
    dist.all_reduce(t)
    return float(t.item())


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, dev):
        self.proc = None
        self.tmp = tempfile.TemporaryDirectory(prefix="rwkv_bench_clocks_")
        self.out = Path(self.tmp.name) / "clocks.csv"
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
            self.fh = open(self.out, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", uuid, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            self.tmp.cleanup()
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                smax = max(smax, float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        self.tmp.cleanup()
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def cuda_timed(fn, steps, stream=None):
    """Run fn() `steps` times between CUDA events on the current stream; ms per step."""
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")  # lets a profiler select the timed launches
    e0.record(s)
    for _ in range(steps):
        fn()
    e1.record(s)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def cuda_timed_flushed(fn, steps):
    """Like cuda_timed for inputs that fit in L2: before every step a 256 MB buffer is
    written (evicting L2) outside the timed interval; each step is bracketed by its own
    CUDA events and the per-step times are averaged."""
    s = torch.cuda.current_stream()
    buf = torch.empty(64 * 1024 * 1024, device=s.device, dtype=torch.float32)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.nvtx.range_push("timed")
    for e0, e1 in ev:
        buf.zero_()
        e0.record(s)
        fn()
        e1.record(s)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    return sum(e0.elapsed_time(e1) for e0, e1 in ev) / steps


# ---------------------------------------------------------------------------
# model construction
# ---------------------------------------------------------------------------
def build_model(dev, cfg_kw, seed=0, dtype=torch.float16):
    from rwkv_mlx_b200.model import RWKV, RWKVConfig, cast_for_inference, init_weights

    cfg = RWKVConfig(**cfg_kw)
    with torch.device(dev):
        m = RWKV(cfg)
    init_weights(m, seed=seed)
    cast_for_inference(m, dtype)
    m.eval()
    return cfg, m


def wkv_algo_bytes(B, T, H, act_bytes, w_bytes):
    """Algorithmic HBM bytes of one forward launch: r,k,v,a,b,y in the activation
    dtype + w in its own dtype (7*E*s when all share one dtype)."""
    E = B * T * H * 64
    return E * (6 * act_bytes + w_bytes)


def cpu_prefill_sample(cfg_kw, tokens_T, steps, seed=0):
    """The reference path on the host cores, on a bounded sample (B=1, T=tokens_T): the
    reference's own WKV-7 Metal kernel body compiled for the CPU (oracle/_ref, built from
    the reference's sources by oracle/build_ref.py; 64 host threads per threadgroup with
    real barriers, as mx.fast.metal_kernel launches it) inside the CPU restatement of the
    model shell (oracle/model_oracle.py).  Where oracle/_ref was not built, the C
    restatement of that kernel (oracle/wkv7_metal_port.c, OpenMP) stands in."""
    from oracle import cpu_wkv7
    from oracle import model_oracle as mo
    from rwkv_mlx_b200.model import RWKV, RWKVConfig, init_weights

    torch.set_num_threads(os.cpu_count() or 1)
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count()))
    cfg = RWKVConfig(**cfg_kw)
    with torch.device("cpu"):
        m = RWKV(cfg)
    init_weights(m, seed=seed)
    sd = {k: v.detach().float() for k, v in m.state_dict().items()}
    del m
    g = torch.Generator().manual_seed(seed)
    idx = torch.randint(0, 65536, (1, tokens_T), generator=g)

    def timed(mode, n):
        with torch.no_grad():
            mo.forward(sd, cfg, idx, wkv=mode)  # warm-up
            times = []
            for _ in range(n):
                t0 = time.perf_counter()
                mo.forward(sd, cfg, idx, wkv=mode)
                times.append(time.perf_counter() - t0)
        return tokens_T / statistics.median(times)

    ref = cpu_wkv7.ref_available()
    value = timed("ref" if ref else "port", steps)
    port = timed("port", steps) if ref else value
    kernel = ("the reference's own WKV-7 Metal kernel body compiled for the CPU (oracle/_ref)" if ref else
              "oracle/wkv7_metal_port.c (C restatement of the reference kernel, OpenMP)")
    return {"value": value, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "reference" if ref else "port",
            "sample": f"L12 D768 GPT-mode forward, fp32, B=1 T={tokens_T}, median of {steps} steps; WKV-7: "
                      f"{kernel}; model shell: oracle/model_oracle.py (torch CPU)",
            "port_value": port,
            "port_note": "the same sample with the WKV-7 recurrence in the OpenMP C restatement of the reference "
                         "kernel (the emulated Metal launch pays for host-thread barriers at every step)"}


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
def split_batch(B_global: int, ws: int, rank: int) -> int:
    """Sequences of a global batch this rank runs (B=8 split over
    the GPUs, 8/4/2/1 per GPU at 1/2/4/8 GPUs)."""
    return B_global // ws + (1 if rank < B_global % ws else 0)


def run_prefill(args, ws, rank, dev, B, model=None, strong=True, with_e2e=True):
    """GPT-mode prefill of B sequences x T tokens on this rank, one CUDA-graph replay of
    the model's forward per step (model.PrefillGraph); `value` = tokens of all ranks /
    max-over-ranks time.  The WKV-7 forward's duration for the roofline is measured with
    CUDA events around each call on its stream in eager steps right after (the kernels
    and their inputs are the same as inside the graph)."""
    from rwkv_mlx_b200 import _native, check_device_error, wkv7
    from rwkv_mlx_b200.model import PrefillGraph

    T = args.seq
    if model is None:
        cfg, model = build_model(dev, CFG_L12, seed=0)
    cfg = model.config
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    idx = torch.randint(0, 65536, (B, T), device=dev, generator=g)
    host_idx = idx.cpu().pin_memory()
    host_out = torch.empty((B, cfg.vocab_size), dtype=torch.float16).pin_memory()

    def eager_step():
        with torch.no_grad():
            logits, _ = model(idx)
        return logits

    for _ in range(args.warmup):
        eager_step()
    torch.cuda.synchronize()
    l0 = _native.launch_count
    eager_step()
    per_step_launches = _native.launch_count - l0  # this repository's kernels in one forward
    graph = PrefillGraph(model, B, T, warmup=1)
    graph(idx)  # inputs resident in the graph's buffer from here on
    for _ in range(args.warmup):
        graph()

    def step():
        return graph()[0]

    torch.cuda.synchronize()

    # ---- device-resident timed region ----
    barrier(ws)
    torch.cuda.synchronize()
    clk = ClockSampler(dev)
    ms = cuda_timed(step, args.steps)
    clocks = clk.stop()
    barrier(ws)
    launches = per_step_launches * args.steps
    check_device_error()
    # WKV-7 forward duration per call (events on its stream), eager steps of the same batch
    wkv7.fwd_timings = []
    cuda_timed(eager_step, args.steps)
    kt = [a.elapsed_time(b) for a, b in wkv7.fwd_timings]
    wkv7.fwd_timings = None
    check_device_error()
    ms_max = max_over_ranks(ms, ws)
    tok_all = sum_over_ranks(B * T, ws)
    value = tok_all / (ms_max / 1e3)

    e2e = None
    if with_e2e:
        # ---- end-to-end through the public API, host buffers ----

        def e2e_step():
            logits, _ = graph(host_idx)  # H2D from pinned host memory into the graph's input
            host_out.copy_(logits[:, -1], non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        barrier(ws)
        t0 = time.perf_counter()
        e2e_ms = cuda_timed(e2e_step, args.steps)
        wall_ms = (time.perf_counter() - t0) * 1e3 / args.steps
        e2e_ms = max_over_ranks(max(e2e_ms, wall_ms), ws)
        e2e = {"value": tok_all / (e2e_ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": B * T * 8,
               "d2h_bytes_per_step": B * cfg.vocab_size * 2,
               "path": "model.PrefillGraph (RWKV.forward captured as a CUDA graph) via the public API; tokens H2D "
                       "from pinned host, last-position logits D2H"}

    hbm, _, src = peaks()
    H = cfg.n_head
    bytes_launch = wkv_algo_bytes(B, T, H, 2, 4)
    k_ms = statistics.mean(kt) if kt else float("nan")
    k_ms = max_over_ranks(k_ms, ws)
    achieved = bytes_launch / (k_ms / 1e3) / 1e9
    B_global = sum_over_ranks(B, ws)
    line = {
        "metric": "prefill tok/s (L12 D768)", "value": value, "unit": "tok/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
        "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "fp16 (fp32 WKV state)",
        "data": "synthetic: random-init weights, uniform-random tokens",
        "config": {"workload": "L12 D768 GPT-mode prefill (BASELINE configs[1])" if strong else
                   "L12 D768 GPT-mode prefill, B=8 per GPU (weak scaling)",
                   "model": "RWKV-v7 L12 D768", "global_batch": B_global, "batch_per_gpu": B, "seq_len": T,
                   "parallelism": f"dp{ws} (batch split, no collective on the data path)", "cuda_graph": True,
                   "l2": "per-step working set (4.3 GB logits at B=8, 0.37 GB weights) far larger than L2"},
        "gpu_launches": launches,
        "roofline": {"kernel": "wkv7_fwd (rwkv_wkv7_forward_ws: tcgen05 forward, plus transition + scan "
                               "launches when the sequence is segmented)",
                     "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "traffic": traffic_for("wkv7_fwd", B, T, H),
                     "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured" else "fallback 6650 GB/s",
                     "algorithmic_bytes_per_launch": bytes_launch, "launch_ms": k_ms, "launches_timed": len(kt),
                     "launch_timing": "CUDA events around each WKV-7 forward call on its stream, eager steps "
                                      "after the graph-timed region",
                     "wkv_share_of_step": (k_ms * len(kt) / args.steps) / ms_max if kt else None},
        "clocks": clocks,
    }
    if e2e is not None:
        line["e2e"] = e2e
    return line, model


def traffic_for(kernel, B, T, H):
    """Per-launch DRAM bytes from the committed ncu summary (scaled by units), or None."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text()).get(kernel)
    if not d:
        return None
    return d["bytes_per_unit"] * B * T * H


def run_wkv(args, ws, rank, dev, backward=False, B=None):
    """WKV-7 op alone at config-2 scale (B=8, T=4096, H=12 per GPU, fp16 + fp32 w).  Below
    B=4 the inputs fit in L2, so L2 is flushed before every step (outside the timing)."""
    from rwkv_mlx_b200 import check_device_error, wkv7

    B, T, H = (args.batch if B is None else B), args.seq, 12
    C = H * 64
    g = torch.Generator(device=dev).manual_seed(rank)
    mk = lambda: torch.randn(B, T, C, device=dev, generator=g).half()
    r, k, v = mk(), mk(), mk()
    w = torch.empty(B, T, C, device=dev).uniform_(-6, -0.5, generator=g)
    kk = torch.nn.functional.normalize(torch.randn(B, T, H, 64, device=dev, generator=g), dim=-1).view(B, T, C)
    a = (-kk).half()
    b = (kk * torch.sigmoid(torch.randn(B, T, C, device=dev, generator=g))).half()
    dy = mk()
    if backward:
        _, ck, _, _ = wkv7._fwd(r, w, k, v, a, b, want_ckpt=True)
        fn = lambda: wkv7._bwd(r, w, k, v, a, b, dy, ck)
        nbytes = B * T * C * (12 * 2 + 4)
    else:
        fn = lambda: wkv7.wkv7(r, w, k, v, a, b)
        nbytes = wkv_algo_bytes(B, T, H, 2, 4)
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    barrier(ws)
    clk = ClockSampler(dev)
    flush = B < 4
    ms = cuda_timed_flushed(fn, args.steps) if flush else cuda_timed(fn, args.steps)
    clocks = clk.stop()
    check_device_error()
    ms = max_over_ranks(ms, ws)
    hbm, _, src = peaks()
    gbs = nbytes / (ms / 1e3) / 1e9
    name = "wkv7_bwd" if backward else "wkv7_fwd"
    return {"metric": f"{name} HBM GB/s", "value": gbs * ws, "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16 (fp32 w, fp32 state)", "data": "synthetic (config 1 distributions)",
            "config": {"workload": f"{name} B={B} T={T} H={H}",
                       "l2": "flushed before every step (256 MB write, untimed)" if flush else "inputs larger than L2"},
            "roofline": {"kernel": name, "bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                         "frac": gbs / hbm, "traffic": traffic_for(name, B, T, H), "peak_source": src},
            "clocks": clocks}


def run_moe(args, ws, rank, dev, ep=None):
    """One LoRA-MoE ChannelMix layer: D=768, hidden 3072, E=8,
    r=16, top-2, 65536 tokens per GPU, per-expert logit bias N(0, 1.5); each rank
    routes its own tokens over a replica of the experts (no collective)."""
    from rwkv_mlx_b200 import _native
    from rwkv_mlx_b200.model import RWKV_CMix_x070, RWKVConfig
    from rwkv_mlx_b200.moe import LoRAMoE_CMix

    ep = (args.ep if ep is None else ep) and ws > 1
    ntok, C = args.moe_tokens, 768
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    cfg = RWKVConfig(n_embd=C, dim_ffn=3072)
    gw = torch.Generator(device=dev).manual_seed(7)  # same weights on every rank
    with torch.device(dev):
        base = RWKV_CMix_x070(cfg, 1)
        if ep:
            from rwkv_mlx_b200.ep import ExpertParallelLoRAMoE

            layer = ExpertParallelLoRAMoE(base, n_experts=8, lora_rank=16, top_k=2)
        else:
            layer = LoRAMoE_CMix(base, n_experts=8, lora_rank=16, top_k=2)
    with torch.no_grad():
        base.x_k.uniform_(0, 1, generator=gw)
        base.key.weight.normal_(0, C ** -0.5, generator=gw)
        base.value.weight.normal_(0, 3072 ** -0.5, generator=gw)
        A = torch.randn(8, C, 16, device=dev, generator=gw) * 0.02
        Bw = torch.randn(8, 16, C, device=dev, generator=gw) * 0.02
        if ep:
            layer.load_experts(A, Bw)
        else:
            layer.lora_A.copy_(A)
            layer.lora_B.copy_(Bw)
        layer.router.gate.weight.normal_(0, C ** -0.5, generator=gw)
    layer = layer.half()
    layer.router.bias = torch.randn(8, device=dev, generator=gw) * 1.5
    x = torch.randn(1, ntok, C, device=dev, generator=g).half()

    def step():
        with torch.no_grad():
            return layer(x)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    l0 = _native.launch_count
    barrier(ws)
    clk = ClockSampler(dev)
    ms = cuda_timed(step, args.steps)
    clocks = clk.stop()
    launches = _native.launch_count - l0
    ms = max_over_ranks(ms, ws)
    # MoE-path kernels alone (the module's path: the router folded into the fused adapter
    # apply for fp16, else router + apply) on the same tokens
    from rwkv_mlx_b200.moe import lora_apply, lora_apply_routed, lora_apply_routed_supported, router_forward

    x2 = x.view(ntok, C)
    with torch.no_grad():
        base_out = base(x).view(ntok, C)
    Ah, Bh = A.half(), Bw.half()
    routed = lora_apply_routed_supported(C, 16, 8, 2, x2.dtype)

    def moe_only():
        if routed:
            return lora_apply_routed(x2, base_out, Ah, Bh, layer.router.gate.weight, 2, layer.router.bias,
                                     out=base_out)[0]
        r = router_forward(x2, layer.router.gate.weight, 2, layer.router.bias)
        return lora_apply(x2, base_out, Ah, Bh, r["inds"], r["scores"], out=base_out)  # as the module does

    for _ in range(args.warmup):
        moe_only()
    moe_ms = cuda_timed(moe_only, args.steps)  # local kernels on this rank's tokens (also under --ep)
    hbm, _, src = peaks()
    algo = ntok * (3 * C * 2 + 2 * (4 + 2))  # x read, base read, out write, inds+scores
    gbs = algo / (moe_ms / 1e3) / 1e9
    return {"metric": "LoRA-MoE ChannelMix tok/s", "value": ntok * ws / (ms / 1e3), "unit": "tok/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (fp32 router)", "data": "synthetic",
            "config": {"workload": "LoRA-MoE CMix D768 F3072 E8 r16 top2 (BASELINE configs[3])",
                       "tokens_per_gpu": ntok,
                       "parallelism": f"ep{ws} (NCCL all-to-all)" if ep else f"dp{ws} (experts replicated)",
                       "l2": "x and outputs (3 x 100 MB) larger than L2"},
            "gpu_launches": launches,
            "roofline": {"kernel": "MoE path (rwkv_moe_lora_apply_routed: router folded into the fused apply, + "
                                   "gate split and finalize)" if routed else "MoE path (router + fused lora_apply)",
                         "bound": "hbm", "achieved": gbs,
                         "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "traffic": traffic_for("moe_path_routed" if routed else "moe_path", ntok, 1, 1),
                         "launch_ms": moe_ms,
                         "algorithmic_bytes": algo, "peak_source": src},
            "clocks": clocks}


def run_moe_full(args, ws, rank, dev):
    """One full-expert MoE ChannelMix layer (MoE_CMix, moe.py:170-242) at the config-4
    shapes: D=768, hidden 3072, E=8 full experts, top-2, 65536 tokens per GPU, per-expert
    logit bias N(0, 1.5); experts replicated on every rank (no collective)."""
    from rwkv_mlx_b200 import _native
    from rwkv_mlx_b200.model import RWKVConfig
    from rwkv_mlx_b200.moe import MoE_CMix

    ntok, C, F, E, k = args.moe_tokens, 768, 3072, 8, 2
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    gw = torch.Generator(device=dev).manual_seed(7)
    with torch.device(dev):
        layer = MoE_CMix(RWKVConfig(n_embd=C, dim_ffn=F), 1, E, k)
    with torch.no_grad():
        layer.x_k.uniform_(0, 1, generator=gw)
        layer.expert_key.normal_(0, C ** -0.5, generator=gw)
        layer.expert_val.normal_(0, F ** -0.5, generator=gw)
        layer.router.gate.weight.normal_(0, C ** -0.5, generator=gw)
    layer = layer.half()
    layer.router.bias = torch.randn(E, device=dev, generator=gw) * 1.5
    seq = 4096
    x = torch.randn(ntok // seq, seq, C, device=dev, generator=g).half()

    def step():
        with torch.no_grad():
            return layer(x)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    l0 = _native.launch_count
    barrier(ws)
    clk = ClockSampler(dev)
    ms = cuda_timed(step, args.steps)
    clocks = clk.stop()
    launches = _native.launch_count - l0
    ms = max_over_ranks(ms, ws)
    _, tflops, src = peaks()
    flop = ntok * k * 4 * C * F  # two products of 2*C*F flops per routed (token, expert)
    achieved = flop / (ms / 1e3) / 1e12
    return {"metric": "full-expert MoE ChannelMix tok/s", "value": ntok * ws / (ms / 1e3), "unit": "tok/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (fp32 router, fp32 accumulate)",
            "data": "synthetic",
            "config": {"workload": "MoE_CMix D768 F3072 E8 top2, config-4 shapes", "tokens_per_gpu": ntok,
                       "parallelism": f"dp{ws} (experts replicated)",
                       "l2": "x, routed rows and key activations (0.8 GB) larger than L2"},
            "gpu_launches": launches,
            "roofline": {"kernel": "whole layer (expert GEMMs on cuBLAS dominate)", "bound": "tensor",
                         "achieved": achieved, "peak": tflops, "unit": "TFLOP/s", "frac": achieved / tflops,
                         "traffic": None, "algorithmic_flop": flop, "peak_source": src},
            "clocks": clocks}


def run_head_loss(args, ws, rank, dev):
    """Output head + training loss (train.py:317-334, 483-489) at the prefill shapes of
    hidden states (B=8, T=4096, C=768) fp16, head (65568, 768),
    uniform-random targets; forward and backward of the fused head + loss (the logits
    are formed and consumed one 8192-column vocabulary chunk at a time)."""
    from rwkv_mlx_b200 import _native
    from rwkv_mlx_b200.loss import head_l2_wrap_loss

    B, T, C, V = args.batch, args.seq, 768, 65568
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    x = torch.randn(B, T, C, device=dev, generator=g).half().requires_grad_(True)
    w = (torch.randn(V, C, device=dev, generator=g) * C ** -0.5).half().requires_grad_(True)
    tg = torch.randint(0, V, (B, T), device=dev, generator=g)

    def step():
        x.grad = None
        w.grad = None
        loss = head_l2_wrap_loss(x, w, tg)
        loss.backward()
        return loss

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats(dev)
    base_mem = torch.cuda.memory_allocated(dev)
    l0 = _native.launch_count
    barrier(ws)
    clk = ClockSampler(dev)
    ms = cuda_timed(step, args.steps)
    clocks = clk.stop()
    launches = _native.launch_count - l0
    peak_extra = torch.cuda.max_memory_allocated(dev) - base_mem
    ms = max_over_ranks(ms, ws)
    _, tflops, src = peaks()
    n = B * T
    flop = 3 * 2 * n * V * C  # logits, d/dx, d/dW (the backward's recomputed logits not credited)
    achieved = flop / (ms / 1e3) / 1e12
    return {"metric": "fused head + l2_wrap_loss fwd+bwd tok/s", "value": n * ws / (ms / 1e3), "unit": "tok/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (fp32 softmax statistics)", "data": "synthetic",
            "config": {"workload": f"head+loss B={B} T={T} C={C} V={V}, chunk 8192",
                       "full_logits_bytes": n * V * 2, "peak_extra_bytes": int(peak_extra),
                       "l2": "logit chunks (0.5 GB) larger than L2"},
            "gpu_launches": launches,
            "roofline": {"kernel": "whole head + loss (GEMMs on cuBLAS dominate)", "bound": "tensor",
                         "achieved": achieved, "peak": tflops, "unit": "TFLOP/s", "frac": achieved / tflops,
                         "traffic": None, "algorithmic_flop": flop, "peak_source": src},
            "clocks": clocks}


def run_decode(args, ws, rank, dev, model=None):
    """Batched RNN-mode decode: L12 D768, 256 sequences per GPU whose
    state comes from a 512-token GPT-mode prefill, greedy steps; tok/s over all ranks."""
    from rwkv_mlx_b200 import _native

    Bs, P = args.decode_seqs, args.decode_prompt
    if model is None:
        cfg, model = build_model(dev, CFG_L12, seed=0)
    l0_build = None
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    prompt = torch.randint(0, 65536, (Bs, P), device=dev, generator=g)
    with torch.no_grad():
        logits, _, states = model.forward_with_state(prompt)
        tok = logits[:, -1].argmax(-1)
        del logits
    from rwkv_mlx_b200.model import DecodeGraph

    l_pre = _native.launch_count
    graph = DecodeGraph(model, states, tok, warmup=0)
    l_graph = _native.launch_count
    l0_build = l_pre  # launches recorded once in the graph, replayed per step

    def step():
        graph.step()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    l0 = _native.launch_count
    barrier(ws)
    clk = ClockSampler(dev)
    ms = cuda_timed(step, args.steps)
    clocks = clk.stop()
    launches = (l_graph - l0_build) * args.steps  # our kernels captured per step x replays
    ms = max_over_ranks(ms, ws)
    hbm, _, src = peaks()
    # the state step kernel's bytes: state read+write + 7 vectors per (seq, head), 12 layers
    return {"metric": "decode tok/s (L12 D768, 256 seqs)", "value": Bs * ws / (ms / 1e3), "unit": "tok/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (fp32 state)", "data": "synthetic",
            "config": {"workload": "RNN-mode greedy decode (BASELINE configs[2])", "seqs_per_gpu": Bs,
                       "prompt": P, "parallelism": f"dp{ws}", "cuda_graph": True},
            "gpu_launches": launches, "clocks": clocks}


def run_config5(args, ws, rank, dev):
    """L24 D1024 RWKV-v7 (16 heads x 64, vocab 65568, ChannelMix
    hidden 3584 = the reference's default for C=1024, model.py:46-47) with LoRA-MoE (E=8,
    top-2, rank 16; adapters and gate ~ N(0, 0.02)) in every ChannelMix, fp16 weights,
    fp32 state.  One step = GPT-mode prefill of a global B=32 x T=4096 (split over the
    ranks by sequence) + a WKV-7 forward/backward micro-batch of B=4 x T=1024 x H=16
    (its 64 (b, h) units split over the ranks, by sequence then by head).  At N>1 every
    LoRA-MoE layer is expert-parallel (experts e on rank e // (8 / N), NCCL all-to-all)."""
    from rwkv_mlx_b200 import _native, check_device_error, wkv7

    T, C, H = args.seq, 1024, 16
    B = split_batch(32, ws, rank)
    cfg_kw = dict(n_layer=24, n_embd=C, vocab_size=65568, moe_num_experts=8, moe_top_k=2, moe_lora_rank=16)
    cfg, model = build_model(dev, cfg_kw, seed=0)
    gw = torch.Generator(device=dev).manual_seed(17)  # identical adapters on every rank
    with torch.no_grad():
        for i, blk in enumerate(model.blocks):
            f = blk.ffn
            A = (torch.randn(8, C, 16, device=dev, generator=gw) * 0.02).to(f.lora_A.dtype)
            Bw = (torch.randn(8, 16, C, device=dev, generator=gw) * 0.02).to(f.lora_B.dtype)
            f.router.gate.weight.copy_(torch.randn(8, C, device=dev, generator=gw) * 0.02)
            if ws > 1:
                from rwkv_mlx_b200.ep import ExpertParallelLoRAMoE

                with torch.device(dev):
                    e = ExpertParallelLoRAMoE(f.base, 8, 16, 2)
                e.load_experts(A.float(), Bw.float())
                e.router.gate.weight.copy_(f.router.gate.weight.float())
                e.lora_A.data = e.lora_A.data.to(torch.float16)
                e.lora_B.data = e.lora_B.data.to(torch.float16)
                e.router.gate.weight.data = e.router.gate.weight.data.to(torch.float16)
                blk.ffn = e
            else:
                f.lora_A.copy_(A)
                f.lora_B.copy_(Bw)
    for p_ in model.parameters():
        p_.requires_grad_(False)
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    idx = torch.randint(0, 65536, (B, T), device=dev, generator=g)
    # WKV-7 backward micro-batch: 4 x 16 = 64 (b, h) units over the ranks
    units = 64 // ws
    mb_B = max(1, 4 // ws)
    mb_H = units // mb_B
    Tm = 1024
    mk = lambda: torch.randn(mb_B, Tm, mb_H * 64, device=dev, generator=g).half()
    r_, k_, v_, dy = mk(), mk(), mk(), mk()
    w_ = torch.empty(mb_B, Tm, mb_H * 64, device=dev).uniform_(-6, -0.5, generator=g)
    kk = torch.nn.functional.normalize(torch.randn(mb_B, Tm, mb_H, 64, device=dev, generator=g), dim=-1)
    a_ = (-kk).reshape(mb_B, Tm, -1).half()
    b_ = (kk.reshape(mb_B, Tm, -1) * torch.sigmoid(torch.randn(mb_B, Tm, mb_H * 64, device=dev, generator=g))).half()

    def micro_bwd():
        _, ck, _, _ = wkv7._fwd(r_, w_, k_, v_, a_, b_, want_ckpt=True)
        return wkv7._bwd(r_, w_, k_, v_, a_, b_, dy, ck)

    def step():
        with torch.no_grad():
            logits, aux = model(idx)
        micro_bwd()
        return logits

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    l0 = _native.launch_count
    barrier(ws)
    clk = ClockSampler(dev)
    ms = cuda_timed(step, args.steps)
    clocks = clk.stop()
    barrier(ws)
    launches = _native.launch_count - l0
    check_device_error()
    ms_max = max_over_ranks(ms, ws)
    mb_ms = max_over_ranks(cuda_timed(micro_bwd, args.steps), ws)
    tok_all = sum_over_ranks(B * T, ws)
    hbm, _, src = peaks()
    bwd_bytes = mb_B * Tm * mb_H * 64 * (12 * 2 + 4)
    return {"metric": "configs[4] step: L24 D1024 LoRA-MoE prefill tok/s (+ WKV-7 bwd micro-batch)",
            "value": tok_all / (ms_max / 1e3), "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp16 (fp32 WKV state, fp32 router)", "data": "synthetic",
            "config": {"workload": "BASELINE configs[4]", "model": "RWKV-v7 L24 D1024, LoRA-MoE E8 r16 top2 in every "
                       "ChannelMix", "global_batch": 32, "batch_per_gpu": B, "seq_len": T,
                       "bwd_micro_batch": {"global": "B=4 T=1024 H=16", "per_gpu": f"B={mb_B} H={mb_H}"},
                       "parallelism": f"dp{ws} + ep{ws} (NCCL all-to-all)" if ws > 1 else "1 GPU"},
            "gpu_launches": launches,
            "wkv7_bwd_micro_batch": {"ms": mb_ms, "achieved_gbs": bwd_bytes / (mb_ms / 1e3) / 1e9,
                                     "frac": bwd_bytes / (mb_ms / 1e3) / 1e9 / hbm,
                                     "note": "forward with snapshots + exact chunked backward"},
            "clocks": clocks}


def run_reference(args):
    """The reference path on the host cores (see cpu_prefill_sample), rank 0 only; the
    other ranks of a multi-GPU launch exit without work."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    sample_T = args.cpu_sample_tokens
    res = cpu_prefill_sample(CFG_L12, sample_T, max(1, args.steps))
    return {"impl": "reference", "metric": "prefill tok/s (L12 D768)", "value": res["value"], "unit": "tok/s",
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "fp32", "data": "synthetic",
            "config": {"workload": "L12 D768 GPT-mode prefill (BASELINE configs[1]), bounded CPU sample"},
            "cpu_baseline": res,
            "e2e": {"value": res["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference is MLX/Metal (MLX is not installable offline, no Apple GPU): its own WKV-7 "
                    "Metal kernel body runs compiled for the host CPU inside a CPU restatement of the model"}


def _brief(d):
    keep = ("metric", "value", "unit", "ms_per_step", "scaling", "n_gpus", "config", "roofline", "gpu_launches",
            "e2e", "clocks")
    return {k: d[k] for k in keep if k in d}


def secondary_lines(args, ws, rank, dev, model, primary):
    """Per-GPU workloads measured in the same run as the headline, each timed on its own
    with CUDA events (max over ranks) and reported with its own roofline where it has
    one: the weak-scaled prefill (B=8 per GPU), the WKV-7 forward and backward at
    B=8 T=4096 H=12, the backward at B=1, the LoRA-MoE ChannelMix layer of BASELINE configs[3] (replicated
    experts, and expert-parallel over NCCL all-to-all at N>1) and the batched decode of
    BASELINE configs[2]."""
    out = {}
    if ws > 1 or args.weak or primary["config"]["batch_per_gpu"] != 8:
        out["prefill_weak_b8_per_gpu"] = _brief(run_prefill(args, ws, rank, dev, 8, model=model, strong=False,
                                                            with_e2e=False)[0])
    else:
        out["prefill_weak_b8_per_gpu"] = "same as the headline at this GPU count (B=8 on one GPU)"
    out["wkv7_fwd_b8_t4096_h12"] = _brief(run_wkv(args, ws, rank, dev, backward=False, B=8))
    out["wkv7_bwd_b8_t4096_h12"] = _brief(run_wkv(args, ws, rank, dev, backward=True, B=8))
    # one sequence per GPU (configs[1] over 8 GPUs): the segmented adjoint chain
    out["wkv7_bwd_b1_t4096_h12"] = _brief(run_wkv(args, ws, rank, dev, backward=True, B=1))
    out["lora_moe_cmix_config3"] = _brief(run_moe(args, ws, rank, dev, ep=False))
    if ws > 1:
        out["lora_moe_cmix_config3_ep"] = _brief(run_moe(args, ws, rank, dev, ep=True))
    out["decode_config2"] = _brief(run_decode(args, ws, rank, dev, model=model))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="prefill",
                    choices=["prefill", "wkv_fwd", "wkv_bwd", "moe", "moe_full", "head_loss", "decode",
                             "config5"])
    ap.add_argument("--moe-tokens", type=int, default=65536)
    ap.add_argument("--ep", action="store_true", help="moe workload: expert-parallel over the ranks")
    ap.add_argument("--decode-seqs", type=int, default=256)
    ap.add_argument("--decode-prompt", type=int, default=512)
    ap.add_argument("--wkv-impl", type=int, default=0, choices=[0, 1, 2, 3],
                    help="WKV-7 forward kernel: 0 auto (tcgen05 for fp16/bf16), 1 step-sequential, "
                         "2 mma.sync chunked, 3 tcgen05 chunked")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--cpu-sample-tokens", type=int, default=128)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--weak", action="store_true",
                    help="prefill: --batch sequences per GPU instead of a global batch split over the GPUs")
    ap.add_argument("--no-secondary", action="store_true",
                    help="prefill: skip the secondary measurements (weak-scaled prefill, WKV-7 forward and "
                         "backward, LoRA-MoE layer, expert-parallel MoE at N>1, decode)")
    args = ap.parse_args()

    if args.impl == "reference":
        line = run_reference(args)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    ws, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.wkv_impl:
        from rwkv_mlx_b200 import _native

        _native.check(_native.lib().rwkv_set_wkv_impl(args.wkv_impl), "rwkv_set_wkv_impl")
    if args.workload == "prefill":
        B = args.batch if args.weak else split_batch(args.batch, ws, rank)
        line, model = run_prefill(args, ws, rank, dev, B, strong=not args.weak)
        if not args.no_secondary:
            line["secondary"] = secondary_lines(args, ws, rank, dev, model, line)
    elif args.workload == "moe":
        line = run_moe(args, ws, rank, dev)
    elif args.workload == "moe_full":
        line = run_moe_full(args, ws, rank, dev)
    elif args.workload == "head_loss":
        line = run_head_loss(args, ws, rank, dev)
    elif args.workload == "decode":
        line = run_decode(args, ws, rank, dev)
    elif args.workload == "config5":
        line = run_config5(args, ws, rank, dev)
    else:
        line = run_wkv(args, ws, rank, dev, backward=args.workload == "wkv_bwd")
    if rank == 0 and ws == 1 and not args.no_cpu_baseline and args.workload == "prefill":
        line["cpu_baseline"] = cpu_prefill_sample(CFG_L12, args.cpu_sample_tokens, 2)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
