"""MoE-layer throughput on B200: `python bench.py --gpus N --steps K --warmup W`.

Workload (BASELINE config 2 / 4): DeepSeek-V2-Lite-shaped MoE layer, hidden
2048, 64 routed experts top-6 (softmax router), intermediate 1408 with SwiGLU,
2 always-on shared experts (intermediate 2816), bf16, T tokens per GPU
(default 4096, the prefill point), x ~ N(0,1), weights ~ N(0,0.02), seed 0.
One step = one full layer forward (router -> grouping + gather -> expert FFN
-> combine) through the public API. Weights (1.1 GB) exceed the 126 MB L2, so
no flush is needed between steps. At N > 1 the 64 experts are sharded
evenly across ranks (expert parallel), each rank holding T tokens.

`--impl reference` times the reference algorithm's CPU restatement (the
oracle; the reference is pure PyTorch and cannot travel to the GPU box) on a
bounded sample of the same workload with all host threads.
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H, E, K_TOP, I, I_SHARED = 2048, 64, 6, 1408, 2816
METRIC = "MoE-layer tokens/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return PEAKS_FALLBACK, "fallback"


def layer_flops(t: int) -> float:
    return 2.0 * t * K_TOP * 3 * H * I + 2.0 * t * 3 * H * I_SHARED + 2.0 * t * H * E


def gateup_flops(rows: int, t_shared: int) -> float:
    return 2.0 * rows * H * 2 * I + 2.0 * t_shared * H * 2 * I_SHARED


def layer_bytes(counts, t: int, w_bytes: int = 2) -> int:
    active = sum(1 for c in counts if c > 0)
    return active * 3 * H * I * w_bytes + 3 * H * I_SHARED * 2 + E * H * 2 + t * H * 2 + t * H * 2


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.15)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in Path(self.path).read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------- distributed
def dist_setup(n: int):
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # plain NCCL all-to-all; NVLS multicast is neither needed nor wanted
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return rank, world, local


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ---------------------------------------------------------------- reference arm
def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    from threadpoolctl import threadpool_limits

    from oracle import moe_oracle as O

    cores = os.cpu_count() or 1
    t_sample = args.ref_tokens
    rng = np.random.default_rng(0)
    # Only the experts a sample routes to are touched; all 64 are generated.
    f32 = lambda *s: (rng.standard_normal(s, dtype=np.float32) * np.float32(0.02))  # noqa: E731
    gate, up, down = f32(E, I, H), f32(E, I, H), f32(E, H, I)
    router = f32(E, H)
    shared = (f32(I_SHARED, H), f32(I_SHARED, H), f32(H, I_SHARED))
    x = rng.standard_normal((t_sample, H), dtype=np.float32)
    times = []
    with threadpool_limits(limits=cores):
        for step in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            O.moe_forward(x, router, gate, up, down, K_TOP, shared=shared)
            dt = time.perf_counter() - t0
            if step >= args.warmup:
                times.append(dt)
    sec = statistics.mean(times)
    value = t_sample / sec
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"C2 DeepSeek-V2-Lite MoE layer, {t_sample}-token sample of the T={args.tokens} step",
                   "hidden": H, "experts": E, "top_k": K_TOP, "intermediate": I, "shared_intermediate": I_SHARED,
                   "tokens_per_gpu": args.tokens, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{t_sample} tokens x {args.steps} steps of the numpy oracle (f32) forward"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_sample(seconds: float = 12.0) -> dict:
    """The oracle's forward on a bounded sample, rank 0 / N=1 only."""
    import numpy as np
    from threadpoolctl import threadpool_limits

    from oracle import moe_oracle as O

    cores = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    f32 = lambda *s: (rng.standard_normal(s, dtype=np.float32) * np.float32(0.02))  # noqa: E731
    gate, up, down = f32(E, I, H), f32(E, I, H), f32(E, H, I)
    router = f32(E, H)
    shared = (f32(I_SHARED, H), f32(I_SHARED, H), f32(H, I_SHARED))
    t_sample = 128
    x = rng.standard_normal((t_sample, H), dtype=np.float32)
    n = 0
    with threadpool_limits(limits=cores):
        O.moe_forward(x, router, gate, up, down, K_TOP, shared=shared)
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < seconds or n < 2:
            O.moe_forward(x, router, gate, up, down, K_TOP, shared=shared)
            n += 1
        sec = (time.perf_counter() - t0) / n
    return {"value": t_sample / sec, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{n} x {t_sample}-token forwards of the numpy oracle (f32, all experts resident)"}


# ---------------------------------------------------------------- B200 arm
def make_inputs(t: int, seed: int, dev):
    import torch

    from dispatch_b200.kernels.moe_forward import SharedExpertWeights, StackedExpertWeights

    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*s, sc=0.02):
        return (torch.randn(*s, generator=g, device=dev) * sc).to(torch.bfloat16)

    router = rnd(E, H)
    ws = StackedExpertWeights(rnd(E, I, H), rnd(E, I, H), rnd(E, H, I))
    sh = SharedExpertWeights(rnd(I_SHARED, H), rnd(I_SHARED, H), rnd(H, I_SHARED))
    gx = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(t, H, generator=gx, device=dev).to(torch.bfloat16)
    return x, router, ws, sh


def time_loop(fn, steps: int, warmup: int, world: int, stream) -> float:
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return start.elapsed_time(end) / steps


def run_b200(args) -> None:
    import torch

    from dispatch_b200 import _lib as L
    from dispatch_b200.kernels.layer import RouterConfig, moe_layer_forward

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    peaks, peak_kind = load_peaks()
    t = args.tokens
    x, router, ws, sh = make_inputs(t, seed=rank * 1000, dev=dev)
    cfg = RouterConfig(top_k=K_TOP)
    bias = None
    if args.routing == "zipf":
        import numpy as np

        bias = torch.from_numpy((-1.2 * np.log(np.arange(E) + 1.0)).astype(np.float32)).to(dev)

    if world > 1:
        from dispatch_b200.kernels.expert_parallel import EPLayer

        ep = EPLayer(router, ws, sh, cfg, rank=rank, world=world, e_score_bias=bias)
        step = lambda: ep(x)  # noqa: E731
        launches_per_step = ep.launches_per_step
        parallelism = f"ep{world}"
    else:
        step = lambda: moe_layer_forward(x, router, ws, cfg, shared=sh, e_score_bias=bias)  # noqa: E731
        launches_per_step = 7  # router GEMM + select, group x2, gate/up GEMM, down GEMM, combine
        parallelism = "single"

    res = moe_layer_forward(x, router, ws, cfg, shared=sh, e_score_bias=bias)
    torch.cuda.synchronize()
    L.check_device_status(dev)
    counts = res.group_sizes.cpu().tolist()

    with ClockSampler(local) as clocks:
        ms = time_loop(step, args.steps, args.warmup, world, stream)
    ms = max_over_ranks(ms, world)
    L.check_device_status(dev)
    value = t * world / (ms * 1e-3)

    # e2e: the public call with host buffers (pinned), copies inside the timed region
    x_host = x.cpu().pin_memory()
    out_host = torch.empty(t, H, dtype=torch.bfloat16).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        out = ep(x_dev) if world > 1 else moe_layer_forward(x_dev, router, ws, cfg, shared=sh, e_score_bias=bias).out
        out_host.copy_(out, non_blocking=True)

    e2e_ms = max_over_ranks(time_loop(e2e_step, max(args.steps // 2, 3), 3, world, stream), world)
    e2e_val = t * world / (e2e_ms * 1e-3)

    # dominant kernel: the gate/up tcgen05 GEMM (+SwiGLU epilogue), timed alone
    roof = gateup_roofline(x, ws, sh, res, peaks, peak_kind, dev, stream)

    sweep = {}
    if world == 1 and not args.no_sweep:
        for tt in (1, 16, 128, 1024):
            xs_ = x[:tt].contiguous()
            r = moe_layer_forward(xs_, router, ws, cfg, shared=sh, e_score_bias=bias)
            torch.cuda.synchronize()
            c = r.group_sizes.cpu().tolist()
            m = time_loop(lambda: moe_layer_forward(xs_, router, ws, cfg, shared=sh, e_score_bias=bias),
                          200, 10, 1, stream)
            b = layer_bytes(c, tt)
            sweep[str(tt)] = {"ms": round(m, 4), "tokens_per_s": round(tt / (m * 1e-3), 1),
                              "hbm_gbs_algorithmic": round(b / (m * 1e-3) / 1e9, 1),
                              "hbm_frac": round(b / (m * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)}
        sweep["4096"] = {"ms": round(ms, 4), "tokens_per_s": round(value, 1),
                         "tflops_algorithmic": round(layer_flops(t) / (ms * 1e-3) / 1e12, 1),
                         "tensor_frac": round(layer_flops(t) / (ms * 1e-3) / 1e12 / peaks["bf16_tflops"], 4)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"C2 DeepSeek-V2-Lite MoE layer (H2048 E64 top6 I1408 + 2 shared), "
                                   f"T={t} tokens/GPU, {args.routing} routing",
                       "hidden": H, "experts": E, "top_k": K_TOP, "intermediate": I, "shared_intermediate": I_SHARED,
                       "tokens_per_gpu": t, "global_tokens": t * world, "routing": args.routing,
                       "parallelism": parallelism, "l2": "inputs larger than L2 (1.1 GB of weights per step)"},
            "layer_tflops_algorithmic": round(layer_flops(t) / (ms * 1e-3) / 1e12, 1),
            "roofline": roof,
            "e2e": {"value": round(e2e_val, 1), "unit": "tokens/s", "h2d_bytes_per_step": t * H * 2,
                    "d2h_bytes_per_step": t * H * 2},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
            "sweep": sweep,
            "peaks": {"kind": peak_kind, "hbm_gbs": peaks["hbm_gbs"], "bf16_tflops": peaks["bf16_tflops"]},
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_sample()
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def gateup_roofline(x, ws, sh, res, peaks, peak_kind, dev, stream) -> dict:
    """Times the gate/up GEMM launch alone (CUDA events on its stream) on the
    step's own grouped rows and reports algorithmic TFLOP/s vs the burst peak."""
    import torch

    from dispatch_b200 import _lib as L
    from dispatch_b200.kernels.grouping import _group

    t = x.shape[0]
    # the layer's own configuration: routed rows pre-gathered by the grouping kernel
    _, offsets, _, _, _, _, xs = _group(res.topk_idx, res.topk_weight, E, x=x, xs_dtype=torch.bfloat16,
                                         want_sorted=False)
    r = xs.shape[0]
    lib = L.lib()
    nbytes = lib.moe_ffn_workspace_bytes(r, I, t, I_SHARED)
    wsb = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    y = torch.empty(r, H, dtype=torch.bfloat16, device=dev)
    ys = torch.empty(t, H, dtype=torch.bfloat16, device=dev)

    def part(p):
        rc = lib.moe_expert_ffn_grouped(
            p, xs.data_ptr(), L.DT_BF16, r, H, offsets.data_ptr(), E, E, None, 0, I, ws.gate.data_ptr(),
            ws.up.data_ptr(), ws.down.data_ptr(), L.DT_BF16, None, None, None, 0, x.data_ptr(), t, I_SHARED,
            sh.gate.data_ptr(), sh.up.data_ptr(), sh.down.data_ptr(), y.data_ptr(), ys.data_ptr(), wsb.data_ptr(),
            nbytes, L.status_word(dev).data_ptr(), stream.cuda_stream)
        L.check(rc, "moe_expert_ffn_grouped")

    n = 50
    ms1 = time_loop(lambda: part(1), n, 5, 1, stream)
    ms2 = time_loop(lambda: part(2), n, 5, 1, stream)
    f1 = gateup_flops(r, t)
    achieved = f1 / (ms1 * 1e-3) / 1e12
    f2 = 2.0 * r * I * H + 2.0 * t * I_SHARED * H
    return {"kernel": "grouped_gemm_kernel<bf16> gate/up + SwiGLU (routed + shared)", "bound": "tensor",
            "achieved": round(achieved, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
            "frac": round(achieved / peaks["bf16_tflops"], 4), "peak_kind": f"{peak_kind} burst",
            "launch_ms": round(ms1, 4), "flops_per_launch": f1, "traffic": None,
            "down_gemm": {"launch_ms": round(ms2, 4), "achieved": round(f2 / (ms2 * 1e-3) / 1e12, 1)}}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--routing", choices=["uniform", "zipf"], default="uniform")
    ap.add_argument("--ref-tokens", type=int, default=64)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
