"""MoE-layer throughput on B200: `python bench.py --gpus N --steps K --warmup W`.

Default workload (and config 4 at N > 1):
DeepSeek-V2-Lite-shaped MoE layer, hidden 2048, 64 routed experts top-6
(softmax router), intermediate 1408 with SwiGLU, 2 always-on shared experts
(intermediate 2816), bf16, T = 4096 tokens per GPU (the prefill point),
x ~ N(0,1), weights ~ N(0,0.02), seed 0. One step = one full layer forward
(router -> grouping + gather -> expert FFN -> combine) through the public API.
The weights (1.1 GB) exceed the 126 MB L2, so no flush is needed between
steps. At N > 1 the experts are sharded evenly across ranks (expert parallel),
each rank holding its own T tokens; rows move by NVLink stores into the
owners' buffers (`--ep-transport peer`, the default) or by NCCL all-to-all
(`--ep-transport nccl`). Before anything is timed, the step's output is
checked on a sample of tokens against an f32 computation of the same layer
with the reference's own bar; a step that disagrees is refused, not timed.

Other configs: `--config c3` (config 3: routed experts int8 weight-only with
bf16 per-channel scales, shared expert bf16; reports the weight footprint),
`--config c5` (config 5: DeepSeek-V3-shaped, hidden 7168, 256 experts top-8
with the sigmoid group-limited router (8 groups, top-4 groups), intermediate
2048, 1 shared expert, int8 routed experts, T = 8192 per GPU).

`--impl reference` times the reference's own CPU path on a bounded sample of
the same workload (CPU_SAMPLE_TOKENS tokens) with all host threads: its
ReferenceMoE.forward (config 2) or its int8 grouped_moe_routed_quantized with
torch_grouped_matmul_dequant (config 3), imported from the offline install of
the reference under baseline/_ref; where that install is absent, the numpy
restatement of the same algorithm (oracle/). The B200 line's `cpu_baseline`
is the same measurement.
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
from dataclasses import dataclass
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer tokens/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


@dataclass(frozen=True)
class Workload:
    name: str
    desc: str
    H: int
    E: int
    k: int
    I: int
    I_s: int
    tokens: int
    router: str = "softmax"
    renorm: bool = False
    n_group: int = 1
    topk_group: int = 1
    scaling: float = 1.0
    int8: bool = False

    def flops(self, t: int) -> float:
        """2*T*k*3*H*I + 2*T*3*H*I_s + 2*T*H*E (router)."""
        return 2.0 * t * self.k * 3 * self.H * self.I + 2.0 * t * 3 * self.H * self.I_s + 2.0 * t * self.H * self.E

    def gateup_flops(self, rows: int, t_shared: int) -> float:
        return 2.0 * rows * self.H * 2 * self.I + 2.0 * t_shared * self.H * 2 * self.I_s

    def down_flops(self, rows: int, t_shared: int) -> float:
        return 2.0 * rows * self.I * self.H + 2.0 * t_shared * self.I_s * self.H

    def bytes(self, counts, t: int) -> int:
        """Active routed weights (+ bf16 scales) + shared + router + x in + out."""
        active = sum(1 for c in counts if c > 0)
        wb, sb = (1, 2) if self.int8 else (2, 0)
        return (active * 3 * self.H * self.I * wb + active * (2 * self.I + self.H) * sb
                + 3 * self.H * self.I_s * 2 + self.E * self.H * 2 + 2 * t * self.H * 2)


WORKLOADS = {
    "c2": Workload("c2", "C2 DeepSeek-V2-Lite MoE layer (H2048 E64 top6 I1408 + 2 shared), bf16", 2048, 64, 6,
                   1408, 2816, 4096),
    "c3": Workload("c3", "C3 DeepSeek-V2-Lite MoE layer, routed experts int8 (bf16 scales), shared bf16", 2048, 64,
                   6, 1408, 2816, 4096, int8=True),
    "c5": Workload("c5", "C5 DeepSeek-V3 MoE layer (H7168 E256 top8, sigmoid 8 groups / top-4, I2048 + 1 shared), "
                   "routed int8", 7168, 256, 8, 2048, 2048, 8192, router="sigmoid_group", renorm=True, n_group=8,
                   topk_group=4, scaling=2.5, int8=True),
}


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return PEAKS_FALLBACK, "fallback"


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


# ---------------------------------------------------------------- CPU arms
# Tokens per CPU forward, for the reference arm and the B200 line's cpu_baseline alike.
CPU_SAMPLE_TOKENS = 128


def oracle_weights(wl: Workload, rng):
    """f32 weights for the oracle (int8 configs: quantised and dequantised)."""
    import numpy as np

    from oracle import moe_oracle as O

    def f32(*s):
        w = rng.standard_normal(s, dtype=np.float32) * np.float32(0.02)
        if wl.int8 and len(s) == 3:
            q, sc = O.quantize_per_channel_int8(w)
            w = O.dequantize_int8(q, O.round_to_bf16(sc))
        return w

    gate, up, down = f32(wl.E, wl.I, wl.H), f32(wl.E, wl.I, wl.H), f32(wl.E, wl.H, wl.I)
    router = f32(wl.E, wl.H)
    shared = (f32(wl.I_s, wl.H), f32(wl.I_s, wl.H), f32(wl.H, wl.I_s))
    return router, gate, up, down, shared


def import_reference_kernels():
    """The reference's own kernel modules (its offline install under
    baseline/_ref when it is not on sys.path), or None."""
    try:
        from dispatch.kernels import moe_forward, quantization, reference_moe  # noqa: PLC0415
    except ImportError:
        ref = ROOT / "baseline" / "_ref"
        if not (ref / "dispatch").is_dir():
            return None
        sys.path.insert(0, str(ref))
        try:
            from dispatch.kernels import moe_forward, quantization, reference_moe  # noqa: PLC0415
        except ImportError:
            return None
    return reference_moe, moe_forward, quantization


def cpu_layer(wl: Workload, t_sample: int):
    """A zero-argument CPU forward of the workload on t_sample tokens, its
    kind ("reference": the reference's own code; "port": the numpy oracle)
    and a description. Weights ~N(0, 0.02), x ~N(0, 1), seed 0."""
    mods = import_reference_kernels()
    if mods is not None and wl.router == "softmax":
        import torch

        reference_moe, moe_forward, quantization = mods
        cfg = reference_moe.MoEConfig(hidden_size=wl.H, moe_intermediate_size=wl.I, n_routed_experts=wl.E,
                                      n_shared_experts=wl.I_s // wl.I, num_experts_per_tok=wl.k)
        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            m = reference_moe.ReferenceMoE(cfg).eval()
        finally:
            torch.set_default_dtype(prev)
        g = torch.Generator().manual_seed(0)
        with torch.no_grad():
            for prm in m.parameters():
                prm.copy_(torch.randn(prm.shape, generator=g) * 0.02)
        x = torch.randn(t_sample, wl.H, generator=g).to(torch.bfloat16)
        if not wl.int8:
            def fn():
                with torch.no_grad():
                    return m(x)

            return fn, "reference", "ReferenceMoE.forward in bf16 (src/dispatch/kernels/reference_moe.py:74-78)"
        q = quantization.quantize_stacked_weights(moe_forward.stack_expert_weights(m.experts))

        def fn():
            with torch.no_grad():
                idx, w = m.route(x)
                out = quantization.grouped_moe_routed_quantized(x, idx, w, q, quantization.torch_grouped_matmul_dequant)
                return out + m.shared_experts(x)

        return fn, "reference", ("ReferenceMoE.route + grouped_moe_routed_quantized(torch_grouped_matmul_dequant) "
                                 "+ shared ExpertMLP in bf16 (src/dispatch/kernels/quantization.py:81-107)")
    import numpy as np

    from oracle import moe_oracle as O

    rng = np.random.default_rng(0)
    router, gate, up, down, shared = oracle_weights(wl, rng)
    x = rng.standard_normal((t_sample, wl.H), dtype=np.float32)

    def fn():
        return O.moe_forward(x, router, gate, up, down, wl.k, shared=shared, renormalize=wl.renorm)

    return fn, "port", "numpy restatement of the reference forward (oracle/moe_oracle.py), f32"


def cpu_sample(wl: Workload, t_sample: int, seconds: float, min_reps: int):
    """Mean seconds per CPU forward on t_sample tokens with all host threads."""
    import torch
    from threadpoolctl import threadpool_limits

    cores = os.cpu_count() or 1
    fn, kind, desc = cpu_layer(wl, t_sample)
    torch.set_num_threads(cores)
    times = []
    with threadpool_limits(limits=cores):
        fn()
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < seconds or len(times) < min_reps:
            s = time.perf_counter()
            fn()
            times.append(time.perf_counter() - s)
    return statistics.mean(times), len(times), cores, kind, desc


def run_reference(args, wl: Workload) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if wl.name == "c5":
        print(json.dumps({"impl": "reference", "unavailable": "the reference has no DeepSeek-V3 (sigmoid group) "
                          "router, and the f32 CPU restatement of config 5 needs ~45 GB of host memory"}),
              flush=True)
        return
    t_sample = CPU_SAMPLE_TOKENS
    sec, reps, cores, kind, desc = cpu_sample(wl, t_sample, 0.0, args.warmup + args.steps)
    value = t_sample / sec
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if kind == "reference" else "f32",
        "data": "synthetic",
        "config": {"workload": f"{wl.desc}; {t_sample}-token sample of the T={wl.tokens} step",
                   "tokens_per_gpu": wl.tokens, "sample_tokens": t_sample, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind,
                         "sample": f"{reps} forwards of {t_sample} tokens: {desc}"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_sample(wl: Workload, seconds: float = 12.0) -> dict:
    """The reference arm's measurement, rank 0 / N=1 only."""
    if wl.name == "c5":
        return {"value": None, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                "sample": "skipped: no reference router for config 5, and its f32 restatement needs ~45 GB"}
    t_sample = CPU_SAMPLE_TOKENS
    sec, reps, cores, kind, desc = cpu_sample(wl, t_sample, seconds, 2)
    return {"value": t_sample / sec, "unit": "tokens/s", "cores": cores, "kind": kind,
            "sample": f"{reps} forwards of {t_sample} tokens: {desc}"}


# ---------------------------------------------------------------- B200 arm
def make_inputs(wl: Workload, t: int, seed: int, dev):
    """Router, experts, shared expert (~N(0, 0.02), seed 0) and x (~N(0,1),
    seed `seed`). int8 configs quantise the routed experts on the device with
    bf16 per-channel scales, one chunk of experts at a time."""
    import torch

    from dispatch_b200.kernels.moe_forward import SharedExpertWeights, StackedExpertWeights
    from dispatch_b200.kernels.quantization import (
        QuantizedStackedExpertWeights,
        QuantizedTensor,
        quantize_per_channel_int8,
    )

    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*s, sc=0.02):
        return (torch.randn(*s, generator=g, device=dev) * sc).to(torch.bfloat16)

    def experts(n, kk):
        if not wl.int8:
            return rnd(wl.E, n, kk)
        qs, ss = [], []
        for e0 in range(0, wl.E, 16):
            q = quantize_per_channel_int8(rnd(min(16, wl.E - e0), n, kk), scale_dtype=torch.bfloat16)
            qs.append(q.data)
            ss.append(q.scale)
        return QuantizedTensor(torch.cat(qs), torch.cat(ss))

    router = rnd(wl.E, wl.H)
    gate, up, down = experts(wl.I, wl.H), experts(wl.I, wl.H), experts(wl.H, wl.I)
    ws = (QuantizedStackedExpertWeights if wl.int8 else StackedExpertWeights)(gate, up, down)
    sh = SharedExpertWeights(rnd(wl.I_s, wl.H), rnd(wl.I_s, wl.H), rnd(wl.H, wl.I_s))
    bias = None
    if wl.router == "sigmoid_group":
        bias = (torch.randn(wl.E, generator=g, device=dev) * 0.01).float()
    gx = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(t, wl.H, generator=gx, device=dev).to(torch.bfloat16)
    return x, router, ws, sh, bias


def weight_footprint(ws) -> int:
    from dispatch_b200.kernels.quantization import QuantizedStackedExpertWeights

    if isinstance(ws, QuantizedStackedExpertWeights):
        return sum(q.data.numel() * q.data.element_size() + q.scale.numel() * q.scale.element_size()
                   for q in (ws.gate, ws.up, ws.down))
    return sum(w.numel() * w.element_size() for w in (ws.gate, ws.up, ws.down))


def check_layer_output(x, out, router, ws, sh, cfg, bias, n_rows: int = 64) -> dict:
    """Refuse-to-time gate (the reference's run_kernel_bench.py:90,169-175 and
    run_engine_race.py refuse a backend that disagrees with the reference):
    n_rows tokens spread over the batch are recomputed in f32 on the GPU from
    the same routing (router ids and weights are batch-invariant) and the
    layer's output rows must pass the reference's assert_matches_reference
    bar (rtol 1.6e-2, atol 1.6e-2 * max|ref|) and, for bf16 experts, also
    rtol 2e-2 / atol 1e-2. Raises AssertionError otherwise."""
    import torch

    from dispatch_b200.kernels.layer import route
    from dispatch_b200.kernels.quantization import QuantizedStackedExpertWeights

    t = x.shape[0]
    rows = torch.linspace(0, t - 1, min(n_rows, t), device=x.device).round().long().unique()
    idx, w = route(x, router, cfg, e_score_bias=bias)
    idx, w = idx[rows].long(), w[rows]
    xf = x[rows].float()
    quant = isinstance(ws, QuantizedStackedExpertWeights)

    def mat(m, e):
        return m.data[e].float() * m.scale[e].float()[:, None] if quant else m[e].float()

    ref = torch.zeros(rows.numel(), x.shape[1], device=x.device)
    for e in torch.unique(idx).tolist():
        r, sl = (idx == e).nonzero(as_tuple=True)
        hh = torch.nn.functional.silu(xf[r] @ mat(ws.gate, e).T) * (xf[r] @ mat(ws.up, e).T)
        ref.index_add_(0, r, (hh @ mat(ws.down, e).T) * w[r, sl, None])
    if sh is not None:
        sg, su, sd = (m.float() for m in (sh.gate, sh.up, sh.down))
        ref += (torch.nn.functional.silu(xf @ sg.T) * (xf @ su.T)) @ sd.T
    got = out[rows].float()
    torch.testing.assert_close(got, ref, rtol=1.6e-2, atol=1.6e-2 * float(ref.abs().max()))
    bar = "assert_matches_reference (rtol 1.6e-2, atol 1.6e-2*max) vs f32 on the dequantised int8 weights"
    if not quant:  # bf16 layers also meet the north-star bf16 bar; int8 ones the reference int8 bar only
        torch.testing.assert_close(got, ref, rtol=2e-2, atol=1e-2)
        bar = "assert_matches_reference (rtol 1.6e-2, atol 1.6e-2*max) and rtol 2e-2/atol 1e-2 vs f32"
    return {"rows": int(rows.numel()), "max_abs_err": round(float((got - ref).abs().max()), 5), "bar": bar}


def router_id_agreement(x, router, cfg, bias) -> dict:
    """Router ids of the route kernels (tensor-core f32 logits, fused
    selection) against a float64 torch selection from float64 logits on the
    same tokens: the fraction of (token, slot) ids in the float64 top-k set,
    and of tokens whose whole top-k set matches. Ids can only differ where two
    experts' scores tie to within the f32 logits' rounding."""
    import torch

    from dispatch_b200.kernels.layer import route

    idx, _ = route(x, router, cfg, e_score_bias=bias)
    lg = x.double() @ router.double().T
    b = 0.0 if bias is None else bias.double()
    if cfg.mode == "softmax":
        s = lg + b
    else:  # group-limited sigmoid: select on sigmoid + bias within the best groups
        s = torch.sigmoid(lg) + b
        t, e = s.shape
        per = e // cfg.n_group
        gsc = s.view(t, cfg.n_group, per).topk(2, dim=-1).values.sum(-1)
        keep = torch.zeros_like(gsc, dtype=torch.bool).scatter_(1, gsc.topk(cfg.topk_group, dim=-1).indices, True)
        s = s.masked_fill(~keep.repeat_interleave(per, 1), float("-inf"))
    ref = s.topk(cfg.top_k, dim=-1).indices
    got = idx.long()
    hits = (got[:, :, None] == ref[:, None, :]).any(-1)
    return {"tokens": int(got.shape[0]), "slot_agreement": round(float(hits.float().mean()), 6),
            "token_set_agreement": round(float(hits.all(-1).float().mean()), 6),
            "vs": "float64 torch selection from float64 logits"}


def time_loop(fn, steps: int, warmup: int, world: int, stream, per_step: list | None = None) -> float:
    """Mean device time of one step (ms) over `steps` timed calls after
    `warmup` untimed ones, CUDA events on `stream`, barriers on both sides.
    If `per_step` is a list, each step's own duration (ms) is appended to it
    (an event between consecutive steps; the total is unchanged)."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1 if per_step is not None else 2)]
    marks[0].record(stream)
    for i in range(steps):
        fn()
        if per_step is not None:
            marks[i + 1].record(stream)
    marks[-1].record(stream)
    torch.cuda.synchronize()
    barrier(world)
    if per_step is not None:
        per_step.extend(marks[i].elapsed_time(marks[i + 1]) for i in range(steps))
    return marks[0].elapsed_time(marks[-1]) / steps


def step_stats(per_step: list, world: int) -> dict:
    """Median and 99th percentile of the per-step times (ms), max over ranks."""
    import statistics

    v = sorted(per_step)
    med = statistics.median(v)
    p99 = v[min(len(v) - 1, int(round(0.99 * (len(v) - 1))))]
    return {"median_ms": round(max_over_ranks(med, world), 4), "p99_ms": round(max_over_ranks(p99, world), 4),
            "steps": len(v)}


def host_copy_ceiling(x_host, out_host, dev, world: int, n: int = 20) -> float:
    """The host link's ceiling for the e2e number: one step's input copy
    (host -> device) and output copy (device -> host) from the same pinned
    buffers, on the copy streams run_host_batches uses, with every rank
    copying at once; returns steps/s (max time over ranks)."""
    import torch

    xd = torch.empty(x_host.shape, dtype=x_host.dtype, device=dev)
    od = torch.zeros(out_host.shape, dtype=out_host.dtype, device=dev)
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier(world)
    cur = torch.cuda.current_stream(dev)
    start.record(cur)
    h2d.wait_stream(cur)
    d2h.wait_stream(cur)
    for _ in range(n):
        with torch.cuda.stream(h2d):
            xd.copy_(x_host, non_blocking=True)
        with torch.cuda.stream(d2h):
            out_host.copy_(od, non_blocking=True)
    cur.wait_stream(h2d)
    cur.wait_stream(d2h)
    end.record(cur)
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end) / n, world)
    barrier(world)
    return 1e3 / ms


def run_b200(args, wl: Workload) -> None:
    import torch

    from dispatch_b200 import _lib as L
    from dispatch_b200.kernels.layer import CapturedLayer, RouterConfig, moe_layer_forward, run_host_batches

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    peaks, peak_kind = load_peaks()
    t = args.tokens or wl.tokens
    x, router, ws, sh, bias = make_inputs(wl, t, seed=rank * 1000, dev=dev)
    cfg = RouterConfig(top_k=wl.k, mode=wl.router, renormalize=wl.renorm, n_group=wl.n_group,
                       topk_group=wl.topk_group, routed_scaling_factor=wl.scaling)
    if args.routing == "zipf":
        if wl.router != "softmax":
            raise SystemExit("--routing zipf applies to the softmax-router configs")
        bias = (-1.2 * torch.log(torch.arange(wl.E, dtype=torch.float32, device=dev) + 1.0))

    ep = None
    if args.profile_ep_sim:
        # profiler driver for the EP kernels on one GPU: W ranks emulated as
        # buffers on this device (dispatch, FFN with return stores, combine)
        if world > 1:
            raise SystemExit("--profile-ep-sim runs on one GPU")
        from dispatch_b200.kernels.ep_sim import simulated_ep_forward

        xs = [x] + [torch.randn(t, wl.H, generator=torch.Generator(device=dev).manual_seed(1000 * r), device=dev)
                    .to(torch.bfloat16) for r in range(1, args.profile_ep_sim)]
        for _ in range(max(args.profile_calls, 1)):
            simulated_ep_forward(xs, router, ws, sh, cfg, bias, check_offsets=False)
        torch.cuda.synchronize()
        L.check_device_status(dev)
        print(f"profile-ep-sim ok: {args.profile_ep_sim} ranks x {wl.name} T={t}", flush=True)
        return
    if args.profile_calls:
        # profiler driver: the bare layer call, no timing and no JSON line
        if world > 1:
            raise SystemExit("--profile-calls runs on one GPU (profile one process, never a multi-rank job)")
        for _ in range(args.profile_calls):
            moe_layer_forward(x, router, ws, cfg, shared=sh, e_score_bias=bias)
        torch.cuda.synchronize()
        L.check_device_status(dev)
        print(f"profile-calls ok: {args.profile_calls} x {wl.name} T={t}", flush=True)
        return

    if world > 1:
        if args.ep_transport == "peer":
            from dispatch_b200.kernels.ep_peer import PeerEPLayer

            ep = PeerEPLayer(router, ws, sh, cfg, rank=rank, world=world, e_score_bias=bias, max_tokens=t)
        else:
            from dispatch_b200.kernels.expert_parallel import EPLayer

            ep = EPLayer(router, ws, sh, cfg, rank=rank, world=world, e_score_bias=bias)

        def layer(xx):
            return ep(xx)

        launches_per_step = ep.launches_for(t) if hasattr(ep, "launches_for") else ep.launches_per_step
        parallelism = f"ep{world} ({args.ep_transport})"
    else:
        def layer(xx):
            return moe_layer_forward(xx, router, ws, cfg, shared=sh, e_score_bias=bias).out

        launches_per_step = 7  # router GEMM + select, group x2, gate/up GEMM, down GEMM, combine
        parallelism = "single"

    res = moe_layer_forward(x, router, ws, cfg, shared=sh, e_score_bias=bias)
    torch.cuda.synchronize()
    L.check_device_status(dev)
    # refuse to time a step whose output disagrees with the f32 reference
    try:
        checked = check_layer_output(x, layer(x), router, ws, sh, cfg, bias)
        torch.cuda.synchronize()
        L.check_device_status(dev)
        ok = 1.0
    except AssertionError as exc:
        checked, ok = {"refused": str(exc).splitlines()[0][:300]}, 0.0
    if max_over_ranks(-ok, world) > -1.0:  # some rank failed the check
        if rank == 0:
            print(json.dumps({"metric": METRIC, "refused": True, "checked": checked}), flush=True)
        if world > 1:
            import torch.distributed as dist

            if hasattr(ep, "close"):
                ep.close()
            dist.destroy_process_group()
        raise SystemExit(1)

    router_ids = router_id_agreement(x, router, cfg, bias)
    torch.cuda.synchronize()

    with ClockSampler(local) as clocks:
        per_step: list = []
        ms = time_loop(lambda: layer(x), args.steps, args.warmup, world, stream, per_step)
    ms = max_over_ranks(ms, world)
    step_dist = step_stats(per_step, world)
    L.check_device_status(dev)
    value = t * world / (ms * 1e-3)

    # e2e: the public host-batch call (run_host_batches) on pinned host buffers;
    # every step's host->device input copy and device->host output copy are in
    # the timed region, on copy streams that overlap the neighbouring steps
    x_host = x.cpu().pin_memory()
    out_host = torch.empty(t, wl.H, dtype=torch.bfloat16).pin_memory()
    # enough batches that filling and draining the copy pipeline stays under ~2% of the run
    n_e2e = max(4 * args.steps, 50)
    e2e_ms = max_over_ranks(
        time_loop(lambda: run_host_batches(layer, [x_host] * n_e2e, [out_host] * n_e2e), 1, 1, world, stream),
        world) / n_e2e
    e2e_val = t * world / (e2e_ms * 1e-3)
    copy_steps_per_s = host_copy_ceiling(x_host, out_host, dev, world)

    # expert-parallel phase split: CUDA events between the phases of a call,
    # mean over calls, max over ranks (names the limiter of the N-GPU step)
    ep_phases = None
    if ep is not None and hasattr(ep, "PHASES"):
        n_ph = 20
        ep.phase_events = []
        for _ in range(n_ph):
            layer(x)
        torch.cuda.synchronize()
        evs, ep.phase_events = ep.phase_events, None
        per_call = len(ep.PHASES) + 1
        dur = torch.zeros(len(ep.PHASES), dtype=torch.float64)
        for c in range(n_ph):
            marks = evs[c * per_call:(c + 1) * per_call]
            for i in range(1, per_call):
                dur[i - 1] += marks[i - 1][1].elapsed_time(marks[i][1]) / n_ph
        if world > 1:
            import torch.distributed as dist

            dd = dur.to(dev)
            dist.all_reduce(dd, op=dist.ReduceOp.MAX)
            dur = dd.cpu()
        ep_phases = {name: round(float(v), 4) for name, v in zip(ep.PHASES, dur)}

    # dominant kernel: the gate/up tcgen05 GEMM (+SwiGLU epilogue), timed alone
    roof = gateup_roofline(wl, x, ws, sh, res, peaks, peak_kind, dev, stream)

    sweep = {}
    if world == 1 and not args.no_sweep:
        for tt in (1, 16, 128, 1024):
            if tt >= t:
                continue
            xs_ = x[:tt].contiguous()
            r = moe_layer_forward(xs_, router, ws, cfg, shared=sh, e_score_bias=bias)
            torch.cuda.synchronize()
            c = r.group_sizes.cpu().tolist()
            m = time_loop(lambda: moe_layer_forward(xs_, router, ws, cfg, shared=sh, e_score_bias=bias),
                          200, 10, 1, stream)
            b = wl.bytes(c, tt)
            # the same step captured in a CUDA graph: device time without the host's launch work
            cap = CapturedLayer(xs_, router, ws, cfg, shared=sh, e_score_bias=bias)
            mg = time_loop(cap.replay, 200, 10, 1, stream)
            sweep[str(tt)] = {"ms": round(m, 4), "tokens_per_s": round(tt / (m * 1e-3), 1),
                              "hbm_gbs_algorithmic": round(b / (m * 1e-3) / 1e9, 1),
                              "hbm_frac": round(b / (m * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                              "graph_ms": round(mg, 4), "graph_tokens_per_s": round(tt / (mg * 1e-3), 1),
                              "graph_hbm_frac": round(b / (mg * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)}
            del cap
        sweep[str(t)] = {"ms": round(ms, 4), "tokens_per_s": round(value, 1),
                         "tflops_algorithmic": round(wl.flops(t) / (ms * 1e-3) / 1e12, 1),
                         "tensor_frac": round(wl.flops(t) / (ms * 1e-3) / 1e12 / peaks["bf16_tflops"], 4)}

    # the same layer with int8 routed experts (C3), so one bench line also
    # measures the int8 GEMM path at the bench's token count
    int8_layer = None
    if world == 1 and not args.no_sweep and not wl.int8:
        int8_layer = int8_layer_line(t, peaks, dev, stream)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "step_ms": step_dist,
            "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if not wl.int8 else "bf16 x int8",
            "data": "synthetic",
            "config": {"workload": f"{wl.desc}, T={t} tokens/GPU, {args.routing} routing",
                       "hidden": wl.H, "experts": wl.E, "top_k": wl.k, "intermediate": wl.I,
                       "shared_intermediate": wl.I_s, "router": wl.router, "tokens_per_gpu": t,
                       "global_tokens": t * world, "routing": args.routing, "parallelism": parallelism,
                       "routed_weight_bytes": weight_footprint(ws),
                       "l2": "inputs larger than L2 (expert weights >= 1.1 GB per step)"},
            "checked": checked,
            "router_ids": router_ids,
            "layer_tflops_algorithmic": round(wl.flops(t) / (ms * 1e-3) / 1e12, 1),
            "roofline": roof,
            "e2e": {"value": round(e2e_val, 1), "unit": "tokens/s", "h2d_bytes_per_step": t * wl.H * 2,
                    "d2h_bytes_per_step": t * wl.H * 2,
                    # the copies alone, every rank at once: the host link's ceiling on e2e
                    "host_copy_ceiling": round(copy_steps_per_s * t * world, 1),
                    "host_copy_gbs_per_gpu": round(copy_steps_per_s * 2 * t * wl.H * 2 / 1e9, 1)},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks.summary(),
            "sweep": sweep,
            "int8_layer": int8_layer,
            "ep_phases_ms": ep_phases,
            "peaks": {"kind": peak_kind, "hbm_gbs": peaks["hbm_gbs"], "bf16_tflops": peaks["bf16_tflops"]},
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_sample(wl)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        if hasattr(ep, "close"):
            ep.close()
        dist.destroy_process_group()


def int8_layer_line(t: int, peaks: dict, dev, stream) -> dict:
    """C3 at T tokens (routed experts int8 with bf16 per-channel scales,
    shared expert bf16): output checked against f32 on the dequantised
    weights (refused, and not timed, if it disagrees), then the step timed as
    a CUDA graph (device time, inputs larger than L2)."""
    import torch

    from dispatch_b200.kernels.layer import CapturedLayer, RouterConfig, moe_layer_forward

    w3 = WORKLOADS["c3"]
    x, router, ws, sh, bias = make_inputs(w3, t, seed=0, dev=dev)
    cfg = RouterConfig(top_k=w3.k, mode=w3.router, renormalize=w3.renorm, n_group=w3.n_group,
                       topk_group=w3.topk_group, routed_scaling_factor=w3.scaling)
    out = moe_layer_forward(x, router, ws, cfg, shared=sh, e_score_bias=bias).out
    torch.cuda.synchronize()
    try:
        checked = check_layer_output(x, out, router, ws, sh, cfg, bias)
    except AssertionError as exc:
        return {"workload": f"{w3.desc}, T={t}", "refused": str(exc).splitlines()[0][:300]}
    cap = CapturedLayer(x, router, ws, cfg, shared=sh, e_score_bias=bias)
    ms = time_loop(cap.replay, 50, 5, 1, stream)
    del cap
    tf = w3.flops(t) / (ms * 1e-3) / 1e12
    return {"workload": f"{w3.desc}, T={t}", "graph_ms": round(ms, 4), "tokens_per_s": round(t / (ms * 1e-3), 1),
            "tflops_algorithmic": round(tf, 1), "tensor_frac": round(tf / peaks["bf16_tflops"], 4),
            "checked": checked}


# DRAM bytes (read + write) of one gate/up launch, per (workload, T, kernel),
# from ncu captures of that kernel on that step (dram__bytes_read.sum +
# dram__bytes_write.sum).
GATEUP_TRAFFIC = {
    ("c2", 4096, "grouped_gemm_kernel<bf16>"): 879.5e6 + 68.4e6,
    ("c2", 4096, "grouped_gemm_pair_kernel"): 911.25e6 + 74.97e6,
}
GATEUP_TRAFFIC_SOURCE = ("ncu capture of this kernel on this step (dram__bytes_read.sum + dram__bytes_write.sum), "
                         "profiles/; not measured in this run")


def gateup_roofline(wl: Workload, x, ws, sh, res, peaks, peak_kind, dev, stream) -> dict:
    """Times the gate/up GEMM launch alone (CUDA events on its stream) on the
    step's own grouped rows and reports algorithmic TFLOP/s vs the burst peak."""
    import torch

    from dispatch_b200 import _lib as L
    from dispatch_b200.kernels.grouping import _group
    from dispatch_b200.kernels.quantization import QuantizedStackedExpertWeights

    t = x.shape[0]
    _, offsets, _, _, _, _, xs = _group(res.topk_idx, res.topk_weight, wl.E, x=x, xs_dtype=torch.bfloat16,
                                         want_sorted=False)
    r = xs.shape[0]
    quant = isinstance(ws, QuantizedStackedExpertWeights)
    g, u, d = (ws.gate.data, ws.up.data, ws.down.data) if quant else (ws.gate, ws.up, ws.down)
    sc = (ws.gate.scale, ws.up.scale, ws.down.scale) if quant else (None, None, None)
    lib = L.lib()
    nbytes = lib.moe_ffn_workspace_bytes(r, wl.I, t, wl.I_s)
    wsb = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    y = torch.empty(r, wl.H, dtype=torch.bfloat16, device=dev)
    ys = torch.empty(t, wl.H, dtype=torch.bfloat16, device=dev)

    def part(p):
        rc = lib.moe_expert_ffn_grouped(
            p, xs.data_ptr(), L.DT_BF16, r, wl.H, offsets.data_ptr(), wl.E, wl.E, None, 0, wl.I, g.data_ptr(),
            u.data_ptr(), d.data_ptr(), L.DT_I8 if quant else L.DT_BF16, L.ptr(sc[0]), L.ptr(sc[1]), L.ptr(sc[2]),
            L.dt(sc[0]) if quant else 0, x.data_ptr(), t, wl.I_s, sh.gate.data_ptr(), sh.up.data_ptr(),
            sh.down.data_ptr(), y.data_ptr(), ys.data_ptr(), wsb.data_ptr(), nbytes,
            L.status_word(dev).data_ptr(), stream.cuda_stream)
        L.check(rc, "moe_expert_ffn_grouped")

    n = 50
    ms1 = time_loop(lambda: part(1), n, 5, 1, stream)
    ms2 = time_loop(lambda: part(2), n, 5, 1, stream)
    f1 = wl.gateup_flops(r, t)
    achieved = f1 / (ms1 * 1e-3) / 1e12
    f2 = wl.down_flops(r, t)
    # the kernel the automatic choice launches for this call
    choice = lib.moe_ffn_kernel_auto(r, wl.E, t, wl.H, wl.I, L.DT_I8 if quant else L.DT_BF16)
    kernel = {L.FFN_KERNEL_PAIR: "grouped_gemm_pair_kernel", L.FFN_KERNEL_WARP: "grouped_gemm_warp_kernel"}.get(
        choice, "grouped_gemm_kernel<int8>" if quant else "grouped_gemm_kernel<bf16>")
    traffic = GATEUP_TRAFFIC.get((wl.name, t, kernel))
    return {"kernel": kernel + " gate/up + SwiGLU (routed + shared)", "bound": "tensor",
            "achieved": round(achieved, 1), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
            "frac": round(achieved / peaks["bf16_tflops"], 4), "peak_kind": f"{peak_kind} burst",
            "launch_ms": round(ms1, 4), "flops_per_launch": f1, "traffic": traffic,
            "traffic_source": GATEUP_TRAFFIC_SOURCE if traffic else "not captured for this config and kernel",
            "down_gemm": {"launch_ms": round(ms2, 4), "achieved": round(f2 / (ms2 * 1e-3) / 1e12, 1)}}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=sorted(WORKLOADS), default="c2")
    ap.add_argument("--tokens", type=int, default=0, help="tokens per GPU (default: the config's)")
    ap.add_argument("--routing", choices=["uniform", "zipf"], default="uniform")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ep-transport", choices=["peer", "nccl"], default="peer",
                    help="N>1: NVLink peer stores fused into dispatch/FFN (peer) or NCCL all-to-all (nccl)")
    ap.add_argument("--profile-calls", type=int, default=0,
                    help="run the layer this many times and exit (a driver for ncu launch lists and captures)")
    ap.add_argument("--profile-ep-sim", type=int, default=0, metavar="W",
                    help="run the expert-parallel layer with W ranks emulated on one GPU (--profile-calls times) "
                         "and exit: a one-GPU driver for ncu captures of the EP kernels")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    wl = WORKLOADS[args.config]
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_b200(args, wl)


if __name__ == "__main__":
    main()
