"""Kernel race on one B200: this library's routed-MoE layer beside the
reference's own contestants -- its naive and persistent Triton grouped GEMMs
at every tile size of its sweep, its int8 Triton kernel, and vLLM's
fused_experts -- on the reference's seeded inputs, with the reference's own
checker and timer (the flow of the reference's scripts/run_engine_race.py:
prepare -> run -> refuse-or-time).

    python -m dispatch_b200.race --out DIR [--tokens 1,4,16,...] [--engines ...]

The reference package must be importable: it is looked up on sys.path and in
``baseline/_ref`` (an offline install of the reference next to this
repository). ``dispatch-b200`` is registered beside the reference's
``ENGINE_NAMES`` (src/dispatch/benchmark/engines/registry.py:11-32) and
``build_engines`` so the reference's registry hands it out like its own
contestants. Every (variant, case) output is checked with the reference's
``assert_matches_reference`` against ``reference_output`` (f32; the int8 race
against the same int8 weights dequantised) before it is timed; a variant that
disagrees, or cannot be prepared, is recorded as refused and not timed.
Timing is the reference's ``time_grouped_gemm`` (triton.testing.do_bench:
25 ms warm-up, 100 ms of repetitions, L2 cleared before each call), so every
contestant pays the same host-side call overhead.

Writes ``race.json`` (one record per variant and case) and ``race.md`` (a
table of mean latencies) into DIR.
"""

from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
B200_ENGINE = "dispatch-b200"


def import_reference():
    """The reference's race modules, or ImportError with the reason."""
    try:
        import dispatch  # noqa: F401, PLC0415
    except ImportError:
        ref = ROOT / "baseline" / "_ref"
        if not (ref / "dispatch").is_dir():
            raise ImportError(f"the reference package is neither importable nor installed under {ref}") from None
        sys.path.insert(0, str(ref))
    from dispatch.benchmark.engines import base, registry  # noqa: PLC0415
    from dispatch.kernels import bench, moe_forward, quantization  # noqa: PLC0415

    return base, registry, bench, moe_forward, quantization


class ReferenceTypedB200Engine:
    """The B200 layer behind the reference's MoEEngine contract, taking the
    reference's weight containers (its StackedExpertWeights and
    QuantizedStackedExpertWeights) as prepared by the race harness."""

    name = B200_ENGINE

    def prepare_bf16(self, weights):
        from dispatch_b200.engines import B200Engine  # noqa: PLC0415
        from dispatch_b200.kernels.moe_forward import StackedExpertWeights  # noqa: PLC0415

        mine = StackedExpertWeights(weights.gate, weights.up, weights.down)
        return B200Engine().prepare_bf16(mine)

    def prepare_int8(self, qweights):
        from dispatch_b200.engines import B200Engine  # noqa: PLC0415
        from dispatch_b200.kernels.quantization import (  # noqa: PLC0415
            QuantizedStackedExpertWeights,
            QuantizedTensor,
        )

        q = lambda t: QuantizedTensor(t.data, t.scale)  # noqa: E731
        mine = QuantizedStackedExpertWeights(q(qweights.gate), q(qweights.up), q(qweights.down))
        return B200Engine().prepare_int8(mine)


def register(registry) -> None:
    """Adds dispatch-b200 to the reference's engine registry (idempotent)."""
    if B200_ENGINE in registry.ENGINE_NAMES:
        return
    registry.ENGINE_NAMES = (*registry.ENGINE_NAMES, B200_ENGINE)
    stock = registry.build_engines

    def build_engines(engine: str, block_ms=registry.DEFAULT_BLOCK_MS):
        if engine == B200_ENGINE:
            return [ReferenceTypedB200Engine()]
        return stock(engine, block_ms)

    registry.build_engines = build_engines


def _first_line(exc: BaseException) -> str:
    text = str(exc).strip() or type(exc).__name__
    return text.splitlines()[0][:300]


def run(out_dir: Path, engines: list[str], tokens: list[int], distributions: list[str],
        precisions: list[str]) -> list[dict]:
    base, registry, bench, moe_forward, quantization = import_reference()
    register(registry)
    device = "cuda"
    weights = base.make_weights(torch.bfloat16, seed=0, device=device)
    qweights = quantization.quantize_stacked_weights(weights)
    oracle = {"bf16": weights, "int8": base.dequantized_weights(qweights)}
    cases = {}
    for t in tokens:
        for d in distributions:
            case = base.make_case(t, d, dtype=torch.bfloat16, seed=0, device=device)
            cases[(t, d)] = (case, {p: base.reference_output(case, oracle[p]) for p in precisions})
    results: list[dict] = []
    for name in engines:
        try:
            variants = registry.build_engines(name)
        except Exception as exc:  # an engine that cannot even be built is a refusal
            results.append({"variant": name, "precision": None, "status": "refused", "reason": _first_line(exc)})
            continue
        for engine in variants:
            for precision in precisions:
                t0 = time.time()
                try:
                    factory = engine.prepare_bf16(weights) if precision == "bf16" else engine.prepare_int8(qweights)
                except Exception as exc:
                    results.append({"variant": engine.name, "precision": precision, "status": "refused",
                                    "reason": _first_line(exc)})
                    continue
                for (t, d), (case, refs) in cases.items():
                    entry = {"variant": engine.name, "engine": name, "precision": precision, "num_tokens": t,
                             "distribution": d}
                    try:
                        bound = factory(case)
                        moe_forward.assert_matches_reference(bound(), refs[precision])
                    except Exception as exc:  # disagreement (or a crash) is recorded, never timed
                        entry.update(status="refused", reason=_first_line(exc))
                        results.append(entry)
                        continue
                    flops = 3 * bench.grouped_gemm_flops(t * base.NUM_EXPERTS_PER_TOK, base.MOE_INTERMEDIATE_SIZE,
                                                         base.HIDDEN_SIZE)
                    s = bench.time_grouped_gemm(bound, label=f"{engine.name}/{precision}/{t}/{d}", flops=flops)
                    entry.update(status="ok", mean_ms=s.mean_latency_ms, p50_ms=s.p50_latency_ms,
                                 p99_ms=s.p99_latency_ms, tflops=s.tflops)
                    results.append(entry)
                print(f"race: {engine.name} {precision} done in {time.time() - t0:.1f} s", flush=True)
    out_dir.mkdir(parents=True, exist_ok=True)
    meta = {"gpu": torch.cuda.get_device_name(), "torch": torch.__version__,
            "versions": {p: base.installed_version(p) for p in ("triton", "vllm", "sglang")},
            "tokens": tokens, "distributions": distributions, "precisions": precisions}
    (out_dir / "race.json").write_text(json.dumps({"meta": meta, "results": results}, indent=1))
    (out_dir / "race.md").write_text(render(results, tokens, distributions, precisions))
    return results


def render(results: list[dict], tokens: list[int], distributions: list[str], precisions: list[str]) -> str:
    """Mean latency (ms) per variant and case; the best reference variant per
    case beside dispatch-b200."""
    lines = []
    for precision in precisions:
        for d in distributions:
            rows = [r for r in results if r.get("precision") == precision and r.get("distribution") == d]
            variants = sorted({r["variant"] for r in rows})
            lines.append(f"\n### {precision}, {d} routing (mean ms, do_bench)\n")
            lines.append("| variant | " + " | ".join(f"T={t}" for t in tokens) + " |")
            lines.append("|---|" + "---|" * len(tokens))
            for v in variants:
                cells = []
                for t in tokens:
                    r = next((r for r in rows if r["variant"] == v and r["num_tokens"] == t), None)
                    cells.append("-" if r is None else (f"{r['mean_ms']:.4f}" if r["status"] == "ok" else "refused"))
                lines.append(f"| {v} | " + " | ".join(cells) + " |")
            best, ours = [], []
            for t in tokens:
                ok = [r for r in rows if r["num_tokens"] == t and r["status"] == "ok"]
                ref = [r["mean_ms"] for r in ok if r["variant"] != B200_ENGINE]
                mine = [r["mean_ms"] for r in ok if r["variant"] == B200_ENGINE]
                best.append(min(ref) if ref else None)
                ours.append(mine[0] if mine else None)
            lines.append("| best reference-side variant / dispatch-b200 | " + " | ".join(
                "-" if (b is None or o is None) else f"{b / o:.2f}x" for b, o in zip(best, ours)) + " |")
    refused = [r for r in results if r.get("status") == "refused"]
    if refused:
        lines.append("\nRefused (not timed):\n")
        seen = set()
        for r in refused:
            key = (r["variant"], r.get("precision"), r.get("reason"))
            if key in seen:
                continue
            seen.add(key)
            lines.append(f"- {r['variant']} ({r.get('precision')}): {r.get('reason')}")
    return "\n".join(lines) + "\n"


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--out", type=Path, required=True)
    ap.add_argument("--engines", default="dispatch-naive,dispatch-persistent,vllm,dispatch-b200")
    ap.add_argument("--tokens", default="1,4,16,64,128,512,2048")
    ap.add_argument("--distributions", default="uniform,zipf")
    ap.add_argument("--precisions", default="bf16,int8")
    a = ap.parse_args()
    split = lambda s: [v for v in s.split(",") if v]  # noqa: E731
    results = run(a.out, split(a.engines), [int(t) for t in split(a.tokens)], split(a.distributions),
                  split(a.precisions))
    print((a.out / "race.md").read_text(), flush=True)
    bad = [r for r in results if r.get("status") == "refused" and r.get("variant") == B200_ENGINE]
    if bad:
        raise SystemExit(f"dispatch-b200 refused on {len(bad)} case(s)")


if __name__ == "__main__":
    main()
