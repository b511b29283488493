"""Sweep the B200 GEMM plans for the model's shapes: the counterpart of the reference's
`scripts/tune_gemm.py`, over this library's plans (so101_gemm_config) instead of Triton tiles.

    python -m so101_smolvla_edge_b200.tune_gemm [--shapes expert|prefix|vision|all] [--batch B]
                                                [--int8] [--top 5]

Prints, per shape, the library's pick (so101_gemm_pick) and the fastest plans of the sweep with
time, TFLOP/s (TOP/s for int8) and the effective weight bandwidth. Times are CUDA-graph replays of
20 launches, so launch overhead is out of all of them (as `do_bench_cudagraph` in the reference).
Plans that a shape cannot take are skipped. `Engine(compile="autotune")` makes the same choice
for the large GEMMs inside the engine, on the engine's own buffers.
"""

from __future__ import annotations

import argparse
import itertools

import torch

from . import _lib as L
from .ops import linear, quantize_weight

# shape set -> (rows per observation, [(name, K, N, epilogue)]); the reference's own sets
# (`scripts/tune_gemm.py` SHAPES) plus the vision tower. N is the output width (the SiLU-gate
# GEMMs read 2N weight rows).
SHAPES = {
    "expert": (50, [("qkv (self)", 720, 1600, "none"), ("q (cross)", 720, 960, "none"),
                    ("o + residual", 960, 720, "residual"), ("gate_up + silu", 720, 2048, "silu_gate"),
                    ("down + residual", 2048, 720, "residual")]),
    "prefix": (241, [("qkv", 960, 1600, "none"), ("o + residual", 960, 960, "residual"),
                     ("gate_up + silu", 960, 2560, "silu_gate"), ("down + residual", 2560, 960, "residual"),
                     ("expert k / v", 320, 320, "none")]),
    "vision": (3072, [("qkv", 768, 2304, "bias"), ("out + residual", 768, 768, "residual"),
                      ("fc1 + gelu", 768, 3072, "gelu"), ("fc2 + residual", 3072, 768, "residual")]),
}  # fmt: skip


def candidates(m: int, dual: bool, int8: bool):
    """Plans to try: weight-streaming swap tiles for few rows, token tiles otherwise."""
    out = [None]
    if m <= 256 and not int8:
        for bn, s in itertools.product((16, 32, 48, 64), (1, 2, 3, 4, 6, 8)):
            if bn >= m or bn == 64:
                out.append((1, bn, s, 0, 0))
    for bn in ((64, 128) if dual else (64, 128, 256)):
        for s in (1, 2, 4):
            out.append((0, bn, s, 0, L.GEMM_ONE_TILE_PER_CTA))
        out.append((0, bn, 1, 0, L.GEMM_PERSISTENT))
        if bn >= 128:
            out.append((0, bn, 1, 0, L.GEMM_PAIR))
    if not dual:
        out.append((0, 192, 1, 0, L.GEMM_PERSISTENT))  # 192-wide tiles (N = 720 in four)
        out.append((0, 192, 1, 0, L.GEMM_PAIR))
    return out


def time_graph(f, reps: int = 20) -> float:
    """Milliseconds per launch of f, from one CUDA-graph replay of `reps` launches."""
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            f()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def sweep(name: str, m: int, k: int, n: int, epi: str, int8: bool, top: int) -> list[tuple]:
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(0)
    dual = epi == "silu_gate"
    w_rows = 2 * n if dual else n
    wf = torch.randn(w_rows, k, device=dev, generator=gen) * 0.02
    kw = {}
    if int8:
        x = torch.randint(-128, 128, (m, k), device=dev, dtype=torch.int8, generator=gen)
        w, ws = quantize_weight(wf)
        kw.update(x_scale=0.01, w_scale=ws)
        wbytes = w_rows * k
    else:
        x = torch.randn(m, k, device=dev, generator=gen).bfloat16()
        w = wf.bfloat16()
        wbytes = 2 * w_rows * k
    if epi in ("bias", "gelu"):
        kw["bias"] = torch.randn(n, device=dev, generator=gen)
    if epi == "gelu":
        kw["gelu"] = True
    if dual:
        kw["silu_gate"] = True
    res = torch.randn(m, n, device=dev, generator=gen) if epi == "residual" else None
    if res is not None:
        kw.update(residual=res, out=res)
    flops = 2.0 * m * w_rows * k
    rows = []
    for cfg in candidates(m, dual, int8):
        try:
            linear(x, w, config=cfg, **kw)
        except (RuntimeError, ValueError):
            continue  # a plan this shape cannot take
        ms = time_graph(lambda cfg=cfg: linear(x, w, config=cfg, **kw))
        rows.append((ms, cfg, flops / ms / 1e9, wbytes / ms / 1e6))
    pick_ms = next(r for r in rows if r[1] is None)
    rows.sort(key=lambda r: r[0])
    unit = "TOP/s" if int8 else "TFLOP/s"
    print(f"\n{name}: M={m} K={k} N={n} ({epi}{', W8A8' if int8 else ''})")
    print(f"  pick                      {pick_ms[0] * 1e3:8.1f} us  {pick_ms[2]:7.0f} {unit}  {pick_ms[3]:7.0f} GB/s")
    for ms, cfg, tf, gbs in rows[:top]:
        print(f"  {str(cfg):24s}  {ms * 1e3:8.1f} us  {tf:7.0f} {unit}  {gbs:7.0f} GB/s")
    return rows


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--shapes", choices=[*SHAPES, "all"], default="all")
    ap.add_argument("--batch", type=int, default=1, help="observations: rows = batch x rows per observation")
    ap.add_argument("--int8", action="store_true", help="W8A8 operands (the vision tower's int8 build)")
    ap.add_argument("--top", type=int, default=5)
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("tune_gemm needs a CUDA device")
    for key in SHAPES if args.shapes == "all" else [args.shapes]:
        rows, shapes = SHAPES[key]
        for name, k, n, epi in shapes:
            sweep(f"{key} {name}", rows * args.batch, k, n, epi, args.int8 and key == "vision", args.top)


if __name__ == "__main__":
    main()
