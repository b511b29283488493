"""Single-kernel cases for profiling (ncu) on the model's real shapes, with seeded random operands.

    python -m so101_smolvla_edge_b200.profile_cases mlp            # so101_mlp: expert SwiGLU block, 50 rows
    python -m so101_smolvla_edge_b200.profile_cases attention_o    # so101_attention_o: expert self layer
    python -m so101_smolvla_edge_b200.profile_cases fc2            # vision fc2 + residual, 3072 rows

Each case launches its kernel (after the producer of its inputs, as in the engine) `--reps` times
and synchronizes, so `ncu -k regex:<kernel> -s 2 -c 1` captures a warm launch. Nothing is checked:
the kernels' parity is the tests' business.
"""

from __future__ import annotations

import argparse

import torch

from .ops import attention_o, linear, mlp, rms_stats


def _rnd(g, *shape, scale=1.0, dtype=torch.float32):
    return (torch.randn(*shape, device="cuda", generator=g) * scale).to(dtype)


def case_mlp(g, reps: int) -> None:
    e = _rnd(g, 50, 720)
    x16 = torch.empty(50, 720, device="cuda", dtype=torch.bfloat16)
    ss = torch.zeros(50, 64, device="cuda")
    w_gu, w_d = _rnd(g, 4096, 720, scale=0.03, dtype=torch.bfloat16), _rnd(g, 720, 2048, scale=0.02, dtype=torch.bfloat16)
    nw = torch.ones(720, device="cuda")
    for _ in range(reps):
        rms_stats(e, x16, ss, nw)
        mlp(x16, w_gu, w_d, e, residual=e, rms=(ss, 1, 1e-5), y16=x16, y16_scale=nw, stat_ss=ss)


def case_attention_o(g, reps: int) -> None:
    qkv = _rnd(g, 50, 1600, dtype=torch.bfloat16)
    k, v = _rnd(g, 291, 320, dtype=torch.bfloat16), _rnd(g, 291, 320, dtype=torch.bfloat16)
    cs = torch.rand(50, 32, device="cuda", generator=g)
    w_o = _rnd(g, 720, 960, scale=0.02, dtype=torch.bfloat16)
    e = _rnd(g, 50, 720)
    x16 = torch.empty(50, 720, device="cuda", dtype=torch.bfloat16)
    ss = torch.zeros(50, 64, device="cuda")
    nw = torch.ones(720, device="cuda")
    own = (qkv[:, 960:1280], qkv[:, 1280:], 241, cs, cs)
    for _ in range(reps):
        rms_stats(e, x16, ss, nw)
        attention_o(qkv[:, :960], k, v, 15, 5, w_o, e, residual=e, cos=cs, sin=cs, causal_from=241, q_offset=241,
                    own=own, y16=x16, y16_scale=nw, stat_ss=ss)  # fmt: skip


def case_fc2(g, reps: int) -> None:
    x = _rnd(g, 3072, 3072, dtype=torch.bfloat16)
    w = _rnd(g, 768, 3072, scale=0.02, dtype=torch.bfloat16)
    r = _rnd(g, 3072, 768)
    for _ in range(reps):
        linear(x, w, residual=r, out=r)


CASES = {"mlp": case_mlp, "attention_o": case_attention_o, "fc2": case_fc2}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--reps", type=int, default=4)
    args = ap.parse_args()
    g = torch.Generator(device="cuda").manual_seed(0)
    CASES[args.case](g, args.reps)
    torch.cuda.synchronize()
    print(f"{args.case}: {args.reps} launches done")


if __name__ == "__main__":
    main()
