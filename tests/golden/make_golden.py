#!/usr/bin/env python3
"""Write the golden fixtures in this directory by running the reference project itself.

    python tests/golden/make_golden.py --reference PATH [--full-seeds 4] [--only WHICH]

Needs the so101-smolvla-edge sources (the `src/` of the reference checkout given by
--reference) and runs them on the CPU in float32, the way `scripts/standin_bundle.py:150` writes
its golden actions: `Engine(bundle, device="cpu", dtype="fp32", cuda_graph=False, warmup=0)`.
The bundles are this package's seeded bundles (`so101_smolvla_edge_b200.bundle`), written to a
temporary directory, so a test can rebuild the same weights anywhere from the seed; each fixture
stores the bundle's checksum to prove it.

Fixtures:
    golden_<case>.npz   small bundles (every action representation, resize + padding, biases
                        and norms perturbed): inputs, actions and every intermediate
    golden_config0.npz  BASELINE configs[0] (3 x 512^2 cameras, 241-token prefix): actions for
                        seeds 0..n-1; for seed 0 the image rows, layer-0 K/V, layer-1 kx and v_t
    golden_int8_<case>.npz  W8A8 vision: activation clips calibrated on 32 observations and the
                        actions of the reference model with its vision linears fake-quantized as
                        the reference's own int8 test does (`tests/test_ov_engine.py:222-236`);
                        for configs[0] the int8 actions of seeds 0..n-1 and seed 0's int8 image
                        rows, and the same again from three runs with the quantizers' float32
                        inputs nudged by one ulp (the reference's own int8 reproducibility band)
"""

from __future__ import annotations

import argparse
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from so101_smolvla_edge_b200.bundle import observation, seeded_bundle, write_bundle  # noqa: E402
from so101_smolvla_edge_b200.spec import ModelSpec  # noqa: E402

# small specs: "tiny" is the reference fixture's own size (head_dim 8, so CPU only); "small" has
# the widths and head sizes the CUDA kernels take and is what the GPU engine tests run
TINY = dict(n_cams=2, image_size=128, patch=16, vis_dim=32, vis_layers=2, vis_heads=4,
            vis_mlp=64, shuffle=4, text_dim=48, n_layers=4, n_heads=6, n_kv=2, head_dim=8,
            text_mlp=96, exp_dim=40, exp_mlp=64, chunk=8, max_state=8, max_action=8, n_steps=3,
            lang_len=3)  # fmt: skip
SMALL = dict(n_cams=2, image_size=128, patch=16, vis_dim=128, vis_layers=2, vis_heads=2,
             vis_mlp=256, shuffle=4, text_dim=192, n_layers=4, n_heads=6, n_kv=2, head_dim=32,
             text_mlp=256, exp_dim=96, exp_mlp=160, chunk=10, max_state=8, max_action=8,
             n_steps=3, lang_len=5)  # fmt: skip
SMALL64 = dict(SMALL, text_dim=320, n_heads=5, n_kv=1, head_dim=64, exp_dim=128, lang_len=7,
               self_attn_every=2)  # fmt: skip
CASES = {
    "tiny_absolute": (TINY, "absolute", (120, 160)),
    "small_absolute": (SMALL, "absolute", (120, 160)),
    "small_delta": (SMALL, "delta", (128, 128)),
    "small_velocity": (SMALL, "velocity", (96, 200)),
    "small64_absolute": (SMALL64, "absolute", (128, 128)),
}


def reference_engine(ref, bundle_dir):
    from so101_smolvla_edge.model.engine import Engine

    return Engine(str(bundle_dir), device="cpu", dtype="fp32", cuda_graph=False, warmup=0)


def intermediates(eng, images, state, noise) -> dict[str, np.ndarray]:
    """Run one chunk stage by stage through the reference engine and keep what each produced."""
    import torch

    s = eng.spec
    for i, c in enumerate(eng.cams):
        eng.img[i].copy_(torch.from_numpy(images[c]))
    eng.state.copy_(torch.from_numpy(state))
    eng.noise.copy_(torch.from_numpy(noise).view_as(eng.noise))
    out = {}
    with torch.no_grad():
        rows = eng._vision()
        out["img_rows"] = rows.numpy().copy()
        out["prefix_rows"] = eng._prefix_rows(rows).numpy().copy()
        eng._prefix(rows)
        L = s.prefix_len
        for i in range(s.n_layers):
            out[f"k_{i}"] = eng.k_pre[i].reshape(L, -1).numpy().copy()
            out[f"v_{i}"] = eng.v_pre[i].reshape(L, -1).numpy().copy()
            if not s.is_self_attn(i):  # (1, nq, L, hd), kv heads repeated: keep one per group
                g = s.n_heads // s.n_kv
                kx = eng.kx[i][0, ::g].transpose(0, 1).reshape(L, -1)
                vx = eng.vx[i][0, ::g].transpose(0, 1).reshape(L, -1)
                out[f"kx_{i}"] = kx.numpy().copy()
                out[f"vx_{i}"] = vx.numpy().copy()
        caches = (eng.ks, eng.vs, eng.kx, eng.vx)
        rope = (eng.cos_s, eng.sin_s, eng.cos_c, eng.sin_c)
        v0 = eng.model.velocity(eng.noise, eng.time_proj[0], *caches, eng.mask_s, *rope)
        out["v0"] = v0[0].numpy().copy()
    out["actions"] = eng.infer(images, state, noise=noise)
    return out


VISION_LINEARS = ("qkv", "out", "fc1", "fc2")


def _quantized_names(spec) -> dict[str, str]:
    names = {"conn.w": "conn"}
    names |= {f"vis.{i}.{n}.w": f"vis.{i}.{n}" for i in range(spec.vis_layers) for n in VISION_LINEARS}
    return names


def calibrate(eng, calib_obs) -> dict[str, float]:
    """The reference test's calibration hook (`tests/test_ov_engine.py:211-225`): max |x| of the
    input of every vision linear except the patch GEMM, over the calibration frames."""
    import torch

    from so101_smolvla_edge.model.smolvla import SmolVLA

    m = eng.model
    names = _quantized_names(m.spec)
    clip: dict[str, float] = {}

    def hook(self, x, w, b=None):
        if w in names:
            clip[names[w]] = max(clip.get(names[w], 0.0), float(x.abs().max()))
        return SmolVLA.lin(self, x, w, b)

    m.lin = hook.__get__(m)
    try:
        for imgs in calib_obs:
            for i, c in enumerate(eng.cams):
                eng.img[i].copy_(torch.from_numpy(imgs[c]))
            with torch.no_grad():
                eng._vision()
    finally:
        del m.lin
    return clip


class fake_quant:
    """W8A8 fake quant of the vision linears on the reference model (`tests/test_ov_engine.py:
    227-236`): inputs per tensor at the clip, weights per output channel, then a float linear."""

    def __init__(self, eng, clip, ulp_seed: int | None = None):
        self.m, self.clip, self.ulp_seed = eng.model, clip, ulp_seed

    def __enter__(self):
        import torch

        from so101_smolvla_edge.model.smolvla import SmolVLA

        names, clip = _quantized_names(self.m.spec), self.clip
        gen = None if self.ulp_seed is None else torch.Generator().manual_seed(self.ulp_seed)

        def lin(self, x, w, b=None):
            if w not in names:
                return SmolVLA.lin(self, x, w, b)
            if gen is not None:  # one float32 ulp up or down per element, before quantizing
                up = torch.rand(x.shape, generator=gen) < 0.5
                x = torch.nextafter(x, torch.where(up, torch.tensor(float("inf")), torch.tensor(float("-inf"))))
            xs = clip[names[w]] / 127.0
            xq = torch.clamp(torch.round(x / xs), -128, 127) * xs
            W = self.p(w)
            ws = (W.abs().amax(1, keepdim=True) / 127.0).clamp(min=1e-8)
            Wq = torch.clamp(torch.round(W / ws), -127, 127) * ws
            return torch.nn.functional.linear(xq, Wq, None if b is None else self.p(b))

        self.m.lin = lin.__get__(self.m)
        return self

    def __exit__(self, *exc):
        del self.m.lin


def calibrate_and_quantize(eng, calib_obs, observations, ulp_runs: int = 0) -> dict[str, np.ndarray]:
    """Clips from the calibration frames, then the fake-quantized chunk of every observation
    (and, for the first, its int8 image rows). With ulp_runs > 0, also the same chunks with every
    quantized linear's input nudged by one float32 ulp (seeds 0..ulp_runs-1): how far the
    reference's own int8 chunk moves under the smallest change of its float32 arithmetic."""

    def run(ulp_seed):
        acts, rows = [], None
        with fake_quant(eng, clip, ulp_seed):
            for k, (images, state, noise) in enumerate(observations):
                if k == 0:
                    got = intermediates(eng, images, state, noise)
                    rows = got["img_rows"]
                    acts.append(got["actions"])
                else:
                    acts.append(eng.infer(images, state, noise=noise))
        return np.stack(acts), rows

    clip = calibrate(eng, calib_obs)
    acts, rows = run(None)
    keys = sorted(clip)
    out = {"clip_names": np.array(keys), "clip_values": np.array([clip[k] for k in keys]),
           "actions_int8": acts, "s0.img_rows_int8": rows}  # fmt: skip
    if ulp_runs:
        runs = [run(u) for u in range(ulp_runs)]
        out["actions_int8_ulp"] = np.stack([a for a, _ in runs])
        out["s0.img_rows_int8_ulp"] = np.stack([r for _, r in runs])
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", required=True, help="the so101-smolvla-edge project checkout")
    ap.add_argument("--full-seeds", type=int, default=4)
    ap.add_argument("--only", choices=["small", "config0", "int8-config0"], default=None,
                    help="write one group of fixtures (default: all)")
    a = ap.parse_args()
    sys.path.insert(0, str(Path(a.reference) / "src"))
    import torch

    torch.set_num_threads(8)
    import so101_smolvla_edge as ref  # noqa: F401  (fails loudly if the reference is absent)

    with tempfile.TemporaryDirectory() as tmp:
        for case, (kw, repr_, hw) in CASES.items() if a.only in (None, "small") else ():
            b = seeded_bundle(ModelSpec(**kw), seed=7, action_repr=repr_, image_hw=hw,
                              state_dim=6, action_dim=6, style="test")  # fmt: skip
            d = write_bundle(b, Path(tmp) / case)
            eng = reference_engine(ref, d)
            rec: dict[str, np.ndarray] = {"checksum": np.array(b.checksum())}
            for seed in (0, 1):
                images, state, noise = observation(b, seed)
                got = intermediates(eng, images, state, noise)
                for k, v in got.items():
                    rec[f"s{seed}.{k}"] = v
            np.savez_compressed(HERE / f"golden_{case}.npz", **rec)
            print(f"{case}: actions {rec['s0.actions'].shape} written", flush=True)
            if case == "small_absolute":
                calib = [observation(b, 1000 + i)[0] for i in range(32)]
                q = calibrate_and_quantize(eng, calib, [observation(b, 0)])
                q["actions_int8"] = q["actions_int8"][0]
                q.pop("s0.img_rows_int8")
                q["checksum"] = np.array(b.checksum())
                q["actions_fp32"] = rec["s0.actions"]
                np.savez_compressed(HERE / f"golden_int8_{case}.npz", **q)
                print(f"{case}: int8 golden written", flush=True)

        if a.only == "small":
            return
        b = seeded_bundle()  # configs[0]
        d = write_bundle(b, Path(tmp) / "config0")
        eng = reference_engine(ref, d)
        if a.only in (None, "config0"):
            rec = {"checksum": np.array(b.checksum())}
            acts = []
            for seed in range(a.full_seeds):
                images, state, noise = observation(b, seed)
                t0 = time.perf_counter()
                if seed == 0:
                    got = intermediates(eng, images, state, noise)
                    for k in ("img_rows", "k_0", "v_0", "kx_1", "vx_1", "v0"):
                        rec[f"s0.{k}"] = got[k]
                    acts.append(got["actions"])
                else:
                    acts.append(eng.infer(images, state, noise=noise))
                print(f"config0 seed {seed}: {time.perf_counter() - t0:.1f} s", flush=True)
            rec["actions"] = np.stack(acts)
            np.savez_compressed(HERE / "golden_config0.npz", **rec)
        fp32 = np.load(HERE / "golden_config0.npz")["actions"]
        calib = [observation(b, 1000 + i)[0] for i in range(32)]
        t0 = time.perf_counter()
        q = calibrate_and_quantize(eng, calib, [observation(b, s) for s in range(fp32.shape[0])],
                                   ulp_runs=3)  # fmt: skip
        q["checksum"] = np.array(b.checksum())
        q["actions_fp32"] = fp32
        np.savez_compressed(HERE / "golden_int8_config0.npz", **q)
        print(f"config0 int8 golden ({fp32.shape[0]} seeds) in {time.perf_counter() - t0:.1f} s", flush=True)


if __name__ == "__main__":
    main()
