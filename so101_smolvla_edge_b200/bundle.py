"""Inference bundles: read the so101-smolvla-edge bundle format, and write seeded stand-ins.

A bundle is a directory with `model.safetensors` (fused weights, `lang.emb`, `norm.*`, `repr.*`)
and `meta.json` (format 1: spec, cameras, image size, state/action dims, action representation),
as `src/so101_smolvla_edge/model/bundle.py:1-16, 303-326` defines it. Loading needs only
safetensors and torch; nothing here touches a GPU.

`seeded_weights` builds the random-weight stand-in the benchmarks and parity tests run on: every
2-D matrix N(0, 0.02), norm weights 1, biases 0, a N(0, 0.02) position table, task-token rows
N(0, 0.02) * sqrt(text_dim), state/action statistics (0, 1). Each tensor draws from its own
numpy PCG64 stream keyed by (seed, crc32(name)), so the bytes are the same on every machine and
do not depend on the order tensors are made in.
"""

from __future__ import annotations

import json
import math
import zlib
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

from .spec import ModelSpec, param_shapes

FORMAT = 1
ACTION_REPRS = ("absolute", "delta", "velocity")

# 3 cameras of 512x512, 48 task tokens, 12-dim state and action
CONFIG0 = dict(n_cams=3, image_size=512, lang_len=48)
CONFIG0_CAMERAS = [
    "observation.images.top_rgb",
    "observation.images.left_rgb",
    "observation.images.right_rgb",
]


class Bundle:
    """A loaded bundle: spec, meta dict and float32 numpy tensors by name."""

    def __init__(self, spec: ModelSpec, meta: dict, tensors: dict[str, np.ndarray]):
        self.spec = spec
        self.meta = meta
        self.tensors = tensors

    @property
    def cameras(self) -> list[str]:
        return list(self.meta["cameras"])

    def checksum(self) -> str:
        """crc32 over every tensor's bytes in name order: identifies a seeded bundle (computed
        once per Bundle; the tensors are not meant to change after loading)."""
        if getattr(self, "_checksum", None) is None:
            c = 0
            for k in sorted(self.tensors):
                c = zlib.crc32(np.ascontiguousarray(self.tensors[k], dtype=np.float32).tobytes(), c)
            self._checksum = f"{c:08x}"
        return self._checksum


def load_bundle(path: str | Path | Bundle) -> Bundle:
    """Read a bundle directory (or pass a `Bundle` through).

    Raises SystemExit on a format mismatch, KeyError on a missing parameter and ValueError on a
    shape mismatch, as the reference loader does.
    """
    if isinstance(path, Bundle):
        return path
    from safetensors.numpy import load_file

    path = Path(path)
    meta = json.loads((path / "meta.json").read_text())
    if meta.get("format") != FORMAT:
        raise SystemExit(f"{path}: bundle format {meta.get('format')}, this code reads {FORMAT}")
    spec = ModelSpec.from_dict(meta["spec"])
    raw = load_file(str(path / "model.safetensors"))
    tensors = {}
    for k, v in raw.items():
        tensors[k] = v.astype(np.float32) if v.dtype != np.float32 else v
    _check(spec, tensors)
    return Bundle(spec, meta, tensors)


def _check(spec: ModelSpec, t: dict[str, np.ndarray]) -> None:
    want = param_shapes(spec)
    missing = sorted(set(want) - set(t))
    if missing:
        raise KeyError(f"bundle is missing {missing[:5]}")
    for k, (shape, _) in want.items():
        if tuple(t[k].shape) != tuple(shape):
            raise ValueError(f"{k}: bundle shape {tuple(t[k].shape)}, expected {shape}")
    for k in ("lang.emb", "norm.state.mean", "norm.state.std", "norm.action.mean",
              "norm.action.std"):  # fmt: skip
        if k not in t:
            raise KeyError(f"bundle is missing {k}")


def _rng(seed: int, name: str) -> np.random.Generator:
    return np.random.default_rng([seed, zlib.crc32(name.encode())])


def seeded_weights(
    spec: ModelSpec,
    seed: int = 0,
    state_dim: int = 12,
    action_dim: int = 12,
    std: float = 0.02,
    style: str = "baseline",
) -> dict[str, np.ndarray]:
    """Random float32 weights for `spec`.

    style "baseline" is the benchmark stand-in (matrices N(0, std), norms 1, biases 0). style
    "test" perturbs everything the baseline leaves constant, for parity tests that must see every
    operand: norm weights 1 + 0.1 N, biases and vectors 0.1 N, matrices N / sqrt(fan_in), the
    statistics of the reference's own test fixture (`tests/conftest.py:76-96`).
    """
    shapes = param_shapes(spec)
    norm_leaf = ("ln_in", "ln_post", "norm")
    norm_suffix = ("ln1.w", "ln2.w", "post_ln.w")

    def make(name: str, shape: tuple[int, ...]) -> np.ndarray:
        r = _rng(seed, name)
        is_norm = name.split(".")[-1] in norm_leaf or name.endswith(norm_suffix)
        if style == "baseline":
            if is_norm:
                return np.ones(shape, np.float32)
            if name == "vis.pos" or len(shape) == 2:
                return r.standard_normal(shape, dtype=np.float32) * np.float32(std)
            return np.zeros(shape, np.float32)
        if is_norm:
            return (1 + 0.1 * r.standard_normal(shape, dtype=np.float32)).astype(np.float32)
        if len(shape) == 2:
            return r.standard_normal(shape, dtype=np.float32) * np.float32(shape[1] ** -0.5)
        return (0.1 * r.standard_normal(shape, dtype=np.float32)).astype(np.float32)

    with ThreadPoolExecutor(8) as ex:
        futs = {k: ex.submit(make, k, shape) for k, (shape, _) in shapes.items()}
        out = {k: f.result() for k, f in futs.items()}
    r = _rng(seed, "lang.emb")
    lang = r.standard_normal((spec.lang_len, spec.text_dim), dtype=np.float32)
    scale = std * math.sqrt(spec.text_dim) if style == "baseline" else 2.0
    out["lang.emb"] = (lang * np.float32(scale)).astype(np.float32)
    if style == "baseline":
        out["repr.mean"] = np.zeros(spec.max_action, np.float32)
        out["repr.std"] = np.ones(spec.max_action, np.float32)
        for k, n in (("state", state_dim), ("action", action_dim)):
            out[f"norm.{k}.mean"] = np.zeros(n, np.float32)
            out[f"norm.{k}.std"] = np.ones(n, np.float32)
    else:
        r = _rng(seed, "stats")
        out["repr.mean"] = (0.1 * r.standard_normal(spec.max_action)).astype(np.float32)
        out["repr.std"] = (0.5 + r.random(spec.max_action)).astype(np.float32)
        for k, n in (("state", state_dim), ("action", action_dim)):
            out[f"norm.{k}.mean"] = (0.2 * r.standard_normal(n)).astype(np.float32)
            out[f"norm.{k}.std"] = (0.5 + r.random(n)).astype(np.float32)
    return out


def seeded_bundle(
    spec: ModelSpec | None = None,
    seed: int = 0,
    action_repr: str = "absolute",
    cameras: list[str] | None = None,
    image_hw: tuple[int, int] | None = None,
    state_dim: int = 12,
    action_dim: int = 12,
    style: str = "baseline",
) -> Bundle:
    """An in-memory seeded bundle; defaults are BASELINE configs[0]."""
    spec = spec or ModelSpec(**CONFIG0)
    if action_repr not in ACTION_REPRS:
        raise ValueError(f"action_repr must be one of {ACTION_REPRS}")
    cams = cameras or (CONFIG0_CAMERAS[: spec.n_cams] if spec.n_cams <= 3 else
                       [f"observation.images.cam{i}" for i in range(spec.n_cams)])  # fmt: skip
    if len(cams) != spec.n_cams:
        raise ValueError("one camera name per camera")
    hw = list(image_hw or (spec.image_size, spec.image_size))
    tensors = seeded_weights(spec, seed, state_dim, action_dim, style=style)
    meta = {
        "format": FORMAT,
        "action_repr": action_repr,
        "task": "seeded stand-in",
        "task_token_ids": [],
        "cameras": cams,
        "image_hw": hw,
        "state_dim": state_dim,
        "action_dim": action_dim,
        "joints": [f"j{i}" for i in range(action_dim)],
        "spec": spec.to_dict(),
        "seed": seed,
        "style": style,
    }
    return Bundle(spec, meta, tensors)


def write_bundle(b: Bundle, out: str | Path) -> Path:
    """Write `b` as a bundle directory (model.safetensors + meta.json)."""
    from safetensors.numpy import save_file

    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    save_file({k: np.ascontiguousarray(v) for k, v in b.tensors.items()},
              str(out / "model.safetensors"))  # fmt: skip
    (out / "meta.json").write_text(json.dumps(b.meta, indent=1))
    return out


def observation(b: Bundle, seed: int) -> tuple[dict[str, np.ndarray], np.ndarray, np.ndarray]:
    """Seeded (images, state, noise) for bundle `b`: uint8 frames U{0..255}, state N(0, 1),
    noise (chunk, max_action) N(0, 1), all from `np.random.default_rng(seed)`."""
    s = b.spec
    rng = np.random.default_rng(seed)
    h, w = b.meta["image_hw"]
    images = {c: rng.integers(0, 256, (h, w, 3), dtype=np.uint8) for c in b.cameras}
    state = rng.standard_normal(b.meta["state_dim"]).astype(np.float32)
    noise = rng.standard_normal((s.chunk, s.max_action)).astype(np.float32)
    return images, state, noise
