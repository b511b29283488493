"""The B200 inference engine: static buffers, one CUDA graph per chunk, the reference's API.

    eng = Engine("bundle/", device="cuda")        # loads, warms up, captures the graph
    chunk = eng.infer({"observation.images.top_rgb": rgb, ...}, state)   # (50, 12) rad

This is `src/so101_smolvla_edge/model/engine.py`'s `Engine` (constructor options, `infer`,
`profile`, `timing`, `kernels`, `graph`, `spec`, `step`) with its three backends — torch, Triton
(`kernels=`) and TensorRT (`vision=`) — replaced by the B200 kernels of libso101_b200.so:

    kernels   "auto" | "b200" run the prefix pass and denoising loop on the B200 kernels;
              "triton" is accepted from reference configs and means the same. "torch" has no
              counterpart here (the float32 torch path is the test oracle, not a backend).
    vision    "cuda" (and the reference's "torch" / "trt") run the vision tower on the B200
              kernels in `trt_precision` "bf16" or "int8" (W8A8, with activation clips).

    compile   "autotune" times the GEMM plans of every GEMM with many token rows (persistent or
              CTA-pair tiles, 128 or 256 wide) and keeps the fastest (`Engine.tuning` reports
              them); other values are accepted and ignored. SO101_AUTOTUNE=1 does the same.

There is no CPU fallback: without a CUDA device or without the library, construction raises.
`batch=B` sizes every buffer for B observations; `infer_batch` runs them as one graph replay.
"""

from __future__ import annotations

import json
import logging
import os
import time
import weakref
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np
import torch

from .bundle import Bundle, load_bundle
from .path import B200Path, unsupported
from .spec import vision_linear_names
from .timing import Timing

log = logging.getLogger("so101_smolvla_edge_b200.engine")

KERNELS = ("auto", "b200", "triton", "torch")
VISIONS = ("cuda", "torch", "trt")


def _resolve_kernels(kernels: str, device: torch.device, dtype: str, spec) -> str:
    """The reference's kernel choice (`pkg/model/engine.py:51-69`), with the B200 kernels as the
    only implementation: anything that cannot run them raises instead of falling back."""
    if kernels not in KERNELS:
        raise ValueError(f"kernels must be one of {KERNELS}, not {kernels!r}")
    if kernels == "torch":
        raise ValueError("kernels='torch' is not served here: this engine runs the B200 kernels only")
    if device.type != "cuda" or not torch.cuda.is_available():
        raise RuntimeError(f"kernels={kernels!r}: the B200 kernels need a CUDA device, got {device}")
    if dtype != "bf16":
        raise ValueError(f"dtype {dtype!r}: the B200 kernels compute bf16 matmuls (fp32 accumulate)")
    why = unsupported(spec)
    if why:
        raise ValueError(f"kernels={kernels!r}: {why}")
    if kernels == "triton":
        log.info("kernels=triton: served by the B200 kernels")
    return "b200"


def load_act_clip(bundle_dir: str | Path | None, act_clip) -> dict[str, float] | None:
    """Activation clips for int8 vision: a dict, a JSON path, or the bundle's trt/act_clip.json
    (the reference's default location, `pkg/cli.py:193-205`)."""
    if isinstance(act_clip, dict):
        return {k: float(v) for k, v in act_clip.items()}
    path = Path(act_clip) if act_clip else (Path(bundle_dir) / "trt" / "act_clip.json" if bundle_dir else None)
    if path is None or not path.exists():
        return None
    return {k: float(v) for k, v in json.loads(path.read_text()).items()}


class Engine:
    """SmolVLA on one B200, one call per action chunk (or per batch of B chunks)."""

    def __init__(
        self,
        bundle: str | Path | Bundle,
        device: str = "cuda",
        dtype: str = "bf16",
        residual: str = "fp32",
        cuda_graph: bool = True,
        compile: bool | str = False,
        warmup: int = 3,
        vision: str = "cuda",
        trt_precision: str = "bf16",
        kernels: str = "auto",
        batch: int = 1,
        act_clip: dict[str, float] | str | Path | None = None,
        pdl: bool | None = None,
        expert_step: str | None = None,
        fold_norms: bool = True,
    ):
        self.device = dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = self.device = torch.device("cuda", torch.cuda.current_device())
        b = load_bundle(bundle)
        self.bundle = b
        self.spec = s = b.spec
        self.meta = b.meta
        self.kernels = _resolve_kernels(kernels, dev, dtype, s)
        if residual != "fp32":
            raise ValueError("residual must be 'fp32': the B200 path keeps float32 residual streams")
        if vision not in VISIONS:
            raise ValueError(f"vision must be one of {VISIONS}, not {vision!r}")
        if trt_precision not in ("bf16", "int8"):
            raise ValueError(f"trt_precision must be 'bf16' or 'int8', not {trt_precision!r}")
        if compile and compile != "autotune":
            log.info("compile=%r ignored: the B200 path is hand-written kernels in a CUDA graph", compile)
        self.vision_precision = trt_precision
        clip = None
        if trt_precision == "int8":
            clip = load_act_clip(None if isinstance(bundle, Bundle) else bundle, act_clip)
            if not clip:
                raise SystemExit("int8 vision needs activation clips: pass act_clip or put them in "
                                 "BUNDLE/trt/act_clip.json (Engine.calibrate writes them)")  # fmt: skip
        self.act_clip = clip
        self.cams = list(b.meta["cameras"])
        self.repr = b.meta["action_repr"]
        self.state_dim, self.action_dim = b.meta["state_dim"], b.meta["action_dim"]
        self.batch = int(batch)
        from . import ops

        if pdl is None:  # programmatic dependent launch: on unless SO101_PDL=0
            pdl = os.environ.get("SO101_PDL", "1") != "0"
        self.pdl = bool(pdl)
        ops.set_pdl(self.pdl)
        torch.cuda.set_device(dev)
        if expert_step is None:  # "fused": the persistent expert-step kernel; default the per-op chain
            expert_step = os.environ.get("SO101_EXPERT_STEP", "auto")
        self.path = B200Path(b, dev, self.batch, trt_precision, clip, expert_step, fold_norms)
        self.tp = self.path  # the reference's attribute for the custom-kernel path
        p = self.path
        self.tuning = None
        if compile == "autotune" or os.environ.get("SO101_AUTOTUNE", "0") == "1":
            # the reference autotunes its prefix GEMMs here (pkg/model/engine.py:219-233); this
            # path times its own GEMM plans for every large GEMM and rebuilds with the fastest
            self.tuning = p.autotune()
        self.img, self.state, self.noise, self.out = p.img, p.state, p.noise, p.out
        self._host_img = torch.zeros(p.img.shape, dtype=torch.uint8).pin_memory()
        self._host_state = torch.zeros(p.state.shape, dtype=torch.float32).pin_memory()
        self._host_noise = torch.zeros(p.noise.shape, dtype=torch.float32).pin_memory()
        self._host_out = torch.zeros(p.out.shape, dtype=torch.float32).pin_memory()
        # batched staging: observation groups copied into pinned memory by helper threads (numpy
        # copies release the GIL), each group's H2D issued as soon as its copy is done
        self._stage_groups = [(g * self.batch // n, (g + 1) * self.batch // n)
                              for n in [min(8, self.batch, os.cpu_count() or 1)] for g in range(n)]  # fmt: skip
        self._pool = ThreadPoolExecutor(len(self._stage_groups)) if len(self._stage_groups) > 1 else None
        if self._pool is not None:  # the helper threads end with the engine
            weakref.finalize(self, self._pool.shutdown, wait=False)
        self.dt = -1.0 / s.n_steps
        self.timing = Timing()
        self._stages = [self._vision, self._prefix, self._denoise]
        self.graph = None
        if cuda_graph:
            self._capture(warmup)
        else:
            with torch.no_grad():
                for _ in range(warmup):
                    self._forward()
            torch.cuda.synchronize(dev)

    # ------------------------------------------------------------------ stages
    def _vision(self) -> None:
        self.path.run("vision")

    def _prefix(self, _rows=None) -> None:
        self.path.run("prefix")

    def _denoise(self) -> None:
        self.path.run("denoise")

    def _forward(self) -> None:
        self._vision()
        self._prefix()
        self._denoise()

    def step(self, k: int) -> torch.Tensor:
        """v_t of denoising step k for the current x_t (the noise buffer), (B, H, max_action)."""
        prog = self.path.velocity_program(k)
        self.path.v_buf.zero_()
        prog.run(torch.cuda.current_stream(self.device).cuda_stream)
        return self.path.v_buf.view(self.batch, self.spec.chunk, self.spec.max_action)

    def _capture(self, warmup: int) -> None:
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                self._forward()
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._forward()
        torch.cuda.synchronize(self.device)

    # ------------------------------------------------------------------ staging
    def _stage(self, images, states, noises) -> None:
        """Host observations -> pinned buffers -> device (async on the current stream). The
        previous call synchronized its stream, so the pinned buffers are free to overwrite."""
        host = (self._host_img, self._host_state, self._host_noise)
        self._stage_into(images, states, noises, host, (self.img, self.state, self.noise))

    def _stage_into(self, images, states, noises, host, dev, draw_noise: bool = True) -> None:
        """Copy B observations into the pinned buffers `host` = (img, state, noise) and issue their
        host-to-device copies into `dev` on the current stream; noises None draws the noise on the
        device instead (or leaves it to the caller, draw_noise False)."""
        B, C_ = self.batch, len(self.cams)
        h_img, h_state, h_noise = host
        d_img, d_state, d_noise = dev
        hi = h_img.numpy()

        def fill(b0: int, b1: int) -> None:
            for bi in range(b0, b1):
                for ci, c in enumerate(self.cams):
                    hi[bi * C_ + ci] = images[bi][c]

        if self._pool is None:
            fill(0, B)
            d_img.copy_(h_img, non_blocking=True)
        else:
            futures = [self._pool.submit(fill, b0, b1) for b0, b1 in self._stage_groups]
            for (b0, b1), f in zip(self._stage_groups, futures, strict=True):
                f.result()
                d_img[b0 * C_ : b1 * C_].copy_(h_img[b0 * C_ : b1 * C_], non_blocking=True)
        h_state.numpy()[:] = np.asarray(states, np.float32).reshape(B, self.state_dim)
        d_state.copy_(h_state, non_blocking=True)
        if noises is None:
            if draw_noise:
                d_noise.normal_()
        else:
            h_noise.numpy()[:] = np.asarray(noises, np.float32).reshape(h_noise.shape)
            d_noise.copy_(h_noise, non_blocking=True)

    def _run(self) -> np.ndarray:
        if self.graph is not None:
            self.graph.replay()
        else:
            self._forward()
        self._host_out.copy_(self.out, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return self._host_out.numpy().copy()

    # ------------------------------------------------------------------ public
    def infer(self, images: dict[str, np.ndarray], state: np.ndarray, noise: np.ndarray | None = None) -> np.ndarray:
        """The action chunk (chunk, action_dim) for one observation (`pkg/model/engine.py:312-344`).

        `images` maps each camera key to an HxWx3 uint8 frame, `state` is (state_dim,); `noise`
        (chunk, max_action) fixes the initial noise."""
        if self.batch != 1:
            raise ValueError(f"this engine holds batch {self.batch}: use infer_batch")
        t0 = time.perf_counter()
        self._stage([images], [state], None if noise is None else [noise])
        out = self._run()[0]
        self.timing.add((time.perf_counter() - t0) * 1e3)
        return out

    def infer_batch(self, images: list[dict[str, np.ndarray]], states, noises=None) -> np.ndarray:
        """Chunks (B, chunk, action_dim) for B observations in one graph replay."""
        if len(images) != self.batch:
            raise ValueError(f"expected {self.batch} observations, got {len(images)}")
        t0 = time.perf_counter()
        self._stage(images, states, noises)
        out = self._run()
        self.timing.add((time.perf_counter() - t0) * 1e3)
        return out

    def infer_stream(self, batches):
        """Serving loop: for an iterable of (images, states[, noises]) batches of this engine's batch
        size, yield each batch's chunks (B, chunk, action_dim) in order. While batch i's graph
        runs, batch i+1's frames are copied into a second set of pinned buffers by the helper
        threads and uploaded on a copy stream into a device staging set; a device-to-device copy
        (about 0.05 ms for 64 observations) moves them into the graph's input buffers before its
        replay. Every batch still pays its own host-to-device and device-to-host copies; they are
        off the GPU's critical path. Results equal infer_batch's on the same inputs."""
        if self.graph is None:
            raise RuntimeError("infer_stream replays the captured graph: build the engine with cuda_graph=True")
        if not hasattr(self, "_stream_bufs"):
            pin = [(torch.zeros_like(h, device="cpu").pin_memory(), torch.zeros_like(s, device="cpu").pin_memory(),
                    torch.zeros_like(n, device="cpu").pin_memory())
                   for h, s, n in [(self._host_img, self._host_state, self._host_noise)]]  # fmt: skip
            self._stream_bufs = {
                "host": [(self._host_img, self._host_state, self._host_noise), pin[0]],
                "dev": (torch.empty_like(self.img), torch.empty_like(self.state), torch.empty_like(self.noise)),
                "copy": torch.cuda.Stream(self.device),
            }
        bufs = self._stream_bufs
        comp, copy = torch.cuda.current_stream(self.device), bufs["copy"]
        staged, consumed, done = (torch.cuda.Event() for _ in range(3))

        def stage(batch, k: int) -> bool:
            """Stage `batch` through pinned set k on the copy stream, after the previous batch was
            consumed; whether its noise is drawn on the device."""
            images, states, *rest = batch
            noises = rest[0] if rest else None
            if len(images) != self.batch:
                raise ValueError(f"expected {self.batch} observations, got {len(images)}")
            copy.wait_event(consumed)
            with torch.cuda.stream(copy):
                # drawn noise comes from the compute stream at consume time, as infer_batch draws it
                self._stage_into(images, states, noises, bufs["host"][k], bufs["dev"], draw_noise=False)
                staged.record(copy)
            return noises is None

        it = iter(batches)
        cur = next(it, None)
        if cur is None:
            return
        consumed.record(comp)  # the staging buffers are free
        try:
            yield from self._stream_loop(it, cur, stage, bufs, comp, staged, consumed, done)
        finally:  # a caller that stops early leaves no upload in flight into the pinned buffers
            copy.synchronize()

    def _stream_loop(self, it, cur, stage, bufs, comp, staged, consumed, done):
        """infer_stream's loop: replay batch i while batch i+1 is staged."""
        draw = stage(cur, 0)
        k = 0
        while cur is not None:
            t0 = time.perf_counter()
            comp.wait_event(staged)
            d_img, d_state, d_noise = bufs["dev"]
            self.img.copy_(d_img, non_blocking=True)
            self.state.copy_(d_state, non_blocking=True)
            if draw:
                self.noise.normal_()
            else:
                self.noise.copy_(d_noise, non_blocking=True)
            consumed.record(comp)
            self.graph.replay()
            self._host_out.copy_(self.out, non_blocking=True)
            done.record(comp)
            nxt = next(it, None)
            if nxt is not None:
                k ^= 1
                draw = stage(nxt, k)  # host copies and upload while the graph runs
            done.synchronize()
            self.timing.add((time.perf_counter() - t0) * 1e3)
            yield self._host_out.numpy().copy()
            cur = nxt

    @torch.no_grad()
    def profile(self, images, state, reps: int = 20) -> dict:
        """Median GPU ms per stage, each stage captured as its own CUDA graph
        (`pkg/model/engine.py:347-379`)."""
        if self.batch == 1:
            self.infer(images, state)
        else:
            self.infer_batch(images, state)
        stages = {"vision": self._vision, "prefix": self._prefix, "denoise": self._denoise}
        graphs = {}
        for name, fn in stages.items():
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            graphs[name] = g
        res = {}
        for name, g in graphs.items():
            ts = []
            for _ in range(reps):
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                torch.cuda.synchronize(self.device)
                ts.append(e0.elapsed_time(e1))
            res[name] = float(np.median(ts))
        return res

    def launches(self) -> int:
        """Kernel launches per chunk replay."""
        return self.path.launches()

    @torch.no_grad()
    def calibrate(self, observations: list[dict[str, np.ndarray]], include_patch: bool = False) -> dict[str, float]:
        """Activation clips for int8 vision: max |input| of each vision linear over the frames of
        `observations`, through this engine's bf16 vision kernels (the calibration of the
        reference's int8 test, `tests/test_ov_engine.py:222-225`). The patch GEMM stays bf16
        unless `include_patch`."""
        if self.vision_precision != "bf16":
            raise ValueError("calibrate on a bf16 engine")
        return self.path.calibrate(observations, self.cams, include_patch)


def clip_names(spec, include_patch: bool = False) -> list[str]:
    names = vision_linear_names(spec)
    return names if include_patch else [n for n in names if n != "patch"]
