"""The chunk on the B200 kernels: vision tower, prefix pass and denoising loop as fixed launch lists.

`B200Path` replaces the reference's two backend seams with one object:

    TritonPath (pkg/model/smolvla_triton.py:46-130)   prefix pass + velocity on custom kernels
    TrtVision  (pkg/model/trt_vision.py:212-252)      vision stage in fixed buffers, bf16 or int8

It owns every buffer the chunk touches (weights, activations, the expert's K/V caches at the kv
heads in token-major (len, n_kv * hd) layout, split-K workspace) and builds three `Program`s —
vision, prefix, denoise — each a list of C-ABI launches with their arguments fixed once. Running a
program issues the launches on the current stream; capturing the three into one CUDA graph is the
engine's chunk. Batch B runs B independent observations through the same launches (GEMMs over
all B's rows at once, attention per observation).

Layout (B observations, C cameras, Np patches per camera, L prefix rows, H action rows):
    img      (B*C, h, w, 3) u8       patches (B*C*Np, 3 P^2)     xv  (B*C*Np, vis_dim) fp32
    x_pre    (B*L, text_dim) fp32 residual stream of the prefix pass
    ck/cv[i] (B, L+H, kv) bf16 self layers: rows [:L] VLM keys/values, rows [L:] this step's own
    kx/vx[i] (B, L, kv) bf16 cross layers: the expert's projections of the VLM keys/values
    x_t      (B*H, max_action) fp32, e (B*H, exp_dim) fp32 expert residual stream
"""

from __future__ import annotations

import ctypes as C
import json
import math
import os
import weakref

import numpy as np
import torch

from . import _lib as L
from .bundle import Bundle
from .ops import DTYPE, workspace
from .spec import ModelSpec, vision_linear_names

REPRS = {"absolute": 0, "delta": 1, "velocity": 2}
STAT_SLOTS = 64  # statistics slots per row for the RMSNorm finished in a GEMM (so101_epilogue.rms_ss)
# Plans `B200Path.autotune` times for a GEMM with many token rows (so101_gemm_config: swap, bn,
# splits, stages, flags): the library's pick, the persistent kernel and the CTA pair at three tile
# widths each. None of them splits K, so the choice never changes the accumulation order.
TUNE_CANDIDATES = (None, (0, 256, 1, 0, L.GEMM_PERSISTENT), (0, 192, 1, 0, L.GEMM_PERSISTENT),
                   (0, 128, 1, 0, L.GEMM_PERSISTENT), (0, 256, 1, 0, L.GEMM_PAIR),
                   (0, 192, 1, 0, L.GEMM_PAIR), (0, 128, 1, 0, L.GEMM_PAIR))  # fmt: skip
TUNE_MIN_ROWS = 1024  # token-tile candidates from this many rows on
# Weight-streaming plans for at most 256 token rows (the expert and the prefix at batch 1): 32- and
# 64-token tiles with 1-8 K splits over a cluster.
TUNE_SMALL = (None,) + tuple((1, bn, s, 0, 0) for bn in (32, 64) for s in (1, 2, 3, 4, 6, 8))
TUNE_SMALL_ROWS = 256
TUNE_MARGIN = 0.97  # a candidate replaces the pick only when at least 3% faster
TUNE_MARGIN_STAGE = 0.998  # in a stage's chain: at least 0.2% of the stage faster
# From this many expert rows (observations x 50 actions) on, the action/time MLP's fp32 output
# projection runs as one bf16 tensor-core GEMM over split operands (so101_split_bf16x3, about 2^-16
# relative; the reference rounds its output to the run dtype right after: model/smolvla.py:285)
# instead of the fp32 CUDA-core linear: 120 -> ~30 us per step at 64 observations.
SPLIT_TIME_OUT_ROWS = 1024


def unsupported(spec: ModelSpec) -> str | None:
    """Why the B200 kernels cannot run this model, or None."""
    hd_v = spec.vis_dim // max(spec.vis_heads, 1)
    if spec.head_dim not in (32, 64, 128):
        return f"head_dim {spec.head_dim} is not 32, 64 or 128"
    if spec.vis_dim % spec.vis_heads or hd_v not in (32, 64, 128):
        return f"vision head size {hd_v} is not 32, 64 or 128"
    if spec.n_heads % spec.n_kv:
        return "n_heads is not a multiple of n_kv"
    ks = {"vis_dim": spec.vis_dim, "patch features": 3 * spec.patch**2, "vis_mlp": spec.vis_mlp,
          "connector": spec.vis_dim * spec.shuffle**2, "text_dim": spec.text_dim,
          "q heads": spec.q_dim, "text_mlp": spec.text_mlp, "kv": spec.kv_dim,
          "exp_dim": spec.exp_dim, "exp_mlp": spec.exp_mlp}  # fmt: skip
    for name, k in ks.items():
        if k % 16:
            return f"{name} width {k} is not a multiple of 16 (TMA rows of 16-byte multiples)"
    for name, n in (("vis_dim", spec.vis_dim), ("text_dim", spec.text_dim), ("exp_dim", spec.exp_dim)):
        if n > 1024:
            return f"{name} {n} is wider than the row kernels' 1024"
    g = spec.grid
    if spec.image_size % spec.patch or g % spec.shuffle:
        return "the patch grid does not divide by the shuffle factor"
    return None


class Program:
    """A fixed list of C-ABI launches; `run` issues them on a stream."""

    def __init__(self, name: str):
        self.name = name
        self.calls: list[tuple[str, object, tuple]] = []
        self._keep: list[object] = []

    def add(self, what: str, fn, *args, keep=()) -> None:
        self.calls.append((what, fn, args))
        self._keep.extend(keep)

    def run(self, stream: int) -> None:
        for what, fn, args in self.calls:
            rc = fn(*args, stream)
            if rc:
                L.check(rc, f"{self.name}/{what}")

    def __len__(self) -> int:
        return len(self.calls)


def _rope(pos: torch.Tensor, hd: int, base: float) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin (len, hd/2) in float32 exactly as the reference builds them
    (pkg/model/smolvla.py:77-85), on the host."""
    half = hd // 2
    exps = (2.0 / hd) * torch.arange(half, dtype=torch.float32)
    ang = pos.float()[:, None] / (base**exps)[None, :]
    return torch.cos(ang), torch.sin(ang)


def _time_proj(s: ModelSpec, w_time: np.ndarray, b: np.ndarray) -> torch.Tensor:
    """Time half of action_time_mlp_in for every step, bias included (pkg/model/engine.py:137-141)."""
    dt = -1.0 / s.n_steps
    t = torch.tensor([1.0 + k * dt for k in range(s.n_steps)], dtype=torch.float32).double()
    frac = torch.linspace(0.0, 1.0, s.exp_dim // 2, dtype=torch.float64)
    period = s.min_period * (s.max_period / s.min_period) ** frac
    ang = t[:, None] * (2 * math.pi / period)[None, :]
    temb = torch.cat([torch.sin(ang), torch.cos(ang)], dim=-1).float()
    return temb @ torch.from_numpy(w_time).T + torch.from_numpy(b)


class Packed:
    """A bundle's weights in the layout the kernels read, on one device: every matrix in bf16,
    the norms, biases and small float32 tables, the folded action/time input projection, the time
    projection table and the RoPE tables, and the int8 per-output-channel copies (with their
    scales) of the vision linears that run W8A8. The B200 counterpart of the reference's load-time
    packing (`pkg/model/bundle.py:303-326`, which casts every parameter to the compute dtype and
    moves it to the device), plus the int8 packing its TensorRT build does
    (`pkg/model/trt_vision.py:131-133`).

    Each tensor crosses to the device once, in float32; the bf16 and int8 copies are made there
    from that upload. Packed sets are kept per (bundle checksum, spec, device, int8 linears) while
    any path uses them, so a second engine on the same bundle reuses the first one's weights
    instead of uploading and packing again (they are read-only: sharing them is safe)."""

    _cache: weakref.WeakValueDictionary = weakref.WeakValueDictionary()
    packs = 0  # how many sets were packed (not reused) in this process

    @classmethod
    def get(cls, b: Bundle, device: torch.device, int8_names, lib) -> Packed:
        key = (b.checksum(), json.dumps(b.spec.__dict__, sort_keys=True, default=str), str(device),
               tuple(int8_names))  # fmt: skip
        pk = cls._cache.get(key)
        if pk is None:
            pk = cls(b, device, tuple(int8_names), lib)
            cls._cache[key] = pk
            cls.packs += 1
        return pk

    def __init__(self, b: Bundle, dev: torch.device, int8_names: tuple[str, ...], lib):
        from .spec import param_shapes

        s, t = b.spec, b.tensors
        self.w: dict[str, torch.Tensor] = {}
        self.wq: dict[str, tuple[torch.Tensor, torch.Tensor]] = {}
        wnames = {"vis.patch.w" if q == "patch" else ("conn.w" if q == "conn" else q + ".w"): q
                  for q in int8_names}  # fmt: skip
        stream = torch.cuda.current_stream(dev).cuda_stream if dev.type == "cuda" else 0
        for name, (_, kind) in param_shapes(s).items():
            f32 = torch.from_numpy(np.ascontiguousarray(t[name], dtype=np.float32)).to(dev)
            self.w[name] = f32.to(torch.bfloat16).contiguous() if kind == "w" else f32.contiguous()
            q = wnames.get(name)
            if q is not None:  # W8A8: per-output-channel int8 from the float32 weights
                n, k = f32.shape
                wq = torch.empty(n, k, dtype=torch.int8, device=dev)
                sc = torch.empty(n, dtype=torch.float32, device=dev)
                L.check(lib.so101_quantize_weight(f32.data_ptr(), L.F32, n, k, wq.data_ptr(), sc.data_ptr(),
                                                  stream), "quantize_weight")  # fmt: skip
                self.wq[q] = (wq, sc)
            if dev.type == "cuda":
                torch.cuda.current_stream(dev).synchronize()  # the float32 upload may go
        for name in ("lang.emb", "norm.state.mean", "norm.state.std", "norm.action.mean",
                     "norm.action.std"):  # fmt: skip
            self.w[name] = torch.from_numpy(np.ascontiguousarray(t[name])).to(dev).float()
        for name, n in (("repr.mean", 0.0), ("repr.std", 1.0)):
            v = t.get(name)
            v = np.full(s.max_action, n, np.float32) if v is None else v
            self.w[name] = torch.from_numpy(np.ascontiguousarray(v)).to(dev).float()
        # act.in and time_in's action half are consecutive linear maps of x_t: fold them once
        w_a = t["act.time_in.w_action"].astype(np.float64)
        self.w["act.ain.w"] = torch.from_numpy((w_a @ t["act.in.w"].astype(np.float64)).astype(np.float32)).to(dev)
        self.w["act.ain.b"] = torch.from_numpy((w_a @ t["act.in.b"].astype(np.float64)).astype(np.float32)).to(dev)
        self.w["time_proj"] = _time_proj(s, t["act.time_in.w_time"], t["act.time_in.b"]).to(dev).contiguous()
        L_, H, hd = s.prefix_len, s.chunk, s.head_dim
        for key, pos in (("p", torch.arange(L_)), ("s", torch.arange(L_, L_ + H)), ("c", torch.arange(H))):
            c, sn = _rope(pos, hd, s.rope_wavelength)
            self.w[f"cos_{key}"], self.w[f"sin_{key}"] = c.to(dev), sn.to(dev)


class B200Path:
    """Weights, buffers and launch programs of one chunk (or B chunks) on one GPU."""

    def __init__(self, bundle: Bundle, device: torch.device, batch: int = 1,
                 vision_precision: str = "bf16", act_clip: dict[str, float] | None = None,
                 expert_step: str = "auto", fold_norms: bool = True, lib=None):  # fmt: skip
        s = self.spec = bundle.spec
        why = unsupported(s)
        if why:
            raise ValueError(f"the B200 kernels cannot run this model: {why}")
        if vision_precision not in ("bf16", "int8"):
            raise ValueError(f"vision precision must be 'bf16' or 'int8', not {vision_precision!r}")
        if vision_precision == "int8" and not act_clip:
            raise ValueError("int8 vision needs activation clips (act_clip)")
        self.bundle, self.meta = bundle, bundle.meta
        self.dev = device
        self.B = B = int(batch)
        self.lib = L.lib() if lib is None else lib  # lib: a stand-in, for host-logic tests only
        self.int8 = vision_precision == "int8"
        self.clip = dict(act_clip or {})
        if self.int8:
            bad = set(self.clip) - set(vision_linear_names(s))
            if bad:
                raise ValueError(f"act_clip names no vision linear: {sorted(bad)[:4]}")
        self.C, self.Np, self.L, self.H = s.n_cams, s.n_patches, s.prefix_len, s.chunk
        self.h_img, self.w_img = bundle.meta["image_hw"]
        self.state_dim, self.action_dim = bundle.meta["state_dim"], bundle.meta["action_dim"]
        self.repr = REPRS[bundle.meta["action_repr"]]
        if expert_step not in ("auto", "fused", "ops"):
            raise ValueError(f"expert_step must be 'auto', 'fused' or 'ops', not {expert_step!r}")
        self.fold = bool(fold_norms)  # RMSNorm split into the GEMMs around it (else an rms_norm launch each)
        # one observation: each expert layer's SwiGLU MLP block in one launch (so101_mlp) unless
        # SO101_FUSED_MLP=0, and its attention, output projection and residual in one launch
        # (so101_attention_o). SO101_ATTN_O: "all" (default; on B200 14.7 against 15.2 us for the
        # attention + GEMM launches over the self layers' 291 keys, 12.1 against 14.2 over the cross
        # layers' 241), "cross" or "0".
        one = self.B == 1 and s.chunk <= 64
        self.mlp_fused = (one and s.exp_mlp % 128 == 0 and s.exp_mlp <= 2048
                          and os.environ.get("SO101_FUSED_MLP", "1") != "0")  # fmt: skip
        mode = os.environ.get("SO101_ATTN_O", "all")
        if mode not in ("cross", "all", "0"):
            raise ValueError(f"SO101_ATTN_O must be 'cross', 'all' or '0', not {mode!r}")
        ok = one and s.head_dim == 64 and s.n_heads <= 16
        self.attn_o_layers = {i for i in range(s.n_layers)
                              if ok and (mode == "all" or (mode == "cross" and not s.is_self_attn(i)))}  # fmt: skip
        # many observations: the masked tcgen05 attention (attention_gqa_tc.cu) serves the expert too;
        # both it and the mma.sync kernel (few observations) read the step's own keys and values from
        # the fused qkv rows and rotate the keys on chip (no rope_kv launch into the cache)
        self.gqa_tc = (s.head_dim == 64 and self.B * s.n_kv >= 64
                       and os.environ.get("SO101_ATTN_GQA_TC", "1") != "0")  # fmt: skip
        self.ws = workspace(device)  # split-K partials and tickets exist before any capture
        self._amax: tuple[torch.Tensor, dict[str, int]] | None = None  # calibration hooks
        self._upload(bundle)
        self._alloc()
        self.xs = self._expert_step(expert_step)
        self.tuned: dict[tuple, tuple | None] = {}  # GEMM signature -> plan chosen by autotune
        self._build_all()

    def _build_all(self) -> None:
        self._sites: dict[tuple, tuple[str, tuple]] = {}  # GEMM signature -> (name, launch args)
        self.progs = {"vision": Program("vision"), "prefix": Program("prefix"),
                      "denoise": Program("denoise")}  # fmt: skip
        self._build_vision(self.progs["vision"])
        self._build_prefix(self.progs["prefix"])
        self._build_denoise(self.progs["denoise"])
        # the reference's backend seams (prefix / velocity / vision from px): the same launches
        # over caller-given rows, time projection and frames
        pl = Program("prefix_layers")
        pl.calls = [c for c in self.progs["prefix"].calls if c[0] != "prefix_tail"]
        pl._keep = [self.progs["prefix"]]
        vx = Program("velocity")
        self._build_step(vx, 0, self.x_seam, self.v_buf, 1.0, tp=self.tp_seam)
        vp = Program("vision_px")
        self._build_vision(vp, source="px")
        self.seams = {"prefix": pl, "velocity": vx, "vision": vp}

    def autotune(self, reps: int = 5) -> dict[str, dict]:
        """Time every candidate plan (TUNE_CANDIDATES; TUNE_SMALL for at most 256 rows) of each
        distinct GEMM with many or few token rows on this GPU, on its first launch site's own
        buffers, and rebuild the programs with the fastest. The B200 counterpart of the reference's autotuned GEMMs (`compile="autotune"`,
        pkg/model/engine.py:219-233, and `scripts/tune_gemm.py`). Rebuilding matters: a residual
        GEMM's plan sets how many statistics slots the next norm's GEMM reads. Overwrites the
        work buffers (the next chunk recomputes them). Returns {site: {"plan", "ms"}}."""
        stream = torch.cuda.current_stream(self.dev).cuda_stream
        report: dict[str, dict] = {}
        for key, (what, args) in self._sites.items():
            times: dict[tuple | None, float] = {}
            for cand in (TUNE_SMALL if key[1] <= TUNE_SMALL_ROWS else TUNE_CANDIDATES):
                cfg = None if cand is None else L.GemmConfig(*cand)
                a = list(args)
                a[12] = None if cfg is None else C.byref(cfg)
                need, tick = C.c_int64(), C.c_int64()
                if self.lib.so101_gemm_workspace(a[0], a[8], a[9], a[10], key[4], a[12], C.byref(need),
                                                 C.byref(tick)) != L.OK or need.value > self.ws.nbytes:  # fmt: skip
                    continue
                if self.lib.so101_gemm(*a, stream) != L.OK:  # a plan this epilogue cannot take
                    continue
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(reps):
                    L.check(self.lib.so101_gemm(*a, stream), f"autotune {what}")
                e1.record()
                e1.synchronize()
                times[cand] = e0.elapsed_time(e1) / reps
            best = min(times, key=times.get)
            if None in times and times[best] > TUNE_MARGIN * times[None]:
                best = None  # within noise of the library's pick: keep it, so engines agree run to run
            self.tuned[key] = best
            report[what] = {"plan": best, "ms": {str(c): t for c, t in times.items()}}
        torch.cuda.synchronize(self.dev)
        self._refine_small(report)
        self._build_all()
        return report

    def _refine_small(self, report: dict[str, dict], runs: int = 3) -> None:
        """The few-row GEMMs (the expert and the prefix at one observation) once more, each
        candidate timed inside its stage's own launch chain rather than alone: there a kernel's
        prologue overlaps its predecessor's tail, which decides among these microsecond GEMMs.
        Coordinate descent, one site at a time, keeping the others' current plans; the stage runs
        eagerly on the engine's buffers (whatever they hold: the next chunk recomputes them)."""
        stream = torch.cuda.current_stream(self.dev)

        def stage_ms(build) -> float:
            prog = Program("refine")
            build(prog)
            prog.run(stream.cuda_stream)  # warm
            best = float("inf")
            for _ in range(runs):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                prog.run(stream.cuda_stream)
                e1.record(stream)
                e1.synchronize()
                best = min(best, e0.elapsed_time(e1))
            return best

        for build, name in ((self._build_denoise, "denoise"), (self._build_prefix, "prefix")):
            names = {c[0] for c in self.progs[name].calls}
            keys = [k for k, (what, _) in self._sites.items()
                    if k[1] <= TUNE_SMALL_ROWS and k[0] == L.BF16 and what in names]  # fmt: skip
            for key in keys:
                what = self._sites[key][0]
                keep = self.tuned.get(key)
                times: dict[tuple | None, float] = {}
                for cand in TUNE_SMALL:
                    self.tuned[key] = cand
                    try:
                        times[cand] = stage_ms(build)
                    except (ValueError, RuntimeError):  # a plan this GEMM cannot take
                        continue
                if not times:
                    self.tuned[key] = keep
                    continue
                best = min(times, key=times.get)
                if keep in times and times[best] > TUNE_MARGIN_STAGE * times[keep]:
                    best = keep  # within noise of the alone-timed pick
                self.tuned[key] = best
                if what in report:
                    report[what]["plan"] = best
                    report[what]["stage_ms"] = {str(c): t for c, t in times.items()}

    # ------------------------------------------------------------------ weights and buffers
    def _upload(self, b: Bundle) -> None:
        """Device weights from the bundle's packed set (see `Packed`): packed once per bundle,
        device and int8 selection, shared by every path built from them."""
        pk = Packed.get(b, self.dev, sorted(self.clip) if self.int8 else (), self.lib)
        self.packed = pk
        self.w, self.wq = pk.w, pk.wq

    def _alloc(self) -> None:
        s, dev, B = self.spec, self.dev, self.B
        C_, Np, L_, H = self.C, self.Np, self.L, self.H
        bf, f32, i8 = torch.bfloat16, torch.float32, torch.int8
        rows_v = B * C_ * Np
        vd, sh = s.vis_dim, s.shuffle
        qdt = lambda name: i8 if (self.int8 and name in self.clip) else bf  # noqa: E731

        def z(*shape, dtype=f32):
            return torch.zeros(*shape, dtype=dtype, device=dev)

        self.img = z(B * C_, self.h_img, self.w_img, 3, dtype=torch.uint8)
        self.state = z(B, self.state_dim)
        self.noise = z(B, H, s.max_action)  # x_t: the noise, denoised in place
        self.out = z(B, H, self.action_dim)
        # vision
        self.patches = z(rows_v, 3 * s.patch**2, dtype=qdt("patch"))
        self.xv = z(rows_v, vd)
        self.hv_bf = z(rows_v, vd, dtype=bf)
        self.hv_i8 = z(rows_v, vd, dtype=i8) if self.int8 else None
        self.qkv_v = z(rows_v, 3 * vd, dtype=bf)
        self.attn_v_bf = z(rows_v, vd, dtype=bf)
        self.attn_v_i8 = z(rows_v, vd, dtype=i8) if self.int8 else None
        self.mlp_v_bf = z(rows_v, s.vis_mlp, dtype=bf)
        self.mlp_v_i8 = z(rows_v, s.vis_mlp, dtype=i8) if self.int8 else None
        self.shuf = z(rows_v // sh**2, vd * sh**2, dtype=qdt("conn"))
        # prefix
        self.x_pre = z(B * L_, s.text_dim)  # the prefix residual stream
        self.h_t = z(B * L_, s.text_dim, dtype=bf)
        self.qkv_t = z(B * L_, s.qkv_dim, dtype=bf)
        self.attn_t = z(B * L_, s.q_dim, dtype=bf)
        self.mlp_t = z(B * L_, s.text_mlp, dtype=bf)
        kv = s.kv_dim
        layers = range(s.n_layers)
        self.ck = [z(B, L_ + H, kv, dtype=bf) if s.is_self_attn(i) else None for i in layers]
        self.cv = [z(B, L_ + H, kv, dtype=bf) if s.is_self_attn(i) else None for i in layers]
        self.kx = [None if s.is_self_attn(i) else z(B, L_, kv, dtype=bf) for i in layers]
        self.vx = [None if s.is_self_attn(i) else z(B, L_, kv, dtype=bf) for i in layers]
        self.k_scratch = z(B * L_, kv, dtype=bf)
        self.ss_t = z(B * L_, STAT_SLOTS)  # per-row sums of squares of the prefix residual stream
        # expert
        self.h0 = z(B * H, s.exp_dim)
        self.e = z(B * H, s.exp_dim)
        self.h_e = z(B * H, s.exp_dim, dtype=bf)
        self.qkv_e = z(B * H, s.qkv_dim, dtype=bf)
        self.attn_e = z(B * H, s.q_dim, dtype=bf)
        self.mlp_e = z(B * H, s.exp_mlp, dtype=bf)
        self.v_buf = z(B * H, s.max_action)
        # inputs of the reference's backend seams (velocity's x_t and time projection, vision's px)
        self.x_seam = z(B * H, s.max_action)
        self.tp_seam = z(s.exp_dim)
        self.px_seam = z(B * C_, 3, s.image_size, s.image_size)
        self.ss_e = z(B * H, STAT_SLOTS)  # per-row sums of squares of the expert residual stream
        # the batched time MLP output: split activations and [W_hi | W_lo | W_hi]
        self.split_out = B * H >= SPLIT_TIME_OUT_ROWS
        if self.split_out:
            wt = self.w["act.time_out.w"]
            hi = wt.to(bf)
            self.w3_time_out = torch.cat([hi, (wt - hi.float()).to(bf), hi], dim=1).contiguous()
            self.h0_3 = z(B * H, 3 * s.exp_dim, dtype=bf)

    def _expert_step(self, mode: str) -> L.ExpertStep | None:
        """The persistent expert-step problem for one observation, or None (per-op launches).

        "fused" requires it (one observation, shapes the library accepts); "auto" and "ops" use the
        per-op launch chain, which is the faster of the two on B200 (0.78 ms against 1.36 ms per
        denoising step at configs[0] when compared, 0.57 ms now with the fused expert kernels): the
        persistent kernel's phases are chains of dependent global-memory round trips plus a grid
        barrier, while consecutive per-op kernels overlap their prologues through programmatic
        dependent launch."""
        s, w = self.spec, self.w
        if mode in ("ops", "auto"):
            return None
        if self.B != 1 or s.n_layers > L.EXPERT_MAX_LAYERS:
            raise ValueError("the fused expert step serves one observation of at most 16 layers")
        H = self.H
        xs = L.ExpertStep()
        xs.n_layers, xs.rows, xs.prefix_len = s.n_layers, H, self.L
        xs.exp_dim, xs.q_dim, xs.kv_dim = s.exp_dim, s.q_dim, s.kv_dim
        xs.n_heads, xs.n_kv, xs.head_dim, xs.mlp_dim = s.n_heads, s.n_kv, s.head_dim, s.exp_mlp
        xs.eps = s.rms_eps
        for i in range(s.n_layers):
            pre, y = f"exp.{i}.", xs.layer[i]
            y.self_attn = int(s.is_self_attn(i))
            y.w_attn = w[pre + ("qkv" if y.self_attn else "q")].data_ptr()
            y.w_o, y.w_gate_up = w[pre + "o"].data_ptr(), w[pre + "gate_up"].data_ptr()
            y.w_down = w[pre + "down"].data_ptr()
            y.ln_in, y.ln_post = w[pre + "ln_in"].data_ptr(), w[pre + "ln_post"].data_ptr()
            kt, vt = (self.ck[i], self.cv[i]) if y.self_attn else (self.kx[i], self.vx[i])
            y.k, y.v = kt.data_ptr(), vt.data_ptr()
        self.q_e = torch.zeros(H, s.q_dim, dtype=torch.bfloat16, device=self.dev)
        xs.e, xs.q, xs.attn, xs.act = (self.e.data_ptr(), self.q_e.data_ptr(), self.attn_e.data_ptr(),
                                       self.mlp_e.data_ptr())  # fmt: skip
        xs.cos_self, xs.sin_self = w["cos_s"].data_ptr(), w["sin_s"].data_ptr()
        xs.cos_cross, xs.sin_cross = w["cos_c"].data_ptr(), w["sin_c"].data_ptr()
        need = C.c_int64()
        L.check(self.lib.so101_expert_step_workspace(C.byref(xs), C.byref(need)), "expert_step_workspace")
        self.xs_ws = torch.zeros(need.value, dtype=torch.uint8, device=self.dev)
        xs.workspace, xs.workspace_bytes = self.xs_ws.data_ptr(), need.value
        return xs

    # ------------------------------------------------------------------ launch helpers
    def _gemm(self, prog: Program, what: str, x: torch.Tensor, w: torch.Tensor, y: torch.Tensor, *,
              bias=None, residual=None, r_period=0, gate=False, gelu=False, out_scale=1.0,
              row_map=(0, 0), x_scale=0.0, w_scale=None, y_qscale=0.0, M=None, rms=None,
              stat=None) -> int:  # fmt: skip
        """One GEMM launch. rms=(ss, slots): finish the RMSNorm of x in the GEMM (x = bf16(residual
        stream * norm weight), row m scaled by its rstd from ss). stat=(ss, x16, norm_w): also
        write the output rows' statistics and bf16(output * norm_w) for the next norm; returns the
        slot count (a separate statistics launch when the GEMM's plan cannot produce them)."""
        m = x.shape[0] if M is None else M
        k = x.shape[1]
        n = w.shape[0] // 2 if gate else w.shape[0]
        a_type = L.I8 if w.dtype == torch.int8 else L.BF16
        key = (a_type, m, n, k, L.EPI_SILU_GATE if gate else (L.EPI_GELU if gelu else L.EPI_NONE), DTYPE[y.dtype],
               -1 if residual is None else DTYPE[residual.dtype], bias is not None, rms is not None,
               stat is not None)  # fmt: skip
        plan = self.tuned.get(key)
        cfg = None if plan is None else L.GemmConfig(*plan)
        cfg_ref = None if cfg is None else C.byref(cfg)
        epi = L.Epilogue(
            epilogue=L.EPI_SILU_GATE if gate else (L.EPI_GELU if gelu else L.EPI_NONE),
            bias=None if bias is None else bias.data_ptr(),
            residual=None if residual is None else residual.data_ptr(),
            ldr=0 if residual is None else residual.stride(0),
            r_type=0 if residual is None else DTYPE[residual.dtype], r_period=r_period,
            out_scale=out_scale, w_scale=None if w_scale is None else w_scale.data_ptr(),
            x_scale=x_scale, y_qscale=y_qscale, row_group=row_map[0], row_stride=row_map[1],
        )  # fmt: skip
        if rms is not None:
            ss, slots = rms
            epi.rms_ss, epi.rms_slots, epi.rms_ld = ss.data_ptr(), slots, ss.stride(0)
            epi.rms_n, epi.rms_eps = float(k), self.spec.rms_eps
        slots_out = 0
        if stat is not None:
            ss, x16, nw = stat
            got = C.c_int()
            if self.lib.so101_gemm_stat_slots(a_type, m, n, k, epi.epilogue, cfg_ref, C.byref(got)) == L.OK \
                    and got.value <= ss.shape[1]:  # fmt: skip
                slots_out = got.value
                epi.stat_ss, epi.stat_ld = ss.data_ptr(), ss.stride(0)
                epi.y16, epi.ld16, epi.y16_scale = x16.data_ptr(), x16.stride(0), nw.data_ptr()
        need, tick = C.c_int64(), C.c_int64()
        L.check(self.lib.so101_gemm_workspace(a_type, m, n, k, epi.epilogue, cfg_ref, C.byref(need),
                                              C.byref(tick)), what)  # fmt: skip
        if need.value > self.ws.nbytes or tick.value > self.ws.tickets.numel():
            raise RuntimeError(f"{what}: split-K workspace too small ({need.value} bytes)")
        args = (a_type, x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), y.data_ptr(), y.stride(0),
                DTYPE[y.dtype], m, n, k, C.byref(epi), cfg_ref, self.ws.partials.data_ptr(), self.ws.nbytes,
                self.ws.tickets.data_ptr(), self.ws.tickets.numel())  # fmt: skip
        prog.add(what, self.lib.so101_gemm, *args, keep=(epi, cfg))
        if (m >= TUNE_MIN_ROWS or (m <= TUNE_SMALL_ROWS and a_type == L.BF16)) and key not in self._sites:
            self._sites[key] = (what, args)
        if stat is not None and slots_out == 0:
            slots_out = self._stats(prog, f"{what}.stats", y, stat[2], stat[1], stat[0])
        return slots_out

    def _stats(self, prog, what, x, nw, x16, ss) -> int:
        """Statistics (one slot) and bf16(x * nw) of the fp32 rows x, for the next norm's GEMM."""
        prog.add(what, self.lib.so101_rms_stats, x.data_ptr(), x.stride(0), x.shape[0], x.shape[1],
                 nw.data_ptr(), x16.data_ptr(), x16.stride(0), ss.data_ptr(), ss.stride(0))  # fmt: skip
        return 1

    def _attn(self, prog, what, q, ldq, bq, k, ldk, bk, v, ldv, bv, o, ldo, bo, *, Lq, Lk, nq, nkv,
              hd, causal_from, q_offset=0, cos=None, sin=None, batch=1, o_qscale=0.0, own=None):  # fmt: skip
        """One attention launch; own=(k_own, v_own, ld, batch stride, own_from, k_cos, k_sin) reads
        keys and values from own_from on from the fused qkv rows and rotates those keys on chip."""
        o_type = L.I8 if o.dtype == torch.int8 else L.BF16
        args = (q, ldq, k, ldk, v, ldv, o.data_ptr() if isinstance(o, torch.Tensor) else o, ldo, o_type, o_qscale,
                Lq, Lk, nq, nkv, hd, causal_from, q_offset, None if cos is None else cos.data_ptr(),
                None if sin is None else sin.data_ptr(), batch, bq, bk, bv, bo)  # fmt: skip
        if own is None:
            prog.add(what, self.lib.so101_attention, *args)
        else:
            k_own, v_own, ld_own, b_own, own_from, k_cos, k_sin = own
            prog.add(what, self.lib.so101_attention_rows, *args, k_own, v_own, ld_own, b_own, own_from,
                     k_cos.data_ptr(), k_sin.data_ptr())  # fmt: skip

    def _attn_o(self, prog, what, q, ldq, bq, k, ldk, bk, v, ldv, bv, *, w_o, y, stat, Lq, Lk, nq, nkv, hd,
                causal_from, q_offset=0, cos=None, sin=None, batch=1, own=None) -> int:  # fmt: skip
        """Attention, output projection and residual in one launch (so101_attention_o): y += attention
        @ w_o^T. stat=(ss, x16, norm_w) also writes the statistics slots (returned) and
        bf16(y * norm_w) for the next norm's GEMM."""
        own_args = (None, None, 0, 0, 0, None, None) if own is None else \
            (*own[:5], own[5].data_ptr(), own[6].data_ptr())  # fmt: skip
        ss, x16, nw = stat if stat is not None else (None, None, None)
        prog.add(what, self.lib.so101_attention_o, q, ldq, k, ldk, v, ldv, Lq, Lk, nq, nkv, hd, causal_from,
                 q_offset, None if cos is None else cos.data_ptr(), None if sin is None else sin.data_ptr(), batch,
                 bq, bk, bv, *own_args, w_o.data_ptr(), w_o.stride(0), w_o.shape[0], y.data_ptr(), y.stride(0),
                 y.data_ptr(), y.stride(0), None if x16 is None else x16.data_ptr(),
                 0 if x16 is None else x16.stride(0), None if nw is None else nw.data_ptr(),
                 None if ss is None else ss.data_ptr(), 0 if ss is None else ss.stride(0))  # fmt: skip
        return (w_o.shape[0] + 127) // 128 if stat is not None else 0

    def _mlp(self, prog, what, x, w_gu, w_down, y, *, rms, stat) -> int:
        """The SwiGLU MLP block in one launch (so101_mlp): y += silu(x gate^T) (x up^T) w_down^T, the
        RMSNorm of x finished from rms=(ss, slots); stat as _attn_o. One observation of <= 64 rows."""
        ss, slots = rms if rms is not None else (None, 0)
        s_ss, x16, nw = stat if stat is not None else (None, None, None)
        prog.add(what, self.lib.so101_mlp, x.data_ptr(), x.stride(0), x.shape[0], 1, x.shape[1],
                 None if ss is None else ss.data_ptr(), slots, 0 if ss is None else ss.stride(0), self.spec.rms_eps,
                 w_gu.data_ptr(), w_gu.stride(0), w_down.shape[1], w_down.data_ptr(), w_down.stride(0),
                 w_down.shape[0], y.data_ptr(), y.stride(0), y.data_ptr(), y.stride(0),
                 None if x16 is None else x16.data_ptr(), 0 if x16 is None else x16.stride(0),
                 None if nw is None else nw.data_ptr(), None if s_ss is None else s_ss.data_ptr(),
                 0 if s_ss is None else s_ss.stride(0))  # fmt: skip
        return (w_down.shape[0] + 127) // 128 if stat is not None else 0

    def _rms(self, prog, what, x, w, y, rows):
        s = self.spec
        prog.add(what, self.lib.so101_rms_norm, x.data_ptr(), x.stride(0), DTYPE[x.dtype], w.data_ptr(),
                 y.data_ptr(), y.stride(0), DTYPE[y.dtype], rows, x.shape[1], s.rms_eps)  # fmt: skip

    def _qs(self, name: str) -> float:
        """Per-tensor int8 scale of linear `name`'s input (0 when it stays bf16)."""
        return self.clip[name] / 127.0 if (self.int8 and name in self.clip) else 0.0

    # ------------------------------------------------------------------ vision
    def fused_patch(self) -> bool:
        """Whether the frames go straight into the patch GEMM (so101_patch_embed), which needs
        frames at the model's size (no resize), 16-pixel patches whose 128-patch blocks are whole
        patch rows of a frame, a bf16 patch GEMM and a feature count that is a multiple of 256.
        Opt-in (SO101_FUSED_PATCH=1): on B200 it is slower than the separate launches (917 against
        670 us at 64 observations, 85 against 25 us at one), because each 128-patch tile streams the
        whole 1.2 MB weight matrix through its ring, far more than the patch rows it saves."""
        s = self.spec
        g = s.image_size // 16
        can = (self.h_img == s.image_size and self.w_img == s.image_size and s.patch == 16
               and s.vis_dim % 256 == 0 and 128 % g == 0 and (g * g) % 128 == 0
               and self._qs("patch") == 0.0 and self._amax is None)  # fmt: skip
        return can and os.environ.get("SO101_FUSED_PATCH", "0") == "1"

    def _build_vision(self, p: Program, source: str = "frames") -> None:
        """The vision tower's launches from the uint8 frames (img), or from preprocessed px
        (source "px", the TrtVision seam)."""
        s, w = self.spec, self.w
        B, C_, Np = self.B, self.C, self.Np
        S = s.image_size
        h, wd = self.h_img, self.w_img
        ratio = max(wd / S, h / S)
        rh, rw = int(h / ratio), int(wd / ratio)
        vd, nh = s.vis_dim, s.vis_heads
        hd = vd // nh
        rows_v = B * C_ * Np
        qs = self._qs("patch")
        if source == "frames" and self.fused_patch():
            pw = w["vis.patch.w"]
            p.add("patch_embed", self.lib.so101_patch_embed, self.img.data_ptr(), B * C_, S, pw.data_ptr(),
                  pw.stride(0), vd, w["vis.patch.b"].data_ptr(), w["vis.pos"].data_ptr(), Np, self.xv.data_ptr(),
                  self.xv.stride(0))  # fmt: skip
        else:
            if source == "px":
                p.add("patchify", self.lib.so101_patchify, self.px_seam.data_ptr(), B * C_, S, s.patch,
                      self.patches.data_ptr(), DTYPE[self.patches.dtype], qs)  # fmt: skip
            else:
                p.add("preprocess", self.lib.so101_preprocess, self.img.data_ptr(), B * C_, h, wd, rh, rw, S,
                      s.patch, self.patches.data_ptr(), DTYPE[self.patches.dtype], qs)  # fmt: skip
            self._lin(p, "patch", self.patches, "vis.patch.w", self.xv, bias=w["vis.patch.b"],
                      residual=w["vis.pos"], r_period=Np)  # fmt: skip
        for i in range(s.vis_layers):
            pre = f"vis.{i}."
            hv = self._vis_in(pre + "qkv", self.hv_bf, self.hv_i8)
            p.add(f"{i}.ln1", self.lib.so101_layer_norm, self.xv.data_ptr(), vd, w[pre + "ln1.w"].data_ptr(),
                  w[pre + "ln1.b"].data_ptr(), hv.data_ptr(), vd, DTYPE[hv.dtype], self._qs(pre + "qkv"),
                  rows_v, vd, s.vis_eps, 1, 0)  # fmt: skip
            self._lin(p, pre + "qkv", hv, pre + "qkv.w", self.qkv_v, bias=w[pre + "qkv.b"])
            av = self._vis_in(pre + "out", self.attn_v_bf, self.attn_v_i8)
            base = self.qkv_v.data_ptr()
            self._attn(p, f"{i}.attn", base, 3 * vd, Np * 3 * vd, base + 2 * vd, 3 * vd, Np * 3 * vd,
                       base + 4 * vd, 3 * vd, Np * 3 * vd, av, vd, Np * vd, Lq=Np, Lk=Np, nq=nh,
                       nkv=nh, hd=hd, causal_from=Np, batch=B * C_,
                       o_qscale=self._qs(pre + "out"))  # fmt: skip
            self._lin(p, pre + "out", av, pre + "out.w", self.xv, bias=w[pre + "out.b"], residual=self.xv)
            hv = self._vis_in(pre + "fc1", self.hv_bf, self.hv_i8)
            p.add(f"{i}.ln2", self.lib.so101_layer_norm, self.xv.data_ptr(), vd, w[pre + "ln2.w"].data_ptr(),
                  w[pre + "ln2.b"].data_ptr(), hv.data_ptr(), vd, DTYPE[hv.dtype], self._qs(pre + "fc1"),
                  rows_v, vd, s.vis_eps, 1, 0)  # fmt: skip
            mv = self._vis_in(pre + "fc2", self.mlp_v_bf, self.mlp_v_i8)
            self._lin(p, pre + "fc1", hv, pre + "fc1.w", mv, bias=w[pre + "fc1.b"], gelu=True,
                      y_qscale=self._qs(pre + "fc2"))  # fmt: skip
            self._lin(p, pre + "fc2", mv, pre + "fc2.w", self.xv, bias=w[pre + "fc2.b"], residual=self.xv)
        p.add("post_ln+shuffle", self.lib.so101_layer_norm, self.xv.data_ptr(), vd,
              w["vis.post_ln.w"].data_ptr(), w["vis.post_ln.b"].data_ptr(), self.shuf.data_ptr(),
              self.shuf.stride(0), DTYPE[self.shuf.dtype], self._qs("conn"), rows_v, vd, s.vis_eps,
              s.shuffle, Np)  # fmt: skip
        self._lin(p, "conn", self.shuf, "conn.w", self.x_pre, out_scale=math.sqrt(s.text_dim),
                  row_map=(C_ * s.img_tokens, self.L))  # fmt: skip

    def _vis_in(self, name: str, bf: torch.Tensor, i8: torch.Tensor | None) -> torch.Tensor:
        return i8 if (self.int8 and name in self.clip) else bf

    def _lin(self, p: Program, q: str, x, wname: str, y, **kw) -> None:
        """A vision linear: int8 operands when `q` has a clip, else bf16."""
        if self._amax is not None:  # calibration: fold max |x| of this linear's input
            amax, idx = self._amax
            p.add(f"amax {q}", self.lib.so101_absmax, x.data_ptr(), x.stride(0), DTYPE[x.dtype],
                  x.shape[0], x.shape[1], amax.data_ptr() + 4 * idx[q])  # fmt: skip
        if self.int8 and q in self.clip:
            wq, ws = self.wq[q]
            self._gemm(p, q, x, wq, y, x_scale=self.clip[q] / 127.0, w_scale=ws, **kw)
        else:
            self._gemm(p, q, x, self.w[wname], y, **kw)

    # ------------------------------------------------------------------ prefix
    def _build_prefix(self, p: Program) -> None:
        s, w = self.spec, self.w
        B, L_, H = self.B, self.L, self.H
        nq, nk, hd, kv, qd = s.n_heads, s.n_kv, s.head_dim, s.kv_dim, s.qkv_dim
        tail = self.C * s.img_tokens
        p.add("prefix_tail", self.lib.so101_prefix_tail, self.state.data_ptr(), self.state_dim,
              w["norm.state.mean"].data_ptr(), w["norm.state.std"].data_ptr(), w["state.w"].data_ptr(),
              s.max_state, w["state.b"].data_ptr(), w["lang.emb"].data_ptr(), s.lang_len, s.text_dim,
              self.x_pre.data_ptr(), s.text_dim, L_, tail, B)  # fmt: skip
        x = self.x_pre
        esz = 2  # bf16 bytes
        # RMSNorm in two halves: the residual GEMM before it writes bf16(x * w) and per-row sums of
        # squares, the GEMM after it scales its rows by rstd (fold); else an rms_norm launch
        fold = self.fold
        slots = self._stats(p, "prefix.stats", x, w["txt.0.ln_in"], self.h_t, self.ss_t) if fold else 0
        for i in range(s.n_layers):
            t = f"txt.{i}."
            if not fold:
                self._rms(p, f"{i}.ln_in", x, w[t + "ln_in"], self.h_t, B * L_)
            self._gemm(p, f"{i}.qkv", self.h_t, w[t + "qkv"], self.qkv_t, rms=(self.ss_t, slots) if fold else None)
            qkv_ptr = self.qkv_t.data_ptr()
            if s.is_self_attn(i):
                k_ptr, v_ptr = self.ck[i].data_ptr(), self.cv[i].data_ptr()
                bk = (L_ + H) * kv
                p.add(f"{i}.rope_kv", self.lib.so101_rope_kv, qkv_ptr, qd, nq, nk, hd,
                      w["cos_p"].data_ptr(), w["sin_p"].data_ptr(), k_ptr, kv, v_ptr, kv, L_, B,
                      L_ * qd, bk, bk)  # fmt: skip
                ldk = ldv = kv
                bv = bk
            else:
                k_ptr = self.k_scratch.data_ptr()
                p.add(f"{i}.rope_k", self.lib.so101_rope_kv, qkv_ptr, qd, nq, nk, hd,
                      w["cos_p"].data_ptr(), w["sin_p"].data_ptr(), k_ptr, kv, None, 0, L_, B,
                      L_ * qd, L_ * kv, 0)  # fmt: skip
                self._gemm(p, f"{i}.exp_k", self.k_scratch, w[f"exp.{i}.k"], self.kx[i].view(B * L_, kv))
                v_view = self.qkv_t[:, (nq + nk) * hd:]
                self._gemm(p, f"{i}.exp_v", v_view, w[f"exp.{i}.v"], self.vx[i].view(B * L_, kv))
                v_ptr = qkv_ptr + (nq + nk) * hd * esz
                ldk, bk, ldv, bv = kv, L_ * kv, qd, L_ * qd
            if i == s.n_layers - 1:
                break  # the last layer's output is never read
            self._attn(p, f"{i}.attn", qkv_ptr, qd, L_ * qd, k_ptr, ldk, bk, v_ptr, ldv, bv, self.attn_t,
                       s.q_dim, L_ * s.q_dim, Lq=L_, Lk=L_, nq=nq, nkv=nk, hd=hd, causal_from=L_ - 1,
                       cos=w["cos_p"], sin=w["sin_p"], batch=B)  # fmt: skip
            if fold:
                slots = self._gemm(p, f"{i}.o", self.attn_t, w[t + "o"], x, residual=x,
                                   stat=(self.ss_t, self.h_t, w[t + "ln_post"]))  # fmt: skip
            else:
                self._gemm(p, f"{i}.o", self.attn_t, w[t + "o"], x, residual=x)
                self._rms(p, f"{i}.ln_post", x, w[t + "ln_post"], self.h_t, B * L_)
            self._gemm(p, f"{i}.gate_up", self.h_t, w[t + "gate_up"], self.mlp_t, gate=True,
                       rms=(self.ss_t, slots) if fold else None)  # fmt: skip
            nxt = (self.ss_t, self.h_t, w[f"txt.{i + 1}.ln_in"]) if fold else None
            slots = self._gemm(p, f"{i}.down", self.mlp_t, w[t + "down"], x, residual=x, stat=nxt)

    # ------------------------------------------------------------------ denoising
    def _build_step(self, p: Program, k: int, x_in: torch.Tensor, x_out: torch.Tensor, dt: float,
                    tp: torch.Tensor | None = None) -> None:
        """One velocity evaluation at step k, folded into x_out += dt * v; tp (exp_dim) replaces
        step k's row of the time projection table."""
        s, w = self.spec, self.w
        B, L_, H = self.B, self.L, self.H
        nq, nk, hd, kv, qd = s.n_heads, s.n_kv, s.head_dim, s.kv_dim, s.qkv_dim
        M = B * H
        tp = w["time_proj"][k] if tp is None else tp
        p.add(f"s{k}.act_time_in", self.lib.so101_linear_f32, x_in.data_ptr(), s.max_action,
              w["act.ain.w"].data_ptr(), s.max_action, w["act.ain.b"].data_ptr(), tp.data_ptr(),
              self.h0.data_ptr(), s.exp_dim, M, s.exp_dim, s.max_action, 2)  # fmt: skip
        e = self.e
        fold = self.fold and self.xs is None
        slots = 0
        if self.split_out and self.xs is None:
            # fp32 linear on the tensor cores: [h_hi | h_hi | h_lo] [W_hi | W_lo | W_hi]^T + b, with
            # the first layer's norm statistics and bf16 operand in the same epilogue
            p.add(f"s{k}.time_split", self.lib.so101_split_bf16x3, self.h0.data_ptr(), s.exp_dim, M, s.exp_dim,
                  self.h0_3.data_ptr(), 3 * s.exp_dim)  # fmt: skip
            slots = self._gemm(p, f"s{k}.time_out", self.h0_3, self.w3_time_out, e, bias=w["act.time_out.b"],
                               stat=(self.ss_e, self.h_e, w["exp.0.ln_in"]) if fold else None)  # fmt: skip
        else:
            p.add(f"s{k}.time_out", self.lib.so101_linear_f32, self.h0.data_ptr(), s.exp_dim,
                  w["act.time_out.w"].data_ptr(), s.exp_dim, w["act.time_out.b"].data_ptr(), None,
                  self.e.data_ptr(), s.exp_dim, M, s.exp_dim, s.exp_dim, 0)  # fmt: skip
            if fold:
                slots = self._stats(p, f"s{k}.stats", e, w["exp.0.ln_in"], self.h_e, self.ss_e)
        if self.xs is not None:
            p.add(f"s{k}.expert_layers", self.lib.so101_expert_step_run, C.byref(self.xs), keep=(self.xs,))
        for i in range(s.n_layers if self.xs is None else 0):
            pre = f"exp.{i}."
            if not fold:
                self._rms(p, f"s{k}.{i}.ln_in", e, w[pre + "ln_in"], self.h_e, M)
            rms = (self.ss_e, slots) if fold else None
            if s.is_self_attn(i):
                self._gemm(p, f"s{k}.{i}.qkv", self.h_e, w[pre + "qkv"], self.qkv_e, rms=rms)
                bk = (L_ + H) * kv
                own = None
                if hd == 64 and (H <= 64 or not self.gqa_tc):  # the step's own keys and values from the qkv rows
                    k_own = self.qkv_e.data_ptr() + nq * hd * 2
                    own = (k_own, k_own + nk * hd * 2, qd, H * qd, L_, w["cos_s"], w["sin_s"])
                else:  # RoPE and the K/V cache rows in a separate launch
                    off = L_ * kv * 2  # bytes to the step's own rows
                    p.add(f"s{k}.{i}.rope_kv", self.lib.so101_rope_kv, self.qkv_e.data_ptr(), qd, nq, nk, hd,
                          w["cos_s"].data_ptr(), w["sin_s"].data_ptr(), self.ck[i].data_ptr() + off, kv,
                          self.cv[i].data_ptr() + off, kv, H, B, H * qd, bk, bk)  # fmt: skip
                operands = (self.qkv_e.data_ptr(), qd, H * qd, self.ck[i].data_ptr(), kv, bk, self.cv[i].data_ptr(),
                            kv, bk)  # fmt: skip
                geom = dict(Lq=H, Lk=L_ + H, nq=nq, nkv=nk, hd=hd, causal_from=L_, q_offset=L_, cos=w["cos_s"],
                            sin=w["sin_s"], batch=B, own=own)  # fmt: skip
            else:
                qv = self.qkv_e[:, : s.q_dim]
                self._gemm(p, f"s{k}.{i}.q", self.h_e, w[pre + "q"], qv, rms=rms)
                operands = (self.qkv_e.data_ptr(), qd, H * qd, self.kx[i].data_ptr(), kv, L_ * kv,
                            self.vx[i].data_ptr(), kv, L_ * kv)  # fmt: skip
                geom = dict(Lq=H, Lk=L_, nq=nq, nkv=nk, hd=hd, causal_from=L_, cos=w["cos_c"], sin=w["sin_c"],
                            batch=B)  # fmt: skip
            post = (self.ss_e, self.h_e, w[pre + "ln_post"]) if fold else None
            if i in self.attn_o_layers:  # attention, output projection and residual in one launch
                slots = self._attn_o(p, f"s{k}.{i}.attn_o", *operands, w_o=w[pre + "o"], y=e, stat=post, **geom)
                if not fold:
                    self._rms(p, f"s{k}.{i}.ln_post", e, w[pre + "ln_post"], self.h_e, M)
            else:
                self._attn(p, f"s{k}.{i}.attn", *operands, self.attn_e, s.q_dim, H * s.q_dim, **geom)
                if fold:
                    slots = self._gemm(p, f"s{k}.{i}.o", self.attn_e, w[pre + "o"], e, residual=e, stat=post)
                else:
                    self._gemm(p, f"s{k}.{i}.o", self.attn_e, w[pre + "o"], e, residual=e)
                    self._rms(p, f"s{k}.{i}.ln_post", e, w[pre + "ln_post"], self.h_e, M)
            # the last layer's output goes to the final norm of so101_expert_out (fp32, from e)
            nxt = (self.ss_e, self.h_e, w[f"exp.{i + 1}.ln_in"]) if fold and i + 1 < s.n_layers else None
            if self.mlp_fused:  # gate/up, SiLU gate, down and residual in one launch
                slots = self._mlp(p, f"s{k}.{i}.mlp", self.h_e, w[pre + "gate_up"], w[pre + "down"], e,
                                  rms=(self.ss_e, slots) if fold else None, stat=nxt)  # fmt: skip
            else:
                self._gemm(p, f"s{k}.{i}.gate_up", self.h_e, w[pre + "gate_up"], self.mlp_e, gate=True,
                           rms=(self.ss_e, slots) if fold else None)  # fmt: skip
                slots = self._gemm(p, f"s{k}.{i}.down", self.mlp_e, w[pre + "down"], e, residual=e, stat=nxt)
        p.add(f"s{k}.out+euler", self.lib.so101_expert_out, e.data_ptr(), s.exp_dim, w["exp.norm"].data_ptr(),
              s.rms_eps, w["act.out.w"].data_ptr(), w["act.out.b"].data_ptr(), x_out.data_ptr(),
              s.max_action, M, s.max_action, s.exp_dim, dt)  # fmt: skip

    def _build_denoise(self, p: Program) -> None:
        s, w = self.spec, self.w
        x = self.noise.view(self.B * self.H, s.max_action)
        for k in range(s.n_steps):
            self._build_step(p, k, x, x, -1.0 / s.n_steps)
        p.add("finish", self.lib.so101_finish, self.noise.data_ptr(), s.max_action, self.state.data_ptr(),
              self.state_dim, w["norm.state.mean"].data_ptr(), w["norm.state.std"].data_ptr(),
              w["repr.mean"].data_ptr(), w["repr.std"].data_ptr(), w["norm.action.mean"].data_ptr(),
              w["norm.action.std"].data_ptr(), self.out.data_ptr(), self.action_dim, self.H, self.repr,
              self.B)  # fmt: skip

    def velocity_program(self, k: int) -> Program:
        """v_t at step k of the current x_t (noise buffer) into v_buf (for parity tests)."""
        p = Program(f"velocity{k}")
        x = self.noise.view(self.B * self.H, self.spec.max_action)
        self._build_step(p, k, x, self.v_buf, 1.0)
        return p

    @torch.no_grad()
    def calibrate(self, observations, cams, include_patch=False) -> dict[str, float]:
        """max |input| per vision linear over the observations' frames (bf16 vision)."""
        names = vision_linear_names(self.spec)
        amax = torch.zeros(len(names), dtype=torch.float32, device=self.dev)
        prog = Program("calibrate")
        self._amax = (amax, {n: i for i, n in enumerate(names)})
        try:
            self._build_vision(prog)
        finally:
            self._amax = None
        stream = torch.cuda.current_stream(self.dev).cuda_stream
        B, C_ = self.B, self.C
        obs = list(observations)
        for start in range(0, len(obs), B):
            chunk = obs[start : start + B]
            chunk += [chunk[-1]] * (B - len(chunk))
            frames = np.stack([o[c] for o in chunk for c in cams])
            self.img.copy_(torch.from_numpy(frames))
            prog.run(stream)
        vals = amax.cpu().tolist()
        return {n: v for n, v in zip(names, vals, strict=True) if include_patch or n != "patch"}

    # ------------------------------------------------------------------ the reference's seams
    def prefix(self, rows: torch.Tensor) -> None:
        """`TritonPath.prefix` (pkg/model/smolvla_triton.py:78-103): the VLM layers over the
        prefix rows (L, text_dim) float32 — (B, L, text_dim) for a batch — filling the self layers'
        key/value rows [:L] (ck, cv) and the cross layers' expert keys/values (kx, vx). Enqueued on
        the current stream."""
        s = self.spec
        want = (self.B, self.L, s.text_dim)
        if rows.numel() != self.B * self.L * s.text_dim or rows.shape[-1] != s.text_dim:
            raise ValueError(f"prefix rows must be {want[1:] if self.B == 1 else want}, got {tuple(rows.shape)}")
        self.x_pre.copy_(rows.reshape(self.B * self.L, s.text_dim))
        self.seams["prefix"].run(self._stream())

    def velocity(self, x_t: torch.Tensor, time_proj: torch.Tensor) -> torch.Tensor:
        """`TritonPath.velocity` (pkg/model/smolvla_triton.py:105-130): v_t (B, chunk, max_action)
        float32 for x_t (B, chunk, max_action) float32 and the time half of the action/time MLP's
        input, time_proj (1, 1, exp_dim) with its bias (the reference's `Engine.time_proj[k]`), over
        the caches the last `prefix` call filled. Returns a fixed buffer that the next call
        overwrites (the caller adds dt * v_t, as the reference's `Engine.step` does)."""
        s = self.spec
        if x_t.numel() != self.B * self.H * s.max_action or time_proj.numel() != s.exp_dim:
            raise ValueError(f"x_t must hold {self.B} x {self.H} x {s.max_action} and time_proj {s.exp_dim} values")
        self.x_seam.copy_(x_t.reshape(self.x_seam.shape))
        self.tp_seam.copy_(time_proj.reshape(s.exp_dim))
        self.v_buf.zero_()
        self.seams["velocity"].run(self._stream())
        return self.v_buf.view(self.B, self.H, s.max_action)

    def encode_images(self, px: torch.Tensor) -> torch.Tensor:
        """`TrtVision.__call__` (pkg/model/trt_vision.py:247-252): px (B * n_cams, 3, S, S) float32
        in [-1, 1] to image rows (B * n_cams * img_tokens, text_dim) float32 (B = 1: one block of
        rows, as the reference's), in bf16 or W8A8 as this path was built. The rows are a view of
        this path's prefix buffer, overwritten by the next call."""
        if tuple(px.shape) != tuple(self.px_seam.shape):
            raise ValueError(f"px must be {tuple(self.px_seam.shape)}, got {tuple(px.shape)}")
        self.px_seam.copy_(px)
        self.seams["vision"].run(self._stream())
        n = self.C * self.spec.img_tokens
        rows = self.x_pre.view(self.B, self.L, -1)[:, :n]
        return rows[0] if self.B == 1 else rows.reshape(self.B * n, -1)

    # ------------------------------------------------------------------ running
    def _stream(self) -> int:
        """The current CUDA stream's handle (0 for a host-only stand-in path)."""
        return torch.cuda.current_stream(self.dev).cuda_stream if self.dev.type == "cuda" else 0

    def run(self, stage: str, stream: int | None = None) -> None:
        st = self._stream() if stream is None else stream
        self.progs[stage].run(st)

    def run_chunk(self, stream: int | None = None) -> None:
        for name in ("vision", "prefix", "denoise"):
            self.run(name, stream)

    def launches(self) -> int:
        return sum(len(p) for p in self.progs.values())
