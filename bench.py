#!/usr/bin/env python3
"""Benchmark: batched SmolVLA chunks/s on 1..8 B200 (replicas), plus batch-1 chunk latency.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N

Workload: a step is one chunk for each of 64 observations per GPU:
3 x 512^2 uint8 cameras, W8A8 int8 SigLIP calibrated on 32 seeded observations, bf16 prefix
(241 rows x 16 layers) and action expert (10 Euler steps x 16 layers), 50 x 12 actions out, as one
CUDA-graph replay of the B200 kernels. Weights are the seeded configs[0] stand-in. Every rank runs
its own replica on its own observations; there is no collective on the data path, only a barrier
and a max over ranks around the timed region.

One JSON line (rank 0): value = chunks/s over all ranks with inputs resident in HBM (CUDA events,
max over ranks); e2e = the same through the serving loop `Engine.infer_stream` from host numpy
buffers (every batch's pinned H2D of frames, state and noise and D2H of its actions inside the
timed region; a batch's host copies and upload overlap the previous batch's graph); latency = the
configs[3] batch-1 bf16 chunk, p50/p99 over 200 `Engine.infer` calls (rank 0); roofline = the
dominant kernel timed alone with CUDA events against MEASURED_PEAKS.json; cpu_baseline = the
float32 CPU oracle (the reference's own algorithm restated) on this host's cores.

reference_gpu = the reference's own Triton and torch engines (baseline/_ref) on the same GPU at
configs[3], each in a child process.

`--impl reference` times the reference's own float32 CPU path (its `Engine(device="cpu")` from
baseline/_ref, else the oracle port) on the host's cores with the same metric and unit; under
torchrun only rank 0 runs it.
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

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BATCH = 64


def metric_name(batch: int) -> str:
    return f"batched chunks/s ({batch} obs/GPU, W8A8 vision, 50x12 actions, 10 steps)"


METRIC = metric_name(BATCH)
UNIT = "chunks/s"
CALIB_SEEDS = range(1000, 1032)


def env_rank() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))  # fmt: skip


# ------------------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi sampled every 100 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")  # fmt: skip

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-i", str(self.idx), "-lms", "100"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)  # fmt: skip
        except OSError:
            self.p = None
        time.sleep(0.25)
        return self

    def __exit__(self, *exc):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self) -> dict:
        self.f.flush()
        rows = [r.split(", ") for r in Path(self.f.name).read_text().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for name, v in zip(names, r[5:9], strict=False):
                    if v.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}  # fmt: skip


def peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ------------------------------------------------------------------------------ the reference
REF_DIR = ROOT / "baseline" / "_ref"  # the reference package (installed there, git-ignored)


def reference_engine_class():
    """The reference's own `Engine` from baseline/_ref, or None when it is not there."""
    if not (REF_DIR / "so101_smolvla_edge").exists():
        return None
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    try:
        from so101_smolvla_edge.model.engine import Engine as RefEngine
    except Exception:  # noqa: BLE001  (a reference that does not import is reported as absent)
        return None
    return RefEngine


def cpu_chunker():
    """(chunk(obs) -> actions, kind, description) for the float32 CPU path: the reference's own
    `Engine(device="cpu", dtype="fp32")` from baseline/_ref when present, else the oracle port."""
    from so101_smolvla_edge_b200.bundle import seeded_bundle, write_bundle

    b = seeded_bundle()
    RefEngine = reference_engine_class()
    if RefEngine is not None:
        d = write_bundle(b, Path(tempfile.mkdtemp(prefix="so101_ref_")) / "config0")
        eng = RefEngine(str(d), device="cpu", dtype="fp32", cuda_graph=False, warmup=0)
        return (lambda o: eng.infer(o[0], o[1], noise=o[2])), "reference", (
            "the reference's own Engine(device='cpu', dtype='fp32', cuda_graph=False) from baseline/_ref")
    from oracle.smolvla_fp32 import Oracle

    o_ = Oracle(b)
    return (lambda o: o_.actions(*o)), "port", "float32 torch CPU oracle (oracle/smolvla_fp32.py)"


def cpu_chunks_per_s(seconds: float = 15.0, min_chunks: int = 2, max_chunks: int | None = None) -> dict:
    """The float32 CPU path on configs[0] at batch 1, on every host thread."""
    import torch

    from so101_smolvla_edge_b200.bundle import observation, seeded_bundle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    b = seeded_bundle()
    chunk, kind, what = cpu_chunker()
    chunk(observation(b, 0))  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        chunk(observation(b, n + 1))
        n += 1
        el = time.perf_counter() - t0
        if (n >= min_chunks and el >= seconds) or (max_chunks and n >= max_chunks):
            break
    return {"value": n / el, "unit": UNIT, "cores": threads, "kind": kind,
            "sample": f"{n} chunks of configs[0] at batch 1 in {el:.1f} s: {what}"}  # fmt: skip


def reference_gpu_probe(kernels: str, chunks: int) -> None:
    """Child process: the reference's own engine on this GPU (configs[3]: batch 1, bf16, one CUDA
    graph per chunk, `vision="torch"`) with `kernels` "triton" or "torch". Prints one JSON line."""
    import torch

    from so101_smolvla_edge_b200.bundle import observation, seeded_bundle, write_bundle

    RefEngine = reference_engine_class()
    if RefEngine is None:
        print(json.dumps({"unavailable": "the reference package is not in baseline/_ref"}))
        return
    b = seeded_bundle()
    d = write_bundle(b, Path(tempfile.mkdtemp(prefix="so101_refgpu_")) / "config0")
    t0 = time.perf_counter()
    eng = RefEngine(str(d), device="cuda", dtype="bf16", kernels=kernels, vision="torch", warmup=3)
    build_s = time.perf_counter() - t0
    obs = [observation(b, s) for s in range(4)]
    for i in range(5):
        eng.infer(obs[i % 4][0], obs[i % 4][1])
    eng.timing.history.clear()
    for i in range(chunks):
        eng.infer(obs[i % 4][0], obs[i % 4][1])
    sm = eng.timing.summary()
    err = None
    gpath = ROOT / "tests" / "golden" / "golden_config0.npz"
    if gpath.exists():
        g = np.load(gpath)
        err = max(float(np.abs(eng.infer(*obs[i][:2], noise=obs[i][2]) - g["actions"][i]).max()) for i in range(4))
    stages = eng.profile(obs[0][0], obs[0][1], reps=10)
    names: dict[str, int] = {}
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof, torch.no_grad():
        eng._fwd()
        torch.cuda.synchronize()
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            names[ev.name] = names.get(ev.name, 0) + 1
    top = sorted(names.items(), key=lambda kv: -kv[1])
    print(json.dumps({"kernels": eng.kernels, "p50_ms": sm["p50_ms"], "p99_ms": sm["p99_ms"], "n": sm["n"],
                      "chunks_per_s": 1e3 / sm["p50_ms"],
                      "stages_ms": stages, "max_err_rad": err, "build_s": build_s,
                      "launches_per_chunk": sum(names.values()),
                      "kernel_names": [f"{k} x{v}" for k, v in top[:24]],
                      "triton_kernels": sum(v for k, v in names.items() if k.startswith("_") or "triton" in k.lower())}),
          flush=True)  # fmt: skip


def reference_gpu(chunks: int) -> dict:
    """The reference's own Triton and torch engines timed on this GPU, each in a child process
    (its Triton JIT, allocator and graphs stay out of this process)."""
    out = {}
    for kernels in ("triton", "torch"):
        try:
            r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--reference-gpu", kernels,
                                "--latency-chunks", str(chunks)], capture_output=True, text=True,
                               timeout=900)  # fmt: skip
            line = [x for x in r.stdout.splitlines() if x.startswith("{")]
            out[kernels] = json.loads(line[-1]) if line else {
                "unavailable": f"exit {r.returncode}: {(r.stderr or r.stdout).strip().splitlines()[-1:]}"}
        except subprocess.TimeoutExpired:
            out[kernels] = {"unavailable": "timed out after 900 s"}
    out["config"] = ("configs[3] through the reference's own Engine from baseline/_ref: batch 1, bf16, "
                     "one CUDA graph per chunk, vision='torch' (TensorRT is not installed); chunks_per_s = "
                     "1000 / p50, the rate of its API, which serves one observation per call")
    return out


def arm_config(world: int, batch: int) -> dict:
    """The workload both arms report (the reference arm times a bounded sample of it)."""
    return {"workload": f"configs[4]: {batch} observations/GPU x (3 x 512^2 u8 cameras, "
                        "241-token prefix, 10 denoise steps), W8A8 SigLIP + bf16 prefix/expert",
            "global_batch": world * batch, "per_gpu_batch": batch,
            "parallelism": f"replicas x{world} (no collective)",
            "l2": "inputs larger than L2 (0.7 GB weights, >4 GB activations per replay)",
            "gemm_plans": "autotuned at engine build (compile='autotune')",
            "act_clip": "the reference's calibration over 32 seeded observations (max |x| per vision linear)",
            "weights": "seeded configs[0] stand-in"}  # fmt: skip


def run_reference(args) -> None:
    """The reference arm: the reference's own float32 CPU path on this host's cores (the reference
    package from baseline/_ref, else the oracle port), one observation per chunk."""
    rank, _, world = env_rank()
    if rank != 0:
        return
    import torch

    from so101_smolvla_edge_b200.bundle import observation, seeded_bundle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    b = seeded_bundle()
    chunk, kind, what = cpu_chunker()
    for w in range(args.warmup):
        chunk(observation(b, 10_000 + w))
    t0 = time.perf_counter()
    for k in range(args.steps):
        chunk(observation(b, k))
    el = time.perf_counter() - t0
    v = args.steps / el
    cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": kind,
           "sample": f"{args.steps} chunks of the workload's observations one at a time (configs[0] "
                     f"weights, all host threads): {what}; chunks/s is per chunk, so the sample "
                     "measures the same metric"}  # fmt: skip
    print(json.dumps({
        "impl": "reference", "metric": metric_name(args.batch), "value": v, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": arm_config(world, args.batch),
        "cpu_baseline": cpu, "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0,
                                     "d2h_bytes_per_step": 0},
    }), flush=True)  # fmt: skip


# ------------------------------------------------------------------------------ ranks
class Ranks:
    """The bench's only cross-rank traffic: a barrier and a max around the timed region.

    `device` is where the reduction tensor lives (a CUDA device for NCCL, the CPU for gloo)."""

    def __init__(self, world: int, device=None):
        self.world = world
        self.device = device

    def barrier(self) -> None:
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()

    def max(self, x: float) -> float:
        if self.world == 1:
            return float(x)
        import torch
        import torch.distributed as dist

        t = torch.tensor([float(x)], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())


def throughput(world: int, per_rank: int, ms_max: float) -> float:
    """Whole-job chunks/s: every rank's chunks over the slowest rank's time."""
    return world * per_rank / (ms_max / 1e3)


# ------------------------------------------------------------------------------ ours
def gemm_kernel_name(plan, M, N, K) -> str:
    """The kernel a tokens-on-M GEMM plan (so101_gemm_config tuple, None: the library's pick) runs."""
    import ctypes as C

    import so101_smolvla_edge_b200._lib as L

    if plan is None:
        cfg = L.GemmConfig()
        L.lib().so101_gemm_pick(L.I8, M, N, K, L.EPI_GELU, C.byref(cfg))
        plan = (cfg.swap, cfg.bn, cfg.splits, cfg.stages, cfg.flags | L.GEMM_PERSISTENT)
    kind = "gemm_pair_kernel" if plan[4] & L.GEMM_PAIR else "gemm_persistent_kernel"
    return f"{kind}<{plan[1]},0,1>"


def observations(b, seeds):
    from so101_smolvla_edge_b200.bundle import observation

    return [observation(b, s) for s in seeds]


def calibrate(b, dev) -> dict[str, float]:
    """Per-tensor activation clips from the 32 calibration observations, through this engine's
    own bf16 vision (Engine.calibrate)."""
    import torch

    from so101_smolvla_edge_b200.engine import Engine

    eng = Engine(b, device=dev, warmup=0, cuda_graph=False, batch=8)
    clip = eng.calibrate([o[0] for o in observations(b, CALIB_SEEDS)])
    del eng
    torch.cuda.empty_cache()
    return clip


INT8_GOLDEN = ROOT / "tests" / "golden" / "golden_int8_config0.npz"


def reference_clips() -> dict[str, float] | None:
    """configs[4]'s calibration: the clips the reference's own calibration hook produced over the
    32 seeded calibration observations (max |x| per vision linear, `tests/test_ov_engine.py:
    222-225`), as the reference reads them from a bundle's trt/act_clip.json. Stored with the int8
    golden chunks that tests/golden/make_golden.py wrote by running the reference."""
    if not INT8_GOLDEN.exists():
        return None
    g = np.load(INT8_GOLDEN)
    return dict(zip(g["clip_names"].tolist(), (float(v) for v in g["clip_values"]), strict=True))


def int8_parity(acts: np.ndarray) -> dict | None:
    """The timed engine's W8A8 chunks for the golden seeds against the reference's own int8
    chunks, beside the reference's one-ulp reproducibility band (how far its own int8 chunk moves
    when its quantizers' float32 inputs move by one ulp) and against float32."""
    if not INT8_GOLDEN.exists():
        return None
    g = np.load(INT8_GOLDEN)
    ref, fp, ulp = g["actions_int8"], g["actions_fp32"], g["actions_int8_ulp"]
    n = ref.shape[0]
    return {"seeds": n,
            "max_err_rad_vs_reference_int8": np.abs(acts[:n] - ref).max(axis=(1, 2)).round(5).tolist(),
            "mean_err_rad_vs_reference_int8": float(np.abs(acts[:n] - ref).mean()),
            "reference_ulp_band_max_rad": float(np.abs(ulp - ref[None]).max()),
            "reference_ulp_band_mean_rad": float(np.abs(ulp - ref[None]).mean()),
            "max_err_rad_vs_fp32": np.abs(acts[:n] - fp).max(axis=(1, 2)).round(5).tolist(),
            "reference_int8_drift_vs_fp32": np.abs(ref - fp).max(axis=(1, 2)).round(5).tolist()}  # fmt: skip


def time_call(fn, args, reps: int = 20) -> float:
    """Average device ms of one C-ABI launch: `reps` launches captured back to back in a CUDA
    graph (no host launch overhead in the interval), CUDA events on the replay stream."""
    import torch

    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        for _ in range(3):
            fn(*args, side.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        st = torch.cuda.current_stream().cuda_stream
        for _ in range(reps):
            fn(*args, st)
    g.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    g.replay()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / reps


def find_call(prog, what: str):
    for name, fn, args in prog.calls:
        if name == what:
            return fn, args
    raise KeyError(what)


def profile_traffic(kernel: str):
    """DRAM bytes per launch of `kernel` from a committed ncu summary, if there is one."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        return json.loads(p.read_text()).get(kernel)
    return None


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    rank, local, world = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    from so101_smolvla_edge_b200.bundle import seeded_bundle
    from so101_smolvla_edge_b200.engine import Engine

    b = seeded_bundle()
    own_clip = calibrate(b, dev)
    clip = reference_clips() or own_clip
    clip_src = "reference" if clip is not own_clip else "engine"
    batch = args.batch
    eng = Engine(b, device=dev, batch=batch, trt_precision="int8", act_clip=clip, warmup=2,
                 pdl=args.pdl, compile="autotune")
    obs = observations(b, range(rank * batch, (rank + 1) * batch))
    imgs, states, noises = [o[0] for o in obs], [o[1] for o in obs], [o[2] for o in obs]
    eng._stage(imgs, states, noises)  # inputs resident in HBM for the device-timed loop
    stream = torch.cuda.current_stream(dev)

    ranks = Ranks(world, dev)

    def barrier():
        torch.cuda.synchronize(dev)
        ranks.barrier()

    max_over_ranks = ranks.max

    # ---- device-timed: one graph replay = 64 chunks per GPU, inputs resident
    for _ in range(args.warmup):
        eng.graph.replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks, torch.cuda.nvtx.range("bench_timed"):
        e0.record(stream)
        for _ in range(args.steps):
            eng.graph.replay()
        e1.record(stream)
        e1.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    value = throughput(world, batch, ms)
    clk = clocks.summary()

    # ---- end to end through the public API (host numpy in, actions out): the serving loop
    # (Engine.infer_stream: each batch's frames copied into pinned memory and uploaded while the
    # previous batch's graph runs; every batch's H2D and D2H inside the timed region)
    for _ in eng.infer_stream([(imgs, states, noises)] * max(2, args.warmup // 2)):
        pass
    barrier()
    t0 = time.perf_counter()
    for out in eng.infer_stream([(imgs, states, noises)] * args.steps):
        pass
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3) / args.steps
    h2d = eng.img.numel() + eng.state.numel() * 4 + eng.noise.numel() * 4
    d2h = eng.out.numel() * 4

    # ---- accuracy of the timed configuration against the reference's goldens: float32, and its
    # own W8A8 chunk (with the reference's clips, and with this engine's own calibration)
    err, parity = None, None
    gpath = ROOT / "tests" / "golden" / "golden_config0.npz"
    if gpath.exists() and rank == 0:
        g = np.load(gpath)
        n = g["actions"].shape[0]
        gobs = observations(b, range(n)) + obs[n:]
        res = eng.infer_batch([o[0] for o in gobs], [o[1] for o in gobs], [o[2] for o in gobs])
        err = float(np.abs(res[:n] - g["actions"]).max())
        parity = int8_parity(res)
        if parity is not None:
            parity["clips"] = clip_src
            if clip_src == "reference":  # the same chunks with the engine's own calibration
                eo = Engine(b, device=dev, batch=n, trt_precision="int8", act_clip=own_clip, warmup=1)
                own = eo.infer_batch([o[0] for o in gobs[:n]], [o[1] for o in gobs[:n]], [o[2] for o in gobs[:n]])
                po = int8_parity(own)
                parity["engine_calibration"] = {k: po[k] for k in ("max_err_rad_vs_reference_int8",
                                                                  "mean_err_rad_vs_reference_int8",
                                                                  "max_err_rad_vs_fp32")}  # fmt: skip
                del eo
                torch.cuda.empty_cache()

    # ---- dominant kernel alone: vision fc1 (int8 W8A8 GEMM + GELU + int8 requant epilogue)
    p = eng.path
    fn, cargs = find_call(p.progs["vision"], "vis.0.fc1")
    with torch.cuda.nvtx.range("roofline_kernel"):
        kms = time_call(fn, cargs)
    s = b.spec
    M, N, K = batch * s.n_cams * s.n_patches, s.vis_mlp, s.vis_dim
    pk, src = peaks()
    int8_peak = 2.0 * pk["bf16_tflops"]
    plans = {k: v["plan"] for k, v in (eng.tuning or {}).items()}
    kname = gemm_kernel_name(plans.get("vis.0.fc1"), M, N, K)
    roof = {"kernel": f"{kname} vis.0.fc1 (W8A8, GELU, int8 out)", "bound": "tensor",
            "achieved": 2.0 * M * N * K / (kms * 1e-3) / 1e12, "peak": int8_peak, "unit": "TOP/s",
            "traffic": profile_traffic("vis.fc1/" + kname.split("<")[0]), "ms": kms,
            "peak_source": f"2 x {src} bf16 dense ({pk['bf16_tflops']} TF/s): int8 dense rate is twice bf16"}  # fmt: skip
    roof["frac"] = roof["achieved"] / roof["peak"]
    # second family: SigLIP self-attention on tcgen05 (4 L^2 d flops per image and head)
    fn, cargs = find_call(p.progs["vision"], "0.attn")
    ams = time_call(fn, cargs, reps=10)
    n_img, hd = batch * s.n_cams, s.vis_dim // s.vis_heads
    aflops = 4.0 * n_img * s.vis_heads * s.n_patches**2 * hd
    roof_attn = {"kernel": "attention_tc_kernel vis.0.attn", "bound": "tensor",
                 "achieved": aflops / (ams * 1e-3) / 1e12, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                 "traffic": profile_traffic("vis.attn"), "ms": ams, "peak_source": f"{src} bf16 dense"}  # fmt: skip
    roof_attn["frac"] = roof_attn["achieved"] / roof_attn["peak"]
    # third family, the largest by launches: the bf16 GEMMs of the batched prefix and expert. The
    # expert's down projection (M = batch x 50, N = 720, K = 2048, fp32 residual epilogue with the
    # next norm's bf16 operand and statistics) timed alone, against the sustained bf16 peak (these
    # GEMMs run inside a long step)
    fn, cargs = find_call(p.progs["denoise"], "s0.0.down")
    gms = time_call(fn, cargs)
    Mg, Ng, Kg = batch * s.chunk, s.exp_dim, s.exp_mlp
    gplan = plans.get("s0.0.down")
    gname = ("gemm_pair_kernel<%d,0,0>" % gplan[1] if gplan and gplan[4] & 8 else
             "gemm_persistent_kernel<%d,0,0>" % gplan[1] if gplan else "library pick")  # fmt: skip
    gbytes = Mg * Kg * 2 + Ng * Kg * 2 + Mg * Ng * (4 + 4 + 2)  # x, W, residual in/out, bf16 copy
    roof_gemm = {"kernel": f"{gname} s0.0.down (M={Mg}, N={Ng}, K={Kg}, bf16, residual + norm operand)",
                 "bound": "tensor", "achieved": 2.0 * Mg * Ng * Kg / (gms * 1e-3) / 1e12,
                 "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s", "ms": gms, "bytes": gbytes,
                 "traffic": profile_traffic("exp.down/" + gname.split("<")[0]),
                 "peak_source": f"{src} bf16 dense, sustained"}  # fmt: skip
    roof_gemm["frac"] = roof_gemm["achieved"] / roof_gemm["peak"]
    launches = eng.launches()
    del eng
    torch.cuda.empty_cache()

    # ---- batch-1 latency: bf16, one CUDA graph per chunk, host in/out (rank 0)
    lat = None
    if rank == 0 and args.latency_chunks > 0:
        e1b = Engine(b, device=dev, warmup=3, pdl=args.pdl, compile="autotune")
        o0 = observations(b, range(4))
        for i in range(5):
            e1b.infer(*o0[i % 4])
        e1b.timing.history.clear()
        for i in range(args.latency_chunks):
            if i == 0:  # one chunk in its own range, for a launch list of the batch-1 chunk
                with torch.cuda.nvtx.range("latency_chunk"):
                    e1b.infer(o0[i % 4][0], o0[i % 4][1])
            else:
                e1b.infer(o0[i % 4][0], o0[i % 4][1])
        sm = e1b.timing.summary()
        errs = None
        if gpath.exists():
            g = np.load(gpath)
            errs = max(float(np.abs(e1b.infer(*o0[i]) - g["actions"][i]).max()) for i in range(4))
        prof = e1b.profile(*o0[0][:2])
        H, E, F, QD, KV, Lp = s.chunk, s.exp_dim, s.exp_mlp, s.q_dim, s.kv_dim, s.prefix_len
        traffic = None  # DRAM bytes per launch from a committed ncu summary, where there is one
        if e1b.path.xs is not None:
            # the fused expert step: every expert weight once per step, plus the K/V rows attention reads
            fn, cargs = find_call(e1b.path.progs["denoise"], "s0.expert_layers")
            gms = time_call(fn, cargs)
            byts = 0
            for i in range(s.n_layers):
                self_attn = s.is_self_attn(i)
                byts += ((QD + 2 * KV) if self_attn else QD) * E * 2 + E * QD * 2 + 2 * F * E * 2 + E * F * 2
                byts += (Lp + H if self_attn else Lp) * KV * 2 * 2
            kname = f"expert_step_kernel s0.expert_layers ({s.n_layers} layers, one launch)"
        elif e1b.path.mlp_fused:
            # the fused SwiGLU block: gate/up and down weights, the token rows in, the residual rows
            # in and out
            fn, cargs = find_call(e1b.path.progs["denoise"], "s0.0.mlp")
            gms = time_call(fn, cargs)
            byts = 2 * F * E * 2 + E * F * 2 + H * E * 2 + 2 * H * E * 4
            kname = "mlp_kernel s0.0.mlp (M=50, gate/up + down fused)"
            traffic = profile_traffic("exp.mlp/mlp_kernel")
        else:
            fn, cargs = find_call(e1b.path.progs["denoise"], "s0.0.gate_up")
            gms = time_call(fn, cargs)
            byts = 2 * F * E * 2 + H * E * 2 + H * F * 2
            kname = "gemm_tc_kernel<swap,dual> s0.0.gate_up (M=50)"
        lat = {"p50_ms": sm["p50_ms"], "p99_ms": sm["p99_ms"], "n": sm["n"],
               "stages_ms": prof, "launches_per_chunk": e1b.launches(), "max_err_rad": errs,
               "config": "configs[3]: batch 1, bf16, one CUDA graph, host frames in -> actions out",
               "roofline_expert": {"kernel": kname, "bound": "hbm", "achieved": byts / (gms * 1e-3) / 1e9,
                                   "bytes": byts, "peak": pk["hbm_gbs"], "unit": "GB/s", "ms": gms, "traffic": traffic,
                                   "frac": byts / (gms * 1e-3) / 1e9 / pk["hbm_gbs"]}}  # fmt: skip
        del e1b
    if world > 1:
        dist.barrier()

    if rank == 0:
        cpu = cpu_chunks_per_s() if world == 1 and not args.no_cpu else None
        ref_gpu = reference_gpu(args.reference_gpu_chunks) if world == 1 and args.reference_gpu_chunks > 0 else None
        line = {
            "metric": metric_name(batch), "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None, "dtype": "int8+bf16", "data": "synthetic",
            "config": arm_config(world, batch),
            "e2e": {"value": throughput(world, batch, e2e_ms), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "gpu_launches": launches * args.steps,
            "pdl": bool(args.pdl),
            "max_err_rad": err,
            "int8_parity": parity,
            "roofline": roof,
            "roofline_attention": roof_attn,
            "roofline_gemm_bf16": roof_gemm,
            "latency": lat,
            "clocks": clk,
            "cpu_baseline": cpu,
            "reference_gpu": ref_gpu,
        }  # fmt: skip
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ------------------------------------------------------------------------------ profiling cases
# Single kernels on the model's real shapes with seeded random operands, for ncu captures
# (`python bench.py --profile-case NAME`): each case launches its kernel --reps times after the
# producer of its inputs, as in the engine, so `ncu -k regex:<kernel> -s 2 -c 1` captures a warm
# launch. Nothing is checked: the kernels' parity is the tests' business.
def _rnd(g, *shape, scale=1.0, dtype=None):
    import torch

    return (torch.randn(*shape, device="cuda", generator=g) * scale).to(dtype or torch.float32)


def case_mlp(g, reps: int) -> None:
    """so101_mlp: the expert's SwiGLU block at one observation (50 rows, 720 -> 2048 -> 720)."""
    import torch

    from so101_smolvla_edge_b200.ops import mlp, rms_stats

    e = _rnd(g, 50, 720)
    x16 = torch.empty(50, 720, device="cuda", dtype=torch.bfloat16)
    ss = torch.zeros(50, 64, device="cuda")
    w_gu = _rnd(g, 4096, 720, scale=0.03, dtype=torch.bfloat16)
    w_d = _rnd(g, 720, 2048, scale=0.02, dtype=torch.bfloat16)
    nw = torch.ones(720, device="cuda")
    for _ in range(reps):
        rms_stats(e, x16, ss, nw)
        mlp(x16, w_gu, w_d, e, residual=e, rms=(ss, 1, 1e-5), y16=x16, y16_scale=nw, stat_ss=ss)


def case_attention_o(g, reps: int) -> None:
    """so101_attention_o: an expert self-attention layer at one observation (50 queries, 291 keys)."""
    import torch

    from so101_smolvla_edge_b200.ops import attention_o, rms_stats

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
    """so101_gemm: vision fc2 plus residual at one observation (3072 rows, K = 3072)."""
    import torch

    from so101_smolvla_edge_b200.ops import linear

    x = _rnd(g, 3072, 3072, dtype=torch.bfloat16)
    w = _rnd(g, 768, 3072, scale=0.02, dtype=torch.bfloat16)
    r = _rnd(g, 3072, 768)
    for _ in range(reps):
        linear(x, w, residual=r, out=r)


def case_expert_down64(g, reps: int) -> None:
    """so101_gemm: the batched expert's down projection at 64 observations (3200 rows, 2048 -> 720)
    with the residual epilogue that writes the next norm's bf16 operand and statistics, on the
    192-wide CTA-pair plan the engine's autotune picks for it."""
    import torch

    from so101_smolvla_edge_b200.ops import linear

    x = _rnd(g, 3200, 2048, dtype=torch.bfloat16)
    w = _rnd(g, 720, 2048, scale=0.02, dtype=torch.bfloat16)
    e = _rnd(g, 3200, 720)
    x16 = torch.empty(3200, 720, device="cuda", dtype=torch.bfloat16)
    ss = torch.zeros(3200, 64, device="cuda")
    nw = torch.ones(720, device="cuda")
    for _ in range(reps):
        linear(x, w, residual=e, out=e, stat=(ss, x16, nw), config=(0, 192, 1, 0, 8))


def case_gqa_prefix(g, reps: int) -> None:
    """so101_attention: the prefix's grouped-query attention at 16 observations (241 rows, 15 / 5
    heads, prefix-LM mask, RoPE), the masked tcgen05 kernel's case."""
    import torch

    from so101_smolvla_edge_b200.ops import attention

    qkv = _rnd(g, 16, 241, 1600, dtype=torch.bfloat16)
    k = _rnd(g, 16, 241, 320, dtype=torch.bfloat16)
    cs = torch.rand(241, 32, device="cuda", generator=g)
    out = torch.empty(16, 241, 960, dtype=torch.bfloat16, device="cuda")
    for _ in range(reps):
        attention(qkv[:, :, :960], k, qkv[:, :, 1280:], 15, 5, cos=cs, sin=cs, causal_from=240, out=out)


PROFILE_CASES = {"mlp": case_mlp, "attention_o": case_attention_o, "fc2": case_fc2,
                 "expert_down64": case_expert_down64, "gqa_prefix": case_gqa_prefix}  # fmt: skip


def run_profile_case(name: str, reps: int) -> None:
    import torch

    g = torch.Generator(device="cuda").manual_seed(0)
    PROFILE_CASES[name](g, reps)
    torch.cuda.synchronize()
    print(f"{name}: {reps} launches done", flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--latency-chunks", type=int, default=200)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--pdl", type=int, default=1, help="programmatic dependent launch (1 on, 0 off)")
    ap.add_argument("--batch", type=int, default=BATCH,
                    help=f"observations per GPU per step (the metric is quoted at {BATCH}; smaller "
                         "batches are for profiling captures that must stay small)")  # fmt: skip
    ap.add_argument("--reference-gpu-chunks", type=int, default=100,
                    help="chunks per reference GPU engine (0: skip the reference's own GPU paths)")
    ap.add_argument("--reference-gpu", choices=["triton", "torch"], default=None, help=argparse.SUPPRESS)
    ap.add_argument("--profile-case", choices=sorted(PROFILE_CASES), default=None,
                    help="launch one kernel on its real shape --reps times (for ncu captures) and exit")
    ap.add_argument("--reps", type=int, default=4)
    a = ap.parse_args()
    if a.profile_case:
        run_profile_case(a.profile_case, a.reps)
        return
    if a.reference_gpu:
        reference_gpu_probe(a.reference_gpu, a.latency_chunks)
        return
    if a.warmup < 3:
        a.warmup = 3
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
