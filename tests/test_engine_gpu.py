"""The B200 engine end to end against the reference's float32 golden chunks (tests/golden/).

max |action - float32 reference| <= 1e-2 rad for bf16 and for W8A8 int8 vision
Stage parity (image rows, prefix K/V, the first velocity) is checked against the
reference's own intermediates at bf16-level tolerances. Graph replay equals eager replay bit for
bit, as the reference requires of its Triton path (`tests/test_triton_engine.py:33-47`).
"""

from __future__ import annotations

import time

import numpy as np
import pytest
import torch
from conftest import case_bundle, config0_bundle, golden, int8_band_check

from so101_smolvla_edge_b200.bundle import observation

pytestmark = pytest.mark.gpu

ACTION_TOL = 1e-2  # rad, BASELINE north star (bf16 against float32)
INT8_FP32_DRIFT = 1.5  # int8 no further from float32 than 1.5x the reference's own int8 drift
GPU_CASES = ["small_absolute", "small_delta", "small_velocity", "small64_absolute"]


def rel(a, b) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-12))


@pytest.fixture(scope="module")
def config0_engine():
    from so101_smolvla_edge_b200.engine import Engine

    eng = Engine(config0_bundle(), warmup=1)
    yield eng
    del eng
    torch.cuda.empty_cache()


@pytest.mark.parametrize("case", GPU_CASES)
def test_small_bundles_match_reference(case):
    """Every action representation, resize + padding, perturbed norms and biases."""
    from so101_smolvla_edge_b200.engine import Engine

    g = golden(case)
    b = case_bundle(case)
    graph = Engine(b, warmup=1)
    eager = Engine(b, warmup=1, cuda_graph=False)
    for seed in (0, 1):
        images, state, noise = observation(b, seed)
        a = graph.infer(images, state, noise)
        e = eager.infer(images, state, noise)
        assert np.array_equal(a, e), "graph replay differs from eager"
        want = g[f"s{seed}.actions"]
        err = np.abs(a - want).max()
        assert err <= ACTION_TOL * max(1.0, np.abs(want).max()), (case, seed, err)


def test_config0_stages_match_reference(config0_engine):
    """configs[0] seed 0: image rows, layer-0 keys/values, layer-1 expert keys, first velocity."""
    g = golden("config0")
    eng = config0_engine
    b = eng.bundle
    images, state, noise = observation(b, 0)
    eng._stage([images], [state], [noise])
    p = eng.path
    p.run("vision")
    torch.cuda.synchronize()
    L, C_ = eng.spec.prefix_len, eng.spec.n_cams
    img_rows = p.x_pre[: C_ * eng.spec.img_tokens].cpu().numpy()
    assert rel(img_rows, g["s0.img_rows"]) < 2e-2, rel(img_rows, g["s0.img_rows"])
    p.run("prefix")
    torch.cuda.synchronize()
    k0 = p.ck[0][0, :L].float().cpu().numpy()
    v0 = p.cv[0][0, :L].float().cpu().numpy()
    kx1 = p.kx[1][0].float().cpu().numpy()
    assert rel(k0, g["s0.k_0"]) < 2e-2, rel(k0, g["s0.k_0"])
    assert rel(v0, g["s0.v_0"]) < 2e-2, rel(v0, g["s0.v_0"])
    assert rel(kx1, g["s0.kx_1"]) < 3e-2, rel(kx1, g["s0.kx_1"])
    v = eng.step(0)[0].cpu().numpy()
    assert rel(v, g["s0.v0"]) < 3e-2, rel(v, g["s0.v0"])


def test_backend_seams_match_reference(config0_engine):
    """The reference's backend seams on the B200 path, fed the reference's own intermediates:
    `encode_images(px)` (TrtVision) gives its image rows, `prefix(rows)` (TritonPath.prefix) its
    layer-0 keys/values and layer-1 expert keys, `velocity(x_t, time_proj)` (TritonPath.velocity)
    its first velocity."""
    from oracle.smolvla_fp32 import Oracle

    g = golden("config0")
    eng = config0_engine
    b, p, s = eng.bundle, eng.path, eng.spec
    images, state, noise = observation(b, 0)
    o = Oracle(b)
    px = o.preprocess(images)
    rows = p.encode_images(px.cuda())
    torch.cuda.synchronize()
    assert rel(rows.cpu().numpy(), g["s0.img_rows"]) < 2e-2
    prefix_rows = o.prefix_rows(torch.from_numpy(g["s0.img_rows"]), torch.from_numpy(state))
    p.prefix(prefix_rows.cuda())
    torch.cuda.synchronize()
    L = s.prefix_len
    assert rel(p.ck[0][0, :L].float().cpu().numpy(), g["s0.k_0"]) < 2e-2
    assert rel(p.cv[0][0, :L].float().cpu().numpy(), g["s0.v_0"]) < 2e-2
    assert rel(p.kx[1][0].float().cpu().numpy(), g["s0.kx_1"]) < 3e-2
    x_t = torch.from_numpy(noise).reshape(1, s.chunk, s.max_action).cuda()
    v = p.velocity(x_t, p.w["time_proj"][0].view(1, 1, -1))
    torch.cuda.synchronize()
    assert v.shape == (1, s.chunk, s.max_action)
    assert rel(v[0].cpu().numpy(), g["s0.v0"]) < 3e-2, rel(v[0].cpu().numpy(), g["s0.v0"])


def test_fused_patch_embedding_equals_separate_preprocessing(config0_engine, monkeypatch):
    """With SO101_FUSED_PATCH=1 the engine's frames go straight into the patch GEMM
    (so101_patch_embed, no patch rows in global memory); by default it launches so101_preprocess
    and the patch GEMM. The image rows agree bit for bit when the patch GEMM does not split K."""
    from so101_smolvla_edge_b200.engine import Engine

    assert not config0_engine.path.fused_patch()  # opt-in
    monkeypatch.setenv("SO101_FUSED_PATCH", "1")
    e1 = Engine(config0_bundle(), warmup=1)
    assert e1.path.fused_patch()
    names = [c[0] for c in e1.path.progs["vision"].calls]
    assert "patch_embed" in names and "preprocess" not in names and "patch" not in names
    images, state, noise = observation(e1.bundle, 2)
    rows = []
    for eng in (e1, config0_engine):
        eng._stage([images], [state], [noise])
        eng._vision()
        torch.cuda.synchronize()
        rows.append(eng.path.xv.clone())
    assert torch.equal(rows[0], rows[1])  # the library's pick for 3072 x 768 x 768 does not split K
    del e1
    torch.cuda.empty_cache()


def test_second_engine_reuses_packed_weights(config0_engine):
    """A second Engine on the same bundle and device skips the upload and packing (the packed
    set is shared) and gives the same chunk bit for bit."""
    from so101_smolvla_edge_b200.engine import Engine
    from so101_smolvla_edge_b200.path import Packed

    n0 = Packed.packs
    t0 = time.perf_counter()
    e2 = Engine(config0_bundle(), warmup=1)
    build_s = time.perf_counter() - t0
    assert Packed.packs == n0 and e2.path.packed is config0_engine.path.packed, build_s
    images, state, noise = observation(e2.bundle, 0)
    assert np.array_equal(e2.infer(images, state, noise), config0_engine.infer(images, state, noise))
    del e2
    torch.cuda.empty_cache()


def test_config0_actions_within_north_star(config0_engine):
    """configs[0] (3 x 512^2 cameras, 241-token prefix, 10 steps): every golden seed within
    1e-2 rad of the reference's float32 chunk; replays are deterministic."""
    g = golden("config0")
    eng = config0_engine
    b = eng.bundle
    errs = []
    for seed in range(g["actions"].shape[0]):
        images, state, noise = observation(b, seed)
        a = eng.infer(images, state, noise)
        errs.append(np.abs(a - g["actions"][seed]).max())
        assert np.array_equal(a, eng.infer(images, state, noise))
    assert max(errs) <= ACTION_TOL, errs


def test_batched_matches_reference_and_single():
    """infer_batch over B observations: every chunk within the action tolerance of the reference's
    float32 chunk (the seeds with goldens) and of the single-chunk engine. The batched GEMMs have
    B times the rows and may tile differently (rows on the MMA M or N side, other K splits), so
    the two engines agree to rounding, not bit for bit."""
    from so101_smolvla_edge_b200.engine import Engine

    case = "small_absolute"
    g = golden(case)
    b = case_bundle(case)
    obs = [observation(b, s) for s in range(3)]
    single = Engine(b, warmup=1)
    batched = Engine(b, warmup=1, batch=3)
    got = batched.infer_batch([o[0] for o in obs], [o[1] for o in obs], [o[2] for o in obs])
    for i, (images, state, noise) in enumerate(obs):
        want = single.infer(images, state, noise)
        scale = max(1.0, np.abs(want).max())
        assert np.abs(got[i] - want).max() <= ACTION_TOL * scale, i
        if f"s{i}.actions" in g:
            ref = g[f"s{i}.actions"]
            assert np.abs(got[i] - ref).max() <= ACTION_TOL * max(1.0, np.abs(ref).max()), i


def test_infer_stream_equals_infer_batch():
    """infer_stream (the next batch staged on a copy stream while the current graph runs) yields,
    batch by batch, the same bits as infer_batch on the same inputs: four batches that cycle
    both pinned buffer sets, given noise and device-drawn noise (the same generator draws in the
    same order), and the engine is still right for infer_batch afterwards."""
    from so101_smolvla_edge_b200.engine import Engine

    b = case_bundle("small_absolute")
    eng = Engine(b, warmup=1, batch=3)
    batches = []
    for k in range(4):
        obs = [observation(b, 3 * k + s) for s in range(3)]
        noises = [o[2] for o in obs] if k != 2 else None
        batches.append(([o[0] for o in obs], [o[1] for o in obs], noises))
    torch.manual_seed(0)
    want = [eng.infer_batch(*bt) if bt[2] is not None else eng.infer_batch(bt[0], bt[1]) for bt in batches]
    torch.manual_seed(0)
    got = list(eng.infer_stream([bt if bt[2] is not None else bt[:2] for bt in batches]))
    assert len(got) == len(want)
    for k, (g_, w_) in enumerate(zip(got, want, strict=True)):
        assert np.array_equal(g_, w_), k
    assert np.array_equal(eng.infer_batch(*batches[0]), want[0])
    del eng
    torch.cuda.empty_cache()


def _int8_check(g, a, scale):
    """W8A8 parity on a small bundle: the int8 chunk matches the reference's own int8 chunk (its
    fake-quant arithmetic, `tests/test_ov_engine.py:227-236`) within the action tolerance, and
    drifts from float32 no further than 1.5x the reference's own int8 drift (the reference's
    criterion for its Triton path against its torch path, `tests/test_triton_engine.py:44-47`)."""
    ref_drift = np.abs(g["actions_int8"] - g["actions_fp32"]).max()
    err_int8 = np.abs(a - g["actions_int8"]).max()
    err_fp32 = np.abs(a - g["actions_fp32"]).max()
    assert err_int8 <= ACTION_TOL * scale, (err_int8, ref_drift)
    assert err_fp32 <= INT8_FP32_DRIFT * ref_drift + 1e-3 * scale, (err_fp32, ref_drift)


def test_int8_vision_small_matches_fake_quant_oracle():
    """W8A8 vision with the golden clips on the small bundle."""
    from so101_smolvla_edge_b200.engine import Engine

    g = golden("int8_small_absolute")
    b = case_bundle("small_absolute")
    clip = dict(zip(g["clip_names"].tolist(), g["clip_values"].tolist(), strict=True))
    eng = Engine(b, warmup=1, trt_precision="int8", act_clip=clip)
    images, state, noise = observation(b, 0)
    a = eng.infer(images, state, noise)
    _int8_check(g, a, max(1.0, np.abs(g["actions_int8"]).max()))


def test_int8_vision_config0():
    """configs[4]'s numerics at batch 1: W8A8 SigLIP with the reference's calibration (32 seeded
    observations, max |x| per linear), bf16 prefix and expert, every golden seed."""
    from so101_smolvla_edge_b200.engine import Engine

    g = golden("int8_config0")
    b = config0_bundle()
    clip = dict(zip(g["clip_names"].tolist(), g["clip_values"].tolist(), strict=True))
    eng = Engine(b, warmup=1, trt_precision="int8", act_clip=clip)
    acts = np.stack([eng.infer(*observation(b, s)) for s in range(g["actions_int8"].shape[0])])
    int8_band_check(g, acts)
    # the vision stage alone: seed 0's image rows against the reference's int8 rows, as far from
    # them as the reference's own one-ulp runs are (max) and no more than 1.25x on average
    images, state, noise = observation(b, 0)
    eng._stage([images], [state], [noise])
    eng._vision()
    torch.cuda.synchronize()
    rows = eng.path.x_pre[: g["s0.img_rows_int8"].shape[0]].cpu().numpy()
    r0, ru = g["s0.img_rows_int8"], g["s0.img_rows_int8_ulp"]
    assert np.abs(rows - r0).max() <= 1.25 * np.abs(ru - r0[None]).max()
    assert np.abs(rows - r0).mean() <= 1.25 * np.abs(ru - r0[None]).mean()
    del eng
    torch.cuda.empty_cache()


def test_int8_timed_configuration_config0():
    """The configuration bench.py times: batch 64, compile="autotune", W8A8 with the
    reference's calibration clips; observations 0..3 are the golden seeds."""
    from so101_smolvla_edge_b200.engine import Engine

    g = golden("int8_config0")
    b = config0_bundle()
    clip = dict(zip(g["clip_names"].tolist(), g["clip_values"].tolist(), strict=True))
    eng = Engine(b, batch=64, warmup=1, trt_precision="int8", act_clip=clip, compile="autotune")
    obs = [observation(b, s) for s in range(64)]
    acts = eng.infer_batch([o[0] for o in obs], [o[1] for o in obs], [o[2] for o in obs])
    int8_band_check(g, acts)
    del eng
    torch.cuda.empty_cache()


def test_calibration_matches_reference_clips():
    """Engine.calibrate over the reference's 32 calibration frames gives its clips (bf16
    activations, so within a few bf16 ulps of the float32 maxima)."""
    from so101_smolvla_edge_b200.engine import Engine

    g = golden("int8_small_absolute")
    b = case_bundle("small_absolute")
    eng = Engine(b, warmup=0, cuda_graph=False)
    clip = eng.calibrate([observation(b, 1000 + i)[0] for i in range(32)])
    want = dict(zip(g["clip_names"].tolist(), g["clip_values"].tolist(), strict=True))
    assert sorted(clip) == sorted(want)
    for k, v in want.items():
        assert abs(clip[k] - v) <= 2e-2 * v, (k, clip[k], v)


def test_unsupported_models_raise():
    """No fallback: a head size the kernels cannot index raises (the reference would fall back
    to torch kernels with a log line, `tests/test_triton_engine.py:90-99`)."""
    from so101_smolvla_edge_b200.engine import Engine

    with pytest.raises(ValueError):
        Engine(case_bundle("tiny_absolute"), warmup=0)
    with pytest.raises(ValueError):
        Engine(case_bundle("small_absolute"), dtype="fp32", warmup=0)


@pytest.mark.parametrize("case", ["small64_absolute", "config0"])
def test_fused_expert_step_matches_per_op_path(case):
    """The persistent expert-step kernel (one cooperative launch per denoising step for all expert
    layers) against the per-op launch chain and the reference's float32 chunk. Both are within the
    action tolerance of the reference; they differ in the RMSNorm statistics' summation order and
    the GEMMs' K splits, so they agree to rounding. Replays of the fused path are deterministic."""
    from so101_smolvla_edge_b200.engine import Engine

    g = golden(case)
    b = config0_bundle() if case == "config0" else case_bundle(case)
    fused = Engine(b, warmup=1, expert_step="fused")
    per_op = Engine(b, warmup=1, expert_step="ops")
    assert fused.path.xs is not None and per_op.path.xs is None
    assert fused.launches() < per_op.launches()
    for seed in (0, 1):
        images, state, noise = observation(b, seed)
        a = fused.infer(images, state, noise)
        assert np.array_equal(a, fused.infer(images, state, noise)), "fused replays differ"
        o = per_op.infer(images, state, noise)
        ref = g["actions"][seed] if case == "config0" else g[f"s{seed}.actions"]
        scale = max(1.0, np.abs(ref).max())
        assert np.abs(a - ref).max() <= ACTION_TOL * scale, (seed, np.abs(a - ref).max())
        assert np.abs(a - o).max() <= ACTION_TOL * scale, (seed, np.abs(a - o).max())
    del fused, per_op
    torch.cuda.empty_cache()


def test_bounded_wait_times_out_and_recovers():
    """A device wait that can never be met ends in SO101_ERR_TIMEOUT, not a hang. The persistent
    expert step's test hook keeps one CTA from arriving at the first grid barrier; with the wait
    bound cut to 50 ms every other CTA gives up, records the timeout, lets its weight copies land,
    frees its TMEM and returns. Nothing traps or faults: the context stays usable, and after the
    status is cleared the next chunk is bit-identical to one computed before."""
    from so101_smolvla_edge_b200 import _lib as L
    from so101_smolvla_edge_b200.engine import Engine

    lib = L.lib()
    b = case_bundle("small64_absolute")
    eng = Engine(b, warmup=1, expert_step="fused", cuda_graph=False)  # hooks reach eager launches
    images, state, noise = observation(b, 0)
    want = eng.infer(images, state, noise)
    assert lib.so101_device_status() == L.OK
    try:
        L.check(lib.so101_expert_step_test_hooks(50_000_000, 3), "test hooks")
        t0 = time.perf_counter()
        eng.infer(images, state, noise)  # every denoising step's launch runs into the bound
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        L.check(lib.so101_expert_step_test_hooks(0, -1), "test hooks")
    assert lib.so101_device_status() == L.ERR_TIMEOUT
    assert elapsed < 0.05 * b.spec.n_steps + 5.0
    L.check(lib.so101_clear_device_status(), "clear status")
    assert lib.so101_device_status() == L.OK
    got = eng.infer(images, state, noise)
    torch.cuda.synchronize()
    assert np.array_equal(got, want)
    assert lib.so101_device_status() == L.OK
    del eng
    torch.cuda.empty_cache()


@pytest.mark.parametrize("attn_o,mlp", [("all", "1"), ("cross", "1"), ("0", "0")])
def test_fused_expert_blocks_match_reference(attn_o, mlp, monkeypatch):
    """configs[0] with the expert layers' attention + output projection (so101_attention_o, on all
    layers, on the cross layers or off) and SwiGLU blocks (so101_mlp, on or off) fused: every
    combination stays within the action tolerance of the reference's float32 chunk, replays bit
    for bit, and fusing removes launches."""
    from so101_smolvla_edge_b200.engine import Engine

    monkeypatch.setenv("SO101_ATTN_O", attn_o)
    monkeypatch.setenv("SO101_FUSED_MLP", mlp)
    g = golden("config0")
    b = config0_bundle()
    eng = Engine(b, warmup=1)
    s = eng.path.spec
    want_o = {"all": s.n_layers, "cross": sum(not s.is_self_attn(i) for i in range(s.n_layers)), "0": 0}[attn_o]
    assert len(eng.path.attn_o_layers) == want_o and eng.path.mlp_fused == (mlp == "1")
    images, state, noise = observation(b, 0)
    a = eng.infer(images, state, noise)
    assert np.array_equal(a, eng.infer(images, state, noise))
    assert np.abs(a - g["actions"][0]).max() <= ACTION_TOL
    del eng
    torch.cuda.empty_cache()


def test_autotuned_engine_matches_reference():
    """compile="autotune" (the reference's autotuned GEMMs) times the GEMM plans of every large
    GEMM and rebuilds the programs with the fastest: configs[0]'s vision GEMMs (3072 rows) are
    tuned, the chunk stays within the action tolerance of the reference's float32 chunk and within
    rounding of the untuned engine (the plans never split K; only the statistics' summation order
    of a re-tiled residual GEMM can move)."""
    from so101_smolvla_edge_b200.engine import Engine

    g = golden("config0")
    b = config0_bundle()
    tuned = Engine(b, warmup=1, compile="autotune")
    assert tuned.tuning and all(v["ms"] for v in tuned.tuning.values())
    images, state, noise = observation(b, 0)
    a = tuned.infer(images, state, noise)
    assert np.array_equal(a, tuned.infer(images, state, noise))
    assert np.abs(a - g["actions"][0]).max() <= ACTION_TOL
    del tuned
    torch.cuda.empty_cache()
