"""Host-side logic that runs without a GPU: bundle format, seeded generation, engine option
checks, the tables the engine builds on the host, timing statistics."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch
from conftest import case_bundle

from so101_smolvla_edge_b200.bundle import load_bundle, observation, seeded_bundle, write_bundle
from so101_smolvla_edge_b200.spec import ModelSpec, param_shapes, vision_linear_names
from so101_smolvla_edge_b200.timing import Timing


def test_bundle_round_trip(tmp_path):
    """A written bundle reads back identically, in the reference's directory format."""
    b = case_bundle("small_delta")
    d = write_bundle(b, tmp_path / "b")
    meta = json.loads((d / "meta.json").read_text())
    assert meta["format"] == 1 and meta["action_repr"] == "delta"
    assert set(meta["spec"]) == set(ModelSpec().to_dict())
    b2 = load_bundle(d)
    assert b2.checksum() == b.checksum()
    assert b2.spec == b.spec


def test_bundle_loader_rejects_bad_bundles(tmp_path):
    b = case_bundle("small_absolute")
    d = write_bundle(b, tmp_path / "b")
    meta = json.loads((d / "meta.json").read_text())
    meta["format"] = 2
    (d / "meta.json").write_text(json.dumps(meta))
    with pytest.raises(SystemExit):
        load_bundle(d)
    meta["format"] = 1
    meta["spec"]["text_dim"] += 16
    (d / "meta.json").write_text(json.dumps(meta))
    with pytest.raises(ValueError):
        load_bundle(d)


def test_param_table_matches_the_reference_names():
    s = ModelSpec(lang_len=48)
    shapes = param_shapes(s)
    assert shapes["txt.0.qkv"][0] == (1600, 960)
    assert shapes["exp.0.qkv"][0] == (1600, 720) and "exp.1.q" in shapes and "exp.1.k" in shapes
    assert shapes["conn.w"][0] == (960, 12288)
    assert s.prefix_len == 241
    names = vision_linear_names(s)
    assert names[0] == "patch" and names[-1] == "conn" and len(names) == 4 * 12 + 2


def test_seeded_generation_is_deterministic_and_independent_of_order():
    s = ModelSpec(**{**dict(n_cams=1, image_size=64, vis_dim=64, vis_layers=1, vis_heads=2, vis_mlp=64,
                            text_dim=64, n_layers=2, n_heads=2, n_kv=1, head_dim=32, text_mlp=64,
                            exp_dim=64, exp_mlp=64, chunk=4, lang_len=2)})  # fmt: skip
    a, b = seeded_bundle(s, seed=3), seeded_bundle(s, seed=3)
    assert a.checksum() == b.checksum()
    assert seeded_bundle(s, seed=4).checksum() != a.checksum()
    # baseline statistics: matrices N(0, 0.02), norms 1, biases 0
    assert np.all(a.tensors["txt.0.ln_in"] == 1) and np.all(a.tensors["vis.0.qkv.b"] == 0)
    assert 0.015 < a.tensors["txt.0.qkv"].std() < 0.025


def test_observation_is_seeded():
    b = case_bundle("small_absolute")
    i1, s1, n1 = observation(b, 5)
    i2, s2, n2 = observation(b, 5)
    assert all(np.array_equal(i1[c], i2[c]) for c in i1) and np.array_equal(s1, s2)
    assert n1.shape == (b.spec.chunk, b.spec.max_action)
    assert i1[b.cameras[0]].dtype == np.uint8 and i1[b.cameras[0]].shape == (120, 160, 3)


def test_engine_refuses_to_fall_back_without_cuda():
    """No CPU fallback: the engine raises where the reference would fall back to torch."""
    from so101_smolvla_edge_b200.engine import _resolve_kernels

    s = case_bundle("small_absolute").spec
    with pytest.raises(ValueError):
        _resolve_kernels("torch", torch.device("cuda"), "bf16", s)
    with pytest.raises(ValueError):
        _resolve_kernels("tensorrt", torch.device("cuda"), "bf16", s)
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError):
            _resolve_kernels("auto", torch.device("cpu"), "bf16", s)


def test_unsupported_specs_are_named():
    from so101_smolvla_edge_b200.path import unsupported

    assert unsupported(case_bundle("small_absolute").spec) is None
    assert unsupported(ModelSpec(lang_len=48)) is None
    assert "head_dim" in unsupported(case_bundle("tiny_absolute").spec)
    assert "multiple of 16" in unsupported(ModelSpec(text_dim=968, lang_len=48))


def test_act_clip_file(tmp_path):
    from so101_smolvla_edge_b200.engine import load_act_clip

    (tmp_path / "trt").mkdir()
    (tmp_path / "trt" / "act_clip.json").write_text(json.dumps({"conn": 2.5, "vis.0.qkv": 4}))
    assert load_act_clip(tmp_path, None) == {"conn": 2.5, "vis.0.qkv": 4.0}
    assert load_act_clip(None, {"conn": 1}) == {"conn": 1.0}
    assert load_act_clip(tmp_path / "missing", None) is None


def test_host_tables_match_the_oracle():
    """RoPE tables and the per-step time projection the engine uploads are the oracle's."""
    from oracle.smolvla_fp32 import rope_tables, time_projection
    from so101_smolvla_edge_b200.path import _rope, _time_proj

    b = case_bundle("small64_absolute")
    s = b.spec
    c1, s1 = _rope(torch.arange(17), 64, 10_000.0)
    c2, s2 = rope_tables(torch.arange(17), 64, 10_000.0)
    assert torch.equal(c1, c2) and torch.equal(s1, s2)
    w = {k: torch.from_numpy(v) for k, v in b.tensors.items()}
    tp = _time_proj(s, b.tensors["act.time_in.w_time"], b.tensors["act.time_in.b"])
    assert torch.allclose(tp, time_projection(s, w), rtol=0, atol=1e-6)


def test_timing_summary_matches_the_reference_quantiles():
    t = Timing()
    assert t.summary() == {}
    for v in range(1, 101):
        t.add(float(v))
    s = t.summary()
    assert s["n"] == 100 and s["p50_ms"] == 50.0 and s["p99_ms"] == 99.0 and s["max_ms"] == 100.0
    for _ in range(1000):
        t.add(1.0)
    assert len(t.history) <= 1000


class _StubLib:
    """Stands in for libso101_b200.so: every entry point records its call and returns 0."""

    def __init__(self):
        self.calls: list[tuple[str, tuple]] = []

    def __getattr__(self, name):
        def fn(*args):
            self.calls.append((name, args))
            return 0

        fn.__name__ = name
        return fn


def test_batched_denoise_launches_on_a_stub_library():
    """The denoising step's launch structure, built against a stub library on the CPU: from 1024
    expert rows on, the time MLP's output projection is so101_split_bf16x3 followed by one
    so101_gemm (with the first layer's norm statistics), not so101_linear_f32; self-attention layers
    read the step's own keys and values from the qkv rows (so101_attention_rows) with no rope_kv
    launch into the cache; at one observation the fp32 linear stays."""
    import torch
    from conftest import case_bundle

    from so101_smolvla_edge_b200.path import B200Path

    b = case_bundle("small64_absolute")
    s = b.spec
    many = B200Path(b, torch.device("cpu"), batch=-(-1024 // s.chunk), lib=_StubLib())
    fns = {what: fn.__name__ for what, fn, _ in many.progs["denoise"].calls}
    assert fns["s0.time_split"] == "so101_split_bf16x3" and fns["s0.time_out"] == "so101_gemm"
    assert many.w3_time_out.shape == (s.exp_dim, 3 * s.exp_dim)
    selfs = [i for i in range(s.n_layers) if s.is_self_attn(i)]
    assert selfs and all(fns[f"s0.{i}.attn"] == "so101_attention_rows" for i in selfs)
    assert not any(".rope_kv" in what for what in fns if what.startswith("s"))
    one = B200Path(b, torch.device("cpu"), lib=_StubLib())
    fns1 = {what: fn.__name__ for what, fn, _ in one.progs["denoise"].calls}
    assert fns1["s0.time_out"] == "so101_linear_f32" and "s0.time_split" not in fns1


def test_backend_seams_on_a_stub_library():
    """The reference's backend seams on B200Path, built against a stub library on the CPU:
    `prefix(rows)` (TritonPath.prefix) runs the prefix layers without the prefix-row launch,
    `velocity(x_t, time_proj)` (TritonPath.velocity) one velocity evaluation fed by the caller's
    time projection, `encode_images(px)` (TrtVision.__call__) the vision launches from px."""
    import torch
    from conftest import case_bundle

    from so101_smolvla_edge_b200.path import B200Path

    b = case_bundle("small64_absolute")
    s = b.spec
    lib = _StubLib()
    p = B200Path(b, torch.device("cpu"), lib=lib)
    names = [c[0] for c in p.progs["prefix"].calls]
    assert names[0] == "prefix_tail"

    rows = torch.randn(s.prefix_len, s.text_dim)
    lib.calls.clear()
    p.prefix(rows)
    assert torch.equal(p.x_pre, rows)
    assert len(lib.calls) == len(names) - 1 and lib.calls[0][0] != "so101_prefix_tail"
    with pytest.raises(ValueError):
        p.prefix(torch.zeros(s.prefix_len - 1, s.text_dim))

    x_t = torch.randn(1, s.chunk, s.max_action)
    tp = torch.randn(1, 1, s.exp_dim)
    lib.calls.clear()
    v = p.velocity(x_t, tp)
    assert v.shape == (1, s.chunk, s.max_action) and v.data_ptr() == p.v_buf.data_ptr()
    assert torch.equal(p.x_seam.view_as(x_t), x_t) and torch.equal(p.tp_seam, tp.reshape(-1))
    first, last = lib.calls[0], lib.calls[-1]
    assert first[0] == "so101_linear_f32" and first[1][0] == p.x_seam.data_ptr()
    assert first[1][5] == p.tp_seam.data_ptr()  # the caller's time projection, not the step table
    assert last[0] == "so101_expert_out" and last[1][6] == p.v_buf.data_ptr()

    px = torch.rand(s.n_cams, 3, s.image_size, s.image_size) * 2 - 1
    lib.calls.clear()
    out = p.encode_images(px)
    assert lib.calls[0][0] == "so101_patchify" and lib.calls[0][1][0] == p.px_seam.data_ptr()
    assert "so101_preprocess" not in [c[0] for c in lib.calls]
    assert out.shape == (s.n_cams * s.img_tokens, s.text_dim)
    assert out.data_ptr() == p.x_pre.data_ptr()


def test_packed_weights_are_shared_per_bundle():
    """A second path on the same bundle and device reuses the first one's packed weights (no
    second upload or int8 packing); another int8 selection gets its own set, and the set is
    dropped with the last path that uses it."""
    import gc

    import torch
    from conftest import case_bundle

    from so101_smolvla_edge_b200.path import B200Path, Packed

    b = case_bundle("small64_absolute")
    lib = _StubLib()
    n0 = Packed.packs
    p1 = B200Path(b, torch.device("cpu"), lib=lib)
    p2 = B200Path(b, torch.device("cpu"), lib=lib)
    assert Packed.packs == n0 + 1 and p1.packed is p2.packed
    assert p1.w["txt.0.qkv"].data_ptr() == p2.w["txt.0.qkv"].data_ptr()
    assert p1.w["txt.0.qkv"].dtype == torch.bfloat16
    clip = {"vis.0.fc1": 3.0, "conn": 5.0}
    lib.calls.clear()
    p3 = B200Path(b, torch.device("cpu"), vision_precision="int8", act_clip=clip, lib=lib)
    assert Packed.packs == n0 + 2 and p3.packed is not p1.packed
    assert sorted(p3.wq) == ["conn", "vis.0.fc1"]
    assert [c[0] for c in lib.calls].count("so101_quantize_weight") == 2
    p4 = B200Path(b, torch.device("cpu"), vision_precision="int8", act_clip=clip, lib=lib)
    assert p4.packed is p3.packed and Packed.packs == n0 + 2
    key_count = len(Packed._cache)
    del p3, p4
    gc.collect()
    assert len(Packed._cache) == key_count - 1
