"""The C ABI library without a GPU: it loads, exports every entry point the header declares, and
rejects bad arguments on the host before touching the device (no compute call is made here)."""

from __future__ import annotations

import ctypes as C

import pytest

from so101_smolvla_edge_b200 import _lib as L


@pytest.fixture(scope="module")
def lib():
    return L.lib()


def test_library_loads_and_exports_every_header_symbol(lib):
    names = L.header_symbols()
    assert len(names) == 31
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert lib.so101_version().decode().endswith("sm_100a")
    assert lib.so101_last_error() == b""


def test_bindings_cover_the_header():
    """Every declared entry point has a ctypes signature (or is bound where it is used)."""
    bound = set(L.SIGNATURES) | {"so101_version", "so101_last_error", "so101_gemm_static"}
    assert set(L.header_symbols()) <= bound


def test_status_codes_match_the_header():
    text = L.HEADER.read_text()
    for name, value in (("SO101_OK", L.OK), ("SO101_ERR_ARG", L.ERR_ARG), ("SO101_ERR_LAUNCH", L.ERR_LAUNCH),
                        ("SO101_ERR_WORKSPACE", L.ERR_WORKSPACE), ("SO101_ERR_TIMEOUT", L.ERR_TIMEOUT),
                        ("SO101_BF16", L.BF16), ("SO101_F32", L.F32), ("SO101_I8", L.I8),
                        ("SO101_EPI_SILU_GATE", L.EPI_SILU_GATE)):  # fmt: skip
        assert f"#define {name} {value}" in text, name


def test_gemm_rejects_bad_arguments_on_the_host(lib):
    epi = L.Epilogue(epilogue=L.EPI_NONE, out_scale=1.0)
    fake = 1 << 20  # never dereferenced: every call below fails its host-side checks
    rc = lib.so101_gemm(L.BF16, None, 64, fake, 64, fake, 64, L.BF16, 8, 8, 64, C.byref(epi), None,
                        None, 0, None, 0, None)  # fmt: skip
    assert rc == L.ERR_ARG  # null x
    rc = lib.so101_gemm(L.BF16, fake, 100, fake, 100, fake, 8, L.BF16, 8, 8, 100, C.byref(epi), None,
                        None, 0, None, 0, None)  # fmt: skip
    assert rc == L.ERR_ARG  # K * 2 bytes not a multiple of 16
    rc = lib.so101_gemm(L.BF16, fake + 8, 64, fake, 64, fake, 64, L.BF16, 8, 8, 64, C.byref(epi), None,
                        None, 0, None, 0, None)  # fmt: skip
    assert rc == L.ERR_ARG  # x not 16-byte aligned
    bad = L.Epilogue(epilogue=7, out_scale=1.0)
    rc = lib.so101_gemm(L.BF16, fake, 64, fake, 64, fake, 64, L.BF16, 8, 8, 64, C.byref(bad), None,
                        None, 0, None, 0, None)  # fmt: skip
    assert rc == L.ERR_ARG  # unknown epilogue
    q = L.Epilogue(epilogue=L.EPI_NONE, out_scale=1.0)
    rc = lib.so101_gemm(L.I8, fake, 64, fake, 64, fake, 64, L.BF16, 8, 8, 64, C.byref(q), None,
                        None, 0, None, 0, None)  # fmt: skip
    assert rc == L.ERR_ARG  # int8 operands without weight scales


def test_split_k_plans_report_their_workspace(lib):
    """The global-workspace split-K plan asks for partials and tickets; the cluster plan for none."""
    need, tick = C.c_int64(), C.c_int64()
    glob = L.GemmConfig(1, 64, 4, 0, L.GEMM_GLOBAL_SPLITK)
    assert lib.so101_gemm_workspace(L.BF16, 50, 720, 2048, L.EPI_NONE, C.byref(glob), C.byref(need),
                                    C.byref(tick)) == L.OK  # fmt: skip
    assert need.value == 6 * 4 * 64 * 128 * 4 and tick.value == 6
    clus = L.GemmConfig(1, 64, 4, 0, 0)
    assert lib.so101_gemm_workspace(L.BF16, 50, 720, 2048, L.EPI_NONE, C.byref(clus), C.byref(need),
                                    C.byref(tick)) == L.OK  # fmt: skip
    assert need.value == 0 and tick.value == 0
    bad = L.GemmConfig(1, 96, 1, 0, 0)  # 96 is not a swap tile width
    assert lib.so101_gemm_workspace(L.BF16, 50, 720, 2048, L.EPI_NONE, C.byref(bad), C.byref(need),
                                    C.byref(tick)) == L.ERR_ARG  # fmt: skip


def test_gemm_pick_heuristic(lib):
    """Few token rows stream weights (swap tiling in 32-token tiles, split over a cluster of at
    most 8); many rows put tokens on the MMA M side with one split."""
    cfg = L.GemmConfig()
    assert lib.so101_gemm_pick(L.BF16, 50, 4096, 720, L.EPI_SILU_GATE, C.byref(cfg)) == L.OK
    assert cfg.swap == 1 and cfg.bn == 32 and 1 <= cfg.splits <= 8
    assert lib.so101_gemm_pick(L.I8, 196608, 3072, 768, L.EPI_GELU, C.byref(cfg)) == L.OK
    assert cfg.swap == 0 and cfg.bn == 256 and cfg.splits == 1


def test_other_entry_points_validate_arguments(lib):
    fake = 1 << 20
    assert lib.so101_attention(fake, 64, fake, 64, fake, 64, fake, 64, L.BF16, 0.0, 10, 10, 4, 3, 64,
                               10, 0, None, None, 1, 0, 0, 0, 0, None) == L.ERR_ARG  # nq % nkv
    assert lib.so101_attention(fake, 64, fake, 64, fake, 64, fake, 64, L.BF16, 0.0, 10, 10, 4, 2, 48,
                               10, 0, None, None, 1, 0, 0, 0, 0, None) == L.ERR_ARG  # head_dim 48
    assert lib.so101_rms_norm(fake, 64, L.I8, fake, fake, 64, L.BF16, 4, 64, 1e-5, None) == L.ERR_ARG
    assert lib.so101_layer_norm(fake, 64, fake, fake, fake, 64, L.I8, 0.0, 4, 64, 1e-6, 1, 0, None) == L.ERR_ARG
    assert lib.so101_preprocess(fake, 1, 10, 10, 10, 10, 100, 16, fake, L.BF16, 0.0, None) == L.ERR_ARG
    assert lib.so101_linear_f32(fake, 3, fake, 3, None, None, fake, 3, 2, 3, 3, 0, None) == L.ERR_ARG
    assert lib.so101_finish(fake, 8, fake, 6, fake, fake, fake, fake, fake, fake, fake, 6, 10, 3, 1, None) == L.ERR_ARG


def test_fused_expert_entry_points_validate_arguments(lib):
    """so101_attention_o and so101_mlp refuse, before touching the GPU, what their kernels cannot
    run: head_dim other than 64, more heads than a cluster holds, an output width that is not a
    multiple of 4, more than 64 rows per observation, a hidden width that is not a multiple of 128
    or needs more than 16 CTAs, unaligned operands."""
    fake, S = 1 << 20, None

    def attn_o(**kw):
        a = dict(q=fake, ldq=1600, k=fake, ldk=320, v=fake, ldv=320, Lq=50, Lk=291, nq=15, nkv=5, hd=64,
                 causal_from=241, q_offset=241, cos=None, sin=None, batch=1, bq=0, bk=0, bv=0, k_own=None,
                 v_own=None, ld_own=0, b_own=0, own_from=0, k_cos=None, k_sin=None, w_o=fake, ldw=960,
                 n_out=720, y=fake, ldy=720, res=None, ldr=0, y16=None, ld16=0, y16_scale=None, stat=None,
                 stat_ld=0)  # fmt: skip
        a.update(kw)
        return lib.so101_attention_o(*a.values(), S)

    def mlp(**kw):
        a = dict(x=fake, ldx=720, rows=50, batch=1, k=720, rms=None, slots=0, rms_ld=0, eps=1e-5, w_gu=fake,
                 ldw1=720, hidden=2048, w_d=fake, ldw2=2048, n_out=720, y=fake, ldy=720, res=None, ldr=0,
                 y16=None, ld16=0, y16_scale=None, stat=None, stat_ld=0)  # fmt: skip
        a.update(kw)
        return lib.so101_mlp(*a.values(), S)

    for bad in (dict(hd=32, ldk=160, ldv=160), dict(nq=20, nkv=5), dict(n_out=718), dict(nq=15, nkv=4),
                dict(w_o=fake + 8), dict(y=fake + 4), dict(ldw=480), dict(k_own=fake, own_from=10)):  # fmt: skip
        assert attn_o(**bad) == L.ERR_ARG, bad
    for bad in (dict(rows=65), dict(hidden=2000, ldw2=2000), dict(hidden=2176, ldw2=2176), dict(n_out=722),
                dict(x=fake + 8), dict(ldx=700), dict(rms=fake, slots=65, rms_ld=65)):  # fmt: skip
        assert mlp(**bad) == L.ERR_ARG, bad


def test_tune_gemm_candidates():
    """The plan sweep (the counterpart of the reference's scripts/tune_gemm.py) offers the pick,
    weight-streaming swap tiles for few rows (not for int8, which has no swap tiles) and the
    token-tile kernels (one tile per CTA with K splits, persistent, CTA pair) for many rows."""
    from so101_smolvla_edge_b200 import _lib as L
    from so101_smolvla_edge_b200.tune_gemm import SHAPES, candidates

    few = candidates(50, dual=False, int8=False)
    assert few[0] is None and any(c and c[0] == 1 for c in few)
    many = candidates(3072, dual=True, int8=True)
    assert not any(c and c[0] == 1 for c in many)
    assert any(c and c[4] == L.GEMM_PAIR for c in many) and all(c is None or c[1] <= 128 for c in many)
    assert set(SHAPES) == {"expert", "prefix", "vision"}


def test_expert_step_test_hooks_validate(lib):
    """The bounded-wait test hook takes a bound of at most 2 s and a CTA index or -1."""
    assert lib.so101_expert_step_test_hooks(-1, -1) == L.ERR_ARG
    assert lib.so101_expert_step_test_hooks(3_000_000_000, -1) == L.ERR_ARG
    assert lib.so101_expert_step_test_hooks(0, -2) == L.ERR_ARG
    assert lib.so101_expert_step_test_hooks(50_000_000, 3) == L.OK
    assert lib.so101_expert_step_test_hooks(0, -1) == L.OK
