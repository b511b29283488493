"""The CPU oracle against the golden vectors the reference itself produced (tests/golden/).

These pin the oracle: every GPU parity test trusts it only because these pass.
"""

from __future__ import annotations

import numpy as np
import pytest
from conftest import case_bundle, config0_bundle, golden

from so101_smolvla_edge_b200.bundle import observation

SMALL_CASES = ["tiny_absolute", "small_absolute", "small_delta", "small_velocity",
               "small64_absolute"]  # fmt: skip


def _close(got, want, rtol=2e-5, atol=2e-6):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    err = np.abs(got - want).max()
    tol = atol + rtol * np.abs(want).max()
    return err <= tol, (err, tol)


@pytest.mark.parametrize("case", SMALL_CASES)
def test_seeded_bundle_is_the_golden_bundle(case):
    """The seeded generator rebuilds the exact weights the golden run used."""
    g = golden(case)
    assert case_bundle(case).checksum() == str(g["checksum"])


@pytest.mark.parametrize("case", SMALL_CASES)
def test_oracle_matches_reference_small(case):
    """Actions and every intermediate match the reference's float32 engine."""
    from oracle.smolvla_fp32 import Oracle

    g = golden(case)
    b = case_bundle(case)
    o = Oracle(b)
    s = b.spec
    for seed in (0, 1):
        images, state, noise = observation(b, seed)
        r = o.run(images, state, noise, keep=True)
        p = f"s{seed}."
        for key, got in (("img_rows", r["img_rows"]), ("prefix_rows", r["rows"]), ("v0", r["v0"])):
            ok, info = _close(got.numpy(), g[p + key])
            assert ok, (key, info)
        for i in range(s.n_layers):
            for kind in ("k", "v", "kx", "vx"):
                if f"{p}{kind}_{i}" in g:
                    ok, info = _close(r["cache"][kind][i].numpy(), g[f"{p}{kind}_{i}"])
                    assert ok, (kind, i, info)
        ok, info = _close(r["actions"].numpy(), g[p + "actions"], rtol=1e-5, atol=1e-6)
        assert ok, info


def test_config0_bundle_checksum():
    g = golden("config0")
    assert config0_bundle().checksum() == str(g["checksum"])


def test_oracle_matches_reference_config0():
    """BASELINE configs[0] at full size: seed 0 stage by stage, and its actions."""
    from oracle.smolvla_fp32 import Oracle

    g = golden("config0")
    b = config0_bundle()
    o = Oracle(b)
    images, state, noise = observation(b, 0)
    r = o.run(images, state, noise, keep=True)
    for key, got in (("img_rows", r["img_rows"]), ("v0", r["v0"]), ("k_0", r["cache"]["k"][0]),
                     ("v_0", r["cache"]["v"][0]), ("kx_1", r["cache"]["kx"][1]),
                     ("vx_1", r["cache"]["vx"][1])):  # fmt: skip
        ok, info = _close(got.numpy(), g[f"s0.{key}"], rtol=1e-4, atol=1e-5)
        assert ok, (key, info)
    # the reference's own fp32 verify tolerance (`pkg/cli.py:75-122`) is 1e-4 rad
    assert np.abs(r["actions"].numpy() - g["actions"][0]).max() < 1e-4


def test_oracle_int8_matches_reference_small():
    """W8A8 vision with the reference's calibration and fake quant, on the small bundle."""
    from oracle.smolvla_fp32 import Oracle

    g = golden("int8_small_absolute")
    b = case_bundle("small_absolute")
    clip = dict(zip(g["clip_names"].tolist(), g["clip_values"].tolist(), strict=True))
    calib = [observation(b, 1000 + i)[0] for i in range(32)]
    mine = Oracle(b).calibrate(calib)
    mine.pop("patch")
    assert sorted(mine) == sorted(clip)
    for k in clip:
        assert abs(mine[k] - clip[k]) <= 1e-5 * clip[k], k
    images, state, noise = observation(b, 0)
    got = Oracle(b, act_clip=clip).actions(images, state, noise)
    assert np.abs(got - g["actions_int8"]).max() < 1e-4
    # quantized at all, and still near float
    assert np.abs(got - g["actions_fp32"]).max() > 1e-6


def test_reference_int8_chunk_band():
    """The reference's own W8A8 chunk moves by several 1e-3 rad when its quantizers' float32
    inputs move by one ulp (three seeded runs per golden seed, written by make_golden.py from the
    reference itself): the band every int8 parity bar here is stated against."""
    g = golden("int8_config0")
    d = np.abs(g["actions_int8_ulp"] - g["actions_int8"][None]).max(axis=(2, 3))  # (runs, seeds)
    assert d.shape[1] == g["actions_int8"].shape[0] >= 4
    assert (d > 2e-3).all() and d.max() < 2e-2, d


def test_oracle_int8_matches_reference_config0():
    """The float32 restatement with the reference's clips lands inside the reference's own
    reproducibility band on every golden seed (it cannot do better: its float32 sums are
    ordered differently, which is more than one ulp)."""
    from conftest import int8_band_check

    from oracle.smolvla_fp32 import Oracle

    g = golden("int8_config0")
    b = config0_bundle()
    clip = dict(zip(g["clip_names"].tolist(), g["clip_values"].tolist(), strict=True))
    o = Oracle(b, act_clip=clip)
    acts = np.stack([o.actions(*observation(b, s)) for s in range(g["actions_int8"].shape[0])])
    int8_band_check(g, acts)
