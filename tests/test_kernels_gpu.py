"""Each CUDA kernel against the float32 torch expression it replaces, through the C ABI.

BASELINE configs[1] (GEMM sweep: M in {50, 241, 3072} over the engine's projection shapes, with
each epilogue) and configs[2] (attention: 15 q / 5 kv heads, head_dim 64, RoPE base 1e5, the
prefix-LM mask over 241 tokens, expert self/cross attention over the cached prefix), plus odd
sizes. Tolerances follow the reference's own kernel tests (`tests/test_kernels.py`): GEMM one
output rounding + fp32 accumulation noise, attention 0.02 * max and 2e-3 * mean, RMSNorm 2^-7.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
F = torch.nn.functional


def _p(t):
    return None if t is None else t.data_ptr()


def rnd(*shape, dtype=torch.float32, scale=1.0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, generator=g, device="cuda") * scale).to(dtype)


def gemm_ref(x, w, bias=None, residual=None, silu_gate=False, gelu=False):
    y = x.float() @ w.float().T
    if bias is not None:
        y = y + bias.float()
    if gelu:
        y = F.gelu(y, approximate="tanh")
    if silu_gate:
        g, u = y.chunk(2, dim=-1)
        y = F.silu(g) * u
    if residual is not None:
        y = y + residual.float()
    return y


def close(got, want, out_dtype):
    """One rounding to the output dtype plus float32 accumulation-order noise
    (`tests/test_kernels.py:200-204` of the reference)."""
    eps = 2**-8 if out_dtype == torch.bfloat16 else 1e-5
    err = (got.float() - want).abs()
    return bool(err.max() <= 2 * eps * want.abs().max() + 1e-4), float(err.max())


# configs[1] (N, K) pairs, then the engine's real fused shapes
NK = [(960, 960), (320, 960), (5120, 960), (960, 2560), (720, 720), (4096, 720), (720, 2048),
      (2304, 768), (3072, 768), (768, 3072), (1600, 960), (1600, 720), (960, 720), (720, 960),
      (320, 320), (768, 768), (960, 12288)]  # fmt: skip
MS = [50, 241, 3072]


@pytest.mark.parametrize("m", MS)
@pytest.mark.parametrize("n,k", NK)
@pytest.mark.parametrize("epi", ["none", "residual"])
def test_gemm_sweep(m, n, k, epi):
    """every shape and row count, plain and with the fp32 residual epilogue."""
    from so101_smolvla_edge_b200.ops import linear

    x = rnd(m, k, dtype=torch.bfloat16)
    w = rnd(n, k, dtype=torch.bfloat16, scale=0.02, seed=1)
    kw = {}
    if epi == "residual":
        kw["residual"] = rnd(m, n, seed=3, scale=10.0)
    got = linear(x, w, **kw)
    want = gemm_ref(x, w, **kw)
    ok, err = close(got, want, got.dtype)
    assert ok, err
    # the configs[1] criterion: 1e-2 relative to the output scale
    assert err <= 1e-2 * want.abs().max()


GEMM_SHAPES = [(50, 720, 1600), (50, 960, 720), (50, 720, 4096), (50, 2048, 720), (241, 960, 1600),
               (241, 960, 5120), (3072, 768, 2304), (7, 104, 40), (64, 64, 64), (1, 4096, 16),
               (130, 136, 200), (200, 960, 1600)]  # fmt: skip


@pytest.mark.parametrize("m,k,n", GEMM_SHAPES)
@pytest.mark.parametrize("epi", ["none", "bias", "residual", "residual_bf16", "silu_gate", "gelu"])
def test_linear_epilogues(m, k, n, epi):
    """Each epilogue matches the float32 reference within one output rounding
    (`tests/test_kernels.py:207-228` of the reference, plus GELU for SigLIP)."""
    from so101_smolvla_edge_b200.ops import linear

    if epi == "silu_gate" and n % 2:
        n += 1
    x = rnd(m, k, dtype=torch.bfloat16)
    w = rnd(n, k, dtype=torch.bfloat16, scale=k**-0.5, seed=1)
    kw = {}
    if epi in ("bias", "gelu"):
        kw["bias"] = rnd(n if epi != "silu_gate" else n // 2, seed=2)
    if epi.startswith("residual"):
        res_dtype = torch.bfloat16 if epi == "residual_bf16" else torch.float32
        kw["residual"] = rnd(m, n, seed=3, scale=10.0).to(res_dtype)
    if epi == "silu_gate":
        kw["silu_gate"] = True
    if epi == "gelu":
        kw["gelu"] = True
    got = linear(x, w, **kw)
    want = gemm_ref(x, w, **kw)
    assert got.shape == want.shape
    ok, err = close(got, want, got.dtype)
    assert ok, err


@pytest.mark.parametrize("swap,bn", [(1, 16), (1, 32), (1, 48), (1, 64), (0, 64), (0, 128), (0, 256)])
@pytest.mark.parametrize("split", [1, 2, 3, 7, 12])
@pytest.mark.parametrize("flags", [0, 1])
def test_tiles_and_split_k_agree_and_repeat(swap, bn, split, flags):
    """Every tile shape, split count and split-K reduction (cluster / workspace) agrees with the
    reference and repeats bit for bit (split-K is deterministic:
    `tests/test_kernels.py:231-243` of the reference)."""
    from so101_smolvla_edge_b200.ops import linear

    x = rnd(50, 2048, dtype=torch.bfloat16)
    w = rnd(720, 2048, dtype=torch.bfloat16, scale=2048**-0.5, seed=1)
    r = rnd(50, 720, seed=2)
    cfg = (swap, bn, split, 0, flags)
    a = linear(x, w, residual=r, config=cfg)
    b = linear(x, w, residual=r, config=cfg)
    assert torch.equal(a, b)
    ok, err = close(a, gemm_ref(x, w, residual=r), torch.float32)
    assert ok, err


@pytest.mark.parametrize("m", [1, 7, 129])
@pytest.mark.parametrize("n,k", [(8, 8), (24, 40), (136, 72), (200, 1000)])
@pytest.mark.parametrize("plan", [None, (1, 16, 1, 0, 0), (1, 64, 2, 0, 1), (0, 64, 1, 0, 4), (0, 128, 1, 0, 2),
                                  (0, 128, 1, 0, 8)])
def test_gemm_edge_shapes(m, n, k, plan):
    """Edge shapes beside the model's: a single token row, ragged rows, outputs narrower than one
    tile, K of one 16-byte piece and K that ends inside a 64-wide block, on the default plan and on
    every tile kind (swap, split over a cluster and through the workspace, one tile per CTA,
    persistent, CTA pair). Results match the float32 product plus residual and repeat bit for bit;
    plans a shape cannot take are refused, never run."""
    from so101_smolvla_edge_b200.ops import linear

    x = rnd(m, k, dtype=torch.bfloat16)
    w = rnd(n, k, dtype=torch.bfloat16, scale=k**-0.5, seed=1)
    r = rnd(m, n, seed=2)
    try:
        a = linear(x, w, residual=r, config=plan)
    except ValueError:  # a plan this shape cannot take: refused on the host (SO101_ERR_ARG)
        assert plan is not None
        return
    assert torch.equal(a, linear(x, w, residual=r, config=plan))
    ok, err = close(a, gemm_ref(x, w, residual=r), torch.float32)
    assert ok, err


@pytest.mark.parametrize("swap,bn,split,flags", [(1, 64, 1, 0), (1, 64, 5, 0), (1, 64, 5, 1), (0, 128, 1, 0),
                                                 (0, 64, 3, 0), (0, 64, 3, 1), (0, 128, 1, 2)])
def test_silu_gate_tiles(swap, bn, split, flags):
    from so101_smolvla_edge_b200.ops import linear

    x = rnd(50, 720, dtype=torch.bfloat16)
    w = rnd(4096, 720, dtype=torch.bfloat16, scale=720**-0.5, seed=1)
    got = linear(x, w, silu_gate=True, config=(swap, bn, split, 0, flags))
    ok, err = close(got, gemm_ref(x, w, silu_gate=True), torch.bfloat16)
    assert ok, err


@pytest.mark.parametrize("m,n,k", [(3072, 2304, 768), (3072, 768, 3072), (1000, 5120, 960), (300, 720, 200)])
@pytest.mark.parametrize("epi", ["gelu", "residual", "silu_gate"])
@pytest.mark.parametrize("plan", ["persistent", "one_tile", "pair", "persistent192", "pair192"])
def test_persistent_matches_one_tile_per_cta(m, n, k, epi, plan):
    """The persistent kernel (256 or 192 columns), one tile per CTA and the CTA-pair kernel (256-row
    tiles over two SMs, cta_group::2, 256 or 192 columns) all match the reference, including tile
    counts that are not a multiple of the grid and pair tiles whose second CTA lies wholly past the
    last row."""
    flags = {"persistent": 2, "one_tile": 4, "pair": 8, "persistent192": 2, "pair192": 8}[plan]
    from so101_smolvla_edge_b200.ops import linear

    x = rnd(m, k, dtype=torch.bfloat16)
    w = rnd(2 * n if epi == "silu_gate" else n, k, dtype=torch.bfloat16, scale=k**-0.5, seed=1)
    kw = {"gelu": {"gelu": True, "bias": rnd(n, seed=2)}, "residual": {"residual": rnd(m, n, seed=3)},
          "silu_gate": {"silu_gate": True}}[epi]
    bn = 128 if epi == "silu_gate" else (192 if plan.endswith("192") else 256)
    got = linear(x, w, config=(0, bn, 1, 0, flags), **kw)
    ok, err = close(got, gemm_ref(x, w, **kw), got.dtype)
    assert ok, err


def test_linear_takes_float32_input_like_lin():
    from so101_smolvla_edge_b200.ops import linear

    x = rnd(50, 720)
    w = rnd(960, 720, dtype=torch.bfloat16, scale=720**-0.5, seed=1)
    assert torch.equal(linear(x, w), linear(x.to(torch.bfloat16), w))


def test_strided_input_view():
    """x may be a column slice of a wider buffer (the fused qkv's value columns)."""
    from so101_smolvla_edge_b200.ops import linear

    qkv = rnd(241, 1600, dtype=torch.bfloat16)
    v = qkv[:, 1280:]
    w = rnd(320, 320, dtype=torch.bfloat16, scale=320**-0.5, seed=1)
    ok, err = close(linear(v, w), gemm_ref(v, w), torch.bfloat16)
    assert ok, err


@pytest.mark.parametrize("m,k,n", [(3072, 768, 2304), (3072, 3072, 768), (192, 12288, 960), (50, 768, 64)])
@pytest.mark.parametrize("flags", [0, 2, 4, 8])
def test_int8_gemm_is_the_fake_quant_product(m, k, n, flags):
    """W8A8: int8 x and w with per-tensor / per-channel scales give the float product of the
    dequantized operands (exact int32 accumulation)."""
    from so101_smolvla_edge_b200.ops import linear, quantize_weight

    wf = rnd(n, k, scale=0.02, seed=1)
    wq, ws = quantize_weight(wf)
    # IEEE float32 quotients (float64 division rounded once); torch's CUDA division by a Python
    # scalar multiplies by the reciprocal instead, which can differ in the last bit
    ws_ref = (wf.abs().amax(1).double() / 127.0).float().clamp(min=1e-8)
    assert torch.equal(ws, ws_ref)
    q = (wf.double() / ws_ref.double()[:, None]).float()
    assert torch.equal(wq.float(), torch.clamp(torch.round(q), -127, 127))
    xs = 0.05
    xq = torch.randint(-128, 128, (m, k), device="cuda", dtype=torch.int8)
    b = rnd(n, seed=2)
    cfg = None if flags == 0 else (0, 128, 1, 0, flags)
    got = linear(xq, wq, bias=b, x_scale=xs, w_scale=ws, out_dtype=torch.float32, config=cfg)
    want = (xq.double() @ wq.double().T) * xs * ws.double() + b.double()
    err = (got.double() - want).abs().max()
    assert err <= 1e-5 * want.abs().max() + 1e-5, float(err)
    # int8 output: requantized by 1 / y_qscale, round half to even, clamped
    yq = linear(xq, wq, bias=b, x_scale=xs, w_scale=ws, out_dtype=torch.int8, y_qscale=0.25, config=cfg)
    want_q = torch.clamp(torch.round(want / 0.25), -128, 127)
    assert (yq.double() - want_q).abs().max() <= 1


# ---------------------------------------------------------------------------------- attention
def attention_ref(q, k, v, n_heads, n_kv, visible, cos=None, sin=None):
    """q rotated in fp32 and rounded to bf16, k/v expanded to the query heads, fp32 softmax."""
    lq, lk, hd = q.shape[0], k.shape[0], k.shape[1] // n_kv
    qq = q[:, : n_heads * hd].reshape(lq, n_heads, hd).float()
    if cos is not None:
        c, s = cos[:, None, :], sin[:, None, :]
        x1, x2 = qq[..., : hd // 2], qq[..., hd // 2 :]
        qq = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).to(torch.bfloat16).float()
    g = n_heads // n_kv
    kk = k.reshape(lk, n_kv, hd).float().transpose(0, 1).repeat_interleave(g, 0)
    vv = v.reshape(lk, n_kv, hd).float().transpose(0, 1).repeat_interleave(g, 0)
    sc = (qq.transpose(0, 1) @ kk.transpose(1, 2)) / hd**0.5
    if visible is not None:
        sc = sc.masked_fill(~visible, float("-inf"))
    return (torch.softmax(sc, -1) @ vv).transpose(0, 1).reshape(lq, n_heads * hd)


def rope_tables(pos, hd, base):
    half = hd // 2
    exps = (2.0 / hd) * torch.arange(half, dtype=torch.float32, device=pos.device)
    ang = pos.float()[:, None] / (base**exps)[None, :]
    return torch.cos(ang), torch.sin(ang)


def visibility(lq, lk, causal_from, q_offset):
    i = torch.arange(lq, device="cuda")[:, None]
    j = torch.arange(lk, device="cuda")[None, :]
    return (j < causal_from) | (j <= i + q_offset)


@pytest.mark.parametrize("case", ["prefix", "expert_self", "expert_cross", "small", "siglip", "odd", "single",
                                  "boundary"])
def test_attention(case):
    """the prefix-LM mask over 241 tokens (192 image + 48 text bidirectional, the
    state token last), expert self attention (50 queries over 241 prefix + 50 causal keys),
    expert cross attention (50 over 241), RoPE base 1e5; SigLIP 1024 tokens unmasked."""
    from so101_smolvla_edge_b200.ops import attention

    L, H = 241, 50
    nq, nk, hd = (15, 5, 64)
    rope = True
    if case == "prefix":
        lq, lk, pos, cf, qo = L, L, torch.arange(L), L - 1, 0
    elif case == "expert_self":
        lq, lk, pos, cf, qo = H, L + H, torch.arange(L, L + H), L, L
    elif case == "expert_cross":
        lq, lk, pos, cf, qo = H, L, torch.arange(H), L, 0
    elif case == "small":
        nq, nk, hd = 4, 2, 32
        lq, lk, pos, cf, qo = 13, 13, torch.arange(13), 12, 0
    elif case == "odd":  # key tiles that do not divide evenly over the split cluster, head_dim 128
        nq, nk, hd = 4, 1, 128
        lq, lk, pos, cf, qo = 37, 450, torch.arange(413, 450), 413, 413
    elif case == "single":  # one query, one key
        nq, nk = 1, 1
        lq, lk, pos, cf, qo = 1, 1, torch.arange(1), 1, 0
    elif case == "boundary":  # 64 queries over 65 keys, causal from the first: the second key tile holds one key
        nq, nk = 3, 1
        lq, lk, pos, cf, qo = 64, 65, torch.arange(1, 65), 0, 1
    else:
        nq, nk, hd, rope = 12, 12, 64, False
        lq, lk, pos, cf, qo = 1024, 1024, torch.arange(1024), 1024, 0
    q = rnd(lq, (nq + 2 * nk) * hd, dtype=torch.bfloat16)
    k = rnd(lk, nk * hd, dtype=torch.bfloat16, seed=1)
    v = rnd(lk, nk * hd, dtype=torch.bfloat16, seed=2)
    cos, sin = rope_tables(pos.cuda(), hd, 100_000.0) if rope else (None, None)
    got = attention(q, k, v, nq, nk, cos=cos, sin=sin, causal_from=cf, q_offset=qo)[0]
    want = attention_ref(q, k, v, nq, nk, visibility(lq, lk, cf, qo), cos, sin)
    err = (got.float() - want).abs()
    assert err.max() <= 0.02 * want.abs().max(), float(err.max())
    assert err.mean() <= 2e-3 * want.abs().mean() + 1e-4, float(err.mean())
    again = attention(q, k, v, nq, nk, cos=cos, sin=sin, causal_from=cf, q_offset=qo)[0]
    assert torch.equal(got, again)


@pytest.mark.parametrize("out", ["bf16", "int8"])
def test_siglip_attention_batched(out):
    """The vision tower's attention: 3 images x 12 heads x 1024 tokens, q/k/v as column slices of
    the fused qkv rows, unmasked (the tcgen05 path), bf16 or int8 output."""
    from so101_smolvla_edge_b200.ops import attention

    B, L, H, hd = 3, 1024, 12, 64
    qkv = rnd(B, L, 3 * H * hd, dtype=torch.bfloat16, scale=2.0)
    q, k, v = qkv[:, :, : H * hd], qkv[:, :, H * hd : 2 * H * hd], qkv[:, :, 2 * H * hd :]
    qs = 0.02
    got = attention(q, k, v, H, H, out_dtype=torch.int8 if out == "int8" else torch.bfloat16,
                    out_qscale=qs if out == "int8" else None)  # fmt: skip
    for b in range(B):
        want = attention_ref(qkv[b], k[b], v[b], H, H, None)
        if out == "int8":
            want_q = torch.clamp(torch.round(want / qs), -128, 127)
            assert (got[b].float() - want_q).abs().max() <= 1
        else:
            err = (got[b].float() - want).abs()
            assert err.max() <= 0.02 * want.abs().max() and err.mean() <= 2e-3 * want.abs().mean() + 1e-4
    again = attention(q, k, v, H, H, out_dtype=got.dtype, out_qscale=qs if out == "int8" else None)
    assert torch.equal(got, again)


@pytest.mark.parametrize("shape", [(13, 1024, "bf16"), (13, 1024, "int8"), (40, 256, "bf16"), (7, 512, "bf16")])
def test_siglip_attention_many_items(shape):
    """The unmasked tcgen05 kernel is persistent: one CTA per SM loops over (query block, head,
    image) items. These shapes give CTAs several items each, with a count that does not divide
    the grid: 624 items of 8 key tiles, 480 items of 2 key tiles (every other tile's next S
    belongs to the next item), 168 items of 4 key tiles (a few CTAs get a second item). The
    queries' double buffer, the hand-back of O between items and the rings running on across
    items are all exercised; sampled images against the float32 reference, replays equal."""
    from so101_smolvla_edge_b200.ops import attention

    B, L, out = shape
    H, hd = 12, 64
    qkv = rnd(B, L, 3 * H * hd, dtype=torch.bfloat16, scale=2.0, seed=B + L)
    q, k, v = qkv[:, :, : H * hd], qkv[:, :, H * hd : 2 * H * hd], qkv[:, :, 2 * H * hd :]
    qs = 0.02
    kw = dict(out_dtype=torch.int8, out_qscale=qs) if out == "int8" else {}
    got = attention(q, k, v, H, H, **kw)
    for b in sorted({0, B // 2, B - 1}):
        want = attention_ref(qkv[b], k[b], v[b], H, H, None)
        if out == "int8":
            assert (got[b].float() - torch.clamp(torch.round(want / qs), -128, 127)).abs().max() <= 1, b
        else:
            err = (got[b].float() - want).abs()
            assert err.max() <= 0.02 * want.abs().max() and err.mean() <= 2e-3 * want.abs().mean() + 1e-4, b
    assert torch.equal(got, attention(q, k, v, H, H, **kw))


@pytest.mark.parametrize("case", ["expert_self", "expert_cross", "prefix", "five_heads_per_kv", "prefix_v_rows",
                                  "long_queries", "one_head_per_kv"])
def test_attention_gqa_batched(case):
    """The batched prefix and expert shapes (hundreds of CTAs, grouped query heads over shared kv
    heads, prefix-LM and causal masks, RoPE on q) against the float32 reference for a sample of the
    batch; replays are equal. "prefix_v_rows" reads
    q and v as column slices of fused qkv rows (the prefix's cross layers), "long_queries" needs two
    256-row query blocks per head. All run the masked tcgen05 kernel (at least 128 CTAs): the
    prefix shapes with two 128-row groups per CTA, the expert's 50-row shapes with one group of two
    stacked heads (and "five_heads_per_kv" with a last CTA of one head)."""
    from so101_smolvla_edge_b200.ops import attention

    B, hd = 48, 64
    nq, nkv, lq, lk, cf, qo = {"expert_self": (15, 5, 50, 291, 241, 241), "expert_cross": (15, 5, 50, 241, 241, 0),
                               "prefix": (15, 5, 241, 241, 240, 0), "five_heads_per_kv": (5, 1, 50, 178, 128, 128),
                               "prefix_v_rows": (15, 5, 241, 241, 240, 0), "long_queries": (3, 1, 300, 300, 299, 0),
                               "one_head_per_kv": (4, 4, 77, 200, 150, 120)}[case]  # fmt: skip
    if case == "prefix_v_rows":
        qkv = rnd(B, lq, (nq + 2 * nkv) * hd, dtype=torch.bfloat16, scale=2.0)
        q, v = qkv[:, :, : nq * hd], qkv[:, :, (nq + nkv) * hd :]
    else:
        q = rnd(B, lq, nq * hd, dtype=torch.bfloat16, scale=2.0)
        v = rnd(B, lk, nkv * hd, dtype=torch.bfloat16, seed=2)
    k = rnd(B, lk, nkv * hd, dtype=torch.bfloat16, seed=1)
    cos, sin = rope_tables(torch.arange(qo, qo + lq, device="cuda"), hd, 10000.0)
    got = attention(q, k, v, nq, nkv, cos=cos, sin=sin, causal_from=cf, q_offset=qo)
    vis = visibility(lq, lk, cf, qo)
    for b in range(0, B, 7):
        want = attention_ref(q[b], k[b], v[b], nq, nkv, vis, cos, sin)
        err = (got[b].float() - want).abs()
        assert err.max() <= 0.02 * want.abs().max() and err.mean() <= 2e-3 * want.abs().mean() + 1e-4, (b, float(err.max()))
    assert torch.equal(got, attention(q, k, v, nq, nkv, cos=cos, sin=sin, causal_from=cf, q_offset=qo))


@pytest.mark.parametrize("batch", [1, 8, 64])
def test_attention_own_rows_equal_rope_cache_then_attention(batch):
    """so101_attention_rows (the step's own keys and values read from the fused qkv rows, the keys
    rotated on chip) against rope_kv writing them into the K/V cache followed by attention over the
    cache: the action expert's self-attention. On the mma.sync kernel (up to 12 observations) the
    bits are the same; on the tcgen05 kernel (from 13) the own keys form their own 64-key tile, so
    the key tiles and the order of the P V sums differ, and the two agree to bf16 rounding. The
    cache's own rows hold unrelated values for the fused call, so they are shown not to be read."""
    from so101_smolvla_edge_b200.ops import attention, rope_kv

    L_, H, nq, nk, hd = 241, 50, 15, 5, 64
    qd = (nq + 2 * nk) * hd
    qkv = rnd(batch, H, qd, dtype=torch.bfloat16, scale=2.0)
    cache_k = rnd(batch, L_ + H, nk * hd, dtype=torch.bfloat16, seed=1)
    cache_v = rnd(batch, L_ + H, nk * hd, dtype=torch.bfloat16, seed=2)
    cos, sin = rope_tables(torch.arange(L_, L_ + H, device="cuda"), hd, 10000.0)
    q = qkv[:, :, : nq * hd]
    own = (qkv[:, :, nq * hd : (nq + nk) * hd], qkv[:, :, (nq + nk) * hd :], L_, cos, sin)
    got = attention(q, cache_k, cache_v, nq, nk, cos=cos, sin=sin, causal_from=L_, q_offset=L_, own=own)
    for b in range(batch):
        rope_kv(qkv[b], nq, nk, cos, sin, cache_k[b, L_:], cache_v[b, L_:])
    want = attention(q, cache_k, cache_v, nq, nk, cos=cos, sin=sin, causal_from=L_, q_offset=L_)
    if batch <= 12:
        assert torch.equal(got, want)
    else:
        err = (got.float() - want.float()).abs()
        assert err.max() <= 2**-7 * want.float().abs().max() and err.mean() <= 2**-9 * want.float().abs().mean()


@pytest.mark.parametrize("tc", ["0", "1"])
@pytest.mark.parametrize(
    "kind,batch,n_out",
    [("self", 1, 720), ("cross", 1, 720), ("self", 2, 720), ("prefix", 1, 960), ("cross", 1, 100), ("long", 1, 720)],
)
def test_attention_o_equals_attention_then_projection(kind, batch, n_out, tc, monkeypatch):
    """so101_attention_o (attention, output projection and residual in one launch, the heads of
    each 128-feature tile summed across a cluster) against the float32 expression (fp32 softmax
    attention, fp32 projection): no further from it than twice the two-launch chain
    (so101_attention's bf16 rows, whose split-key merge rounds differently, projected in fp32)
    + 1e-3 * max|projection|. y16 and the statistics slots are checked against the fused output
    itself: bf16(y * w) exactly, per-tile sums of squares to fp32 rounding; a second call repeats
    the bits. The expert's self (own rows rotated on chip, causal onto its own rows) and cross
    attention at 50 rows, a batch of two, a 241-row prefix (4 query blocks) and a ragged
    100-feature output, with the attention on tcgen05 (the default) and as the mma.sync flash loop
    (SO101_ATTN_O_TC=0); cross attention over 420 keys (more than the tcgen05 form's six key tiles)
    always takes the flash loop."""
    from so101_smolvla_edge_b200.ops import attention, attention_o, rope_kv

    monkeypatch.setenv("SO101_ATTN_O_TC", tc)
    L_, nq, nk, hd = (420 if kind == "long" else 241), 15, 5, 64
    H = 241 if kind == "prefix" else 50
    qd = (nq + 2 * nk) * hd
    qkv = rnd(batch, H, qd, dtype=torch.bfloat16, scale=2.0)
    q = qkv[:, :, : nq * hd]
    if kind == "self":
        k = rnd(batch, L_ + H, nk * hd, dtype=torch.bfloat16, seed=1)
        v = rnd(batch, L_ + H, nk * hd, dtype=torch.bfloat16, seed=2)
        cos, sin = rope_tables(torch.arange(L_, L_ + H, device="cuda"), hd, 100000.0)
        kw = dict(cos=cos, sin=sin, causal_from=L_, q_offset=L_,
                  own=(qkv[:, :, nq * hd : (nq + nk) * hd], qkv[:, :, (nq + nk) * hd :], L_, cos, sin))
    elif kind in ("cross", "long"):
        k = rnd(batch, L_, nk * hd, dtype=torch.bfloat16, seed=1)
        v = rnd(batch, L_, nk * hd, dtype=torch.bfloat16, seed=2)
        cos, sin = rope_tables(torch.arange(H, device="cuda"), hd, 100000.0)
        kw = dict(cos=cos, sin=sin, causal_from=L_)
    else:  # the prefix's own attention: keys are the rows themselves, prefix-LM mask
        k, v = qkv[:, :, nq * hd : (nq + nk) * hd], qkv[:, :, (nq + nk) * hd :]
        cos, sin = rope_tables(torch.arange(H, device="cuda"), hd, 100000.0)
        kw = dict(cos=cos, sin=sin, causal_from=H - 1)
    w_o = rnd(n_out, nq * hd, dtype=torch.bfloat16, scale=0.02, seed=3)
    res = rnd(batch * H, n_out, seed=4)
    scale = 1.0 + 0.1 * rnd(n_out, seed=5)
    tiles = (n_out + 127) // 128
    y = res.clone()
    y16 = torch.zeros(batch * H, n_out, dtype=torch.bfloat16, device="cuda")
    ss = torch.full((batch * H, 64), -1.0, device="cuda")
    assert attention_o(q, k, v, nq, nk, w_o, y, residual=y, y16=y16, y16_scale=scale, stat_ss=ss, **kw) == tiles
    kc, vc, vis = k, v, visibility(H, k.shape[1], kw.get("causal_from", k.shape[1]), kw.get("q_offset", 0))
    if kind == "self":  # the reference cache holds the rotated own keys and the own values
        kc, vc = k.clone(), v.clone()
        for b in range(batch):
            rope_kv(qkv[b], nq, nk, cos, sin, kc[b, L_:], vc[b, L_:])
    a_ref = torch.cat([attention_ref(q[b], kc[b], vc[b], nq, nk, vis, cos, sin) for b in range(batch)])
    want = res + a_ref @ w_o.float().T
    chain = res + attention(q, k, v, nq, nk, **kw).reshape(batch * H, nq * hd).float() @ w_o.float().T
    size = (want - res).abs().max().item()
    err, err_chain = (y - want).abs().max().item(), (chain - want).abs().max().item()
    assert err <= 2 * err_chain + 1e-3 * size, (err, err_chain, size)
    assert torch.equal(y16, (y * scale).to(torch.bfloat16))
    sq = F.pad(y * y, (0, tiles * 128 - n_out)).view(batch * H, tiles, 128).sum(-1)
    assert torch.allclose(ss[:, :tiles], sq, rtol=1e-5, atol=1e-6)
    assert bool((ss[:, tiles:] == -1.0).all())  # no slot past the tiles is written
    y2 = res.clone()
    attention_o(q, k, v, nq, nk, w_o, y2, residual=y2, **kw)
    assert torch.equal(y2, y)


def test_attention_batched_and_strided():
    """A batch of independent problems with k and v as views into the fused qkv rows."""
    from so101_smolvla_edge_b200.ops import attention

    B, L, nq, nk, hd = 3, 241, 15, 5, 64
    qkv = rnd(B, L, (nq + 2 * nk) * hd, dtype=torch.bfloat16)
    k, v = qkv[:, :, nq * hd : (nq + nk) * hd], qkv[:, :, (nq + nk) * hd :]
    got = attention(qkv, k, v, nq, nk, causal_from=L - 1)
    for b in range(B):
        want = attention_ref(qkv[b], k[b], v[b], nq, nk, visibility(L, L, L - 1, 0))
        assert (got[b].float() - want).abs().max() <= 0.02 * want.abs().max()


@pytest.mark.parametrize("rows,offset", [(50, 241), (241, 0), (7, 3)])
def test_rope_kv(rows, offset):
    """rope_kv writes rotated k and plain v into their cache rows and nothing else; the
    rotation is torch's per-operation fp32 arithmetic, so the bf16 keys match bit for bit."""
    from so101_smolvla_edge_b200.ops import rope_kv

    nq, nk, hd = 15, 5, 64
    qkv = rnd(rows, (nq + 2 * nk) * hd, dtype=torch.bfloat16, scale=3.0)
    cos, sin = rope_tables(torch.arange(offset, offset + rows, device="cuda"), hd, 10_000.0)
    cache_k = torch.zeros(offset + rows + 5, nk * hd, dtype=torch.bfloat16, device="cuda")
    cache_v = torch.zeros_like(cache_k)
    rope_kv(qkv, nq, nk, cos, sin, cache_k[offset : offset + rows], cache_v[offset : offset + rows])
    k = qkv[:, nq * hd : (nq + nk) * hd].reshape(rows, nk, hd).float()
    c, s = cos[:, None, :], sin[:, None, :]
    want = torch.cat([k[..., :32] * c - k[..., 32:] * s, k[..., 32:] * c + k[..., :32] * s], -1)
    want = want.to(torch.bfloat16).reshape(rows, nk * hd)
    assert torch.equal(cache_k[offset : offset + rows], want)
    assert torch.equal(cache_v[offset : offset + rows], qkv[:, (nq + nk) * hd :])
    assert not cache_k[:offset].any() and not cache_k[offset + rows :].any()


@pytest.mark.parametrize("rows,n", [(50, 720), (241, 960), (7, 33), (1, 1024)])
@pytest.mark.parametrize("in_dtype", [torch.float32, torch.bfloat16])
def test_rms_norm(rows, n, in_dtype):
    from so101_smolvla_edge_b200.ops import rms_norm

    x = rnd(1, rows, n, scale=30.0).to(in_dtype)
    w = 1 + 0.1 * rnd(n, seed=1)
    want = F.rms_norm(x.float(), (n,), w, 1e-5).to(torch.bfloat16)
    got = rms_norm(x, w, 1e-5)
    assert got.shape == want.shape and got.dtype == torch.bfloat16
    assert (got.float() - want.float()).abs().max() <= 2**-7 * want.float().abs().max()
    assert (got.float() - want.float()).abs().mean() <= 1e-3 * want.float().abs().mean()


def test_layer_norm_and_pixel_shuffle():
    """LayerNorm then the SmolVLM pixel shuffle, written in one pass."""
    from so101_smolvla_edge_b200.ops import layer_norm

    x = rnd(2 * 1024, 768, scale=3.0)
    w, b = 1 + 0.1 * rnd(768, seed=1), 0.1 * rnd(768, seed=2)
    ln = F.layer_norm(x, (768,), w, b, 1e-6)
    plain = layer_norm(x, w, b, 1e-6)
    assert (plain.float() - ln).abs().max() <= 2**-7 * ln.abs().max()
    shuf = layer_norm(x, w, b, 1e-6, shuffle=4, tokens_per_image=1024)
    v = ln.reshape(2, 8, 4, 8, 4, 768).permute(0, 1, 3, 2, 4, 5).reshape(2 * 64, 768 * 16)
    assert (shuf.float() - v).abs().max() <= 2**-7 * v.abs().max()


@pytest.mark.parametrize("silu", [False, True])
def test_linear_f32_tiles_agree_bit_for_bit(silu):
    """The fp32 action/time MLP linear: many rows take the register-blocked 128 x 64 tiles, few rows
    the latency kernel; both accumulate every output over k in order, so the first rows of a
    3200-row call equal a 50-row call bit for bit, and both match float64 within fp32 rounding."""
    from so101_smolvla_edge_b200.ops import linear_f32

    x = rnd(3200, 720)
    w = rnd(720, 720, scale=720**-0.5, seed=1)
    b, b2 = rnd(720, seed=2), rnd(720, seed=3)
    big = linear_f32(x, w, b, b2, silu=silu)
    small = linear_f32(x[:50].contiguous(), w, b, b2, silu=silu)
    assert torch.equal(big[:50], small)
    want = x.double() @ w.double().T + b.double() + b2.double()
    if silu:
        want = want * torch.sigmoid(want)
    assert (big.double() - want).abs().max() <= 1e-4 * want.abs().max()
    odd = linear_f32(x[:1000, :32].contiguous(), w[:77, :32].contiguous())  # ragged tiles, short K
    assert torch.allclose(odd.double(), x[:1000, :32].double() @ w[:77, :32].double().T, rtol=1e-5, atol=1e-5)


def test_split_bf16x3_linear_matches_fp32():
    """The batched time MLP's output projection on the tensor cores: so101_split_bf16x3 writes
    [hi | hi | lo] of the fp32 activations, one bf16 GEMM against [W_hi | W_lo | W_hi] sums the three
    cross products in fp32; the result is the fp32 linear to about 2^-16 relative (the split's
    lo x lo term and the bf16 rounding of each lo part), far inside the bf16 rounding the reference
    applies to it next (model/smolvla.py:285)."""
    from so101_smolvla_edge_b200 import _lib as L
    from so101_smolvla_edge_b200.ops import linear

    x = rnd(3200, 720)
    w = rnd(720, 720, scale=720**-0.5, seed=1)
    b = rnd(720, seed=2)
    x3 = torch.empty(3200, 3 * 720, dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    L.check(L.lib().so101_split_bf16x3(x.data_ptr(), 720, 3200, 720, x3.data_ptr(), 3 * 720, stream), "split")
    hi = x.to(torch.bfloat16)
    assert torch.equal(x3[:, :720], hi) and torch.equal(x3[:, 720:1440], hi)
    assert torch.equal(x3[:, 1440:], (x - hi.float()).to(torch.bfloat16))
    wh = w.to(torch.bfloat16)
    w3 = torch.cat([wh, (w - wh.float()).to(torch.bfloat16), wh], dim=1).contiguous()
    got = linear(x3, w3, bias=b, out_dtype=torch.float32)
    want = x.double() @ w.double().T + b.double()
    assert (got.double() - want).abs().max() <= 2**-15 * want.abs().max()
    # odd sizes are refused on the host: K not a multiple of 4
    assert L.lib().so101_split_bf16x3(x.data_ptr(), 720, 3200, 718, x3.data_ptr(), 3 * 720, stream) == L.ERR_ARG


@pytest.mark.parametrize("rows", [50, 3200, 1037])
def test_expert_out_head_and_euler_step(rows):
    """so101_expert_out: x_t += dt * (rms_norm(e) @ w_out^T + b_out), one block per row, at one and
    at 64 observations and a ragged count, within fp32 rounding of float64."""
    from so101_smolvla_edge_b200 import _lib as L

    K, N, eps, dt = 720, 32, 1e-6, -0.1
    e = rnd(rows, K, scale=3.0)
    nw = 1.0 + 0.1 * rnd(K, seed=1)
    w = rnd(N, K, scale=K**-0.5, seed=2)
    b = rnd(N, seed=3)
    x = rnd(rows, N, seed=4)
    want = x.double() + dt * (((e.double() * torch.rsqrt((e.double() ** 2).mean(-1, keepdim=True) + eps)) * nw.double())
                              @ w.double().T + b.double())  # fmt: skip
    stream = torch.cuda.current_stream().cuda_stream
    L.check(L.lib().so101_expert_out(e.data_ptr(), K, nw.data_ptr(), eps, w.data_ptr(), b.data_ptr(), x.data_ptr(),
                                     N, rows, N, K, dt, stream), "expert_out")  # fmt: skip
    assert (x.double() - want).abs().max() <= 1e-5 * want.abs().max()


# ------------------------------------------------------------------ RMSNorm finished in the GEMM
def _rms_ref(x, w, eps):
    x = x.float()
    return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps) * w.float()


@pytest.mark.parametrize("rows,batch,k,hidden,n_out,use_rms", [
    (50, 1, 720, 2048, 720, True), (50, 2, 720, 2048, 720, True), (64, 1, 960, 1024, 960, False),
    (7, 1, 128, 128, 100, True)])  # fmt: skip
def test_mlp_block_matches_chain(rows, batch, k, hidden, n_out, use_rms):
    """so101_mlp (gate/up, SiLU gate, down and residual in one launch, the hidden features split
    over a cluster) against the float32 block computed from the same bf16 operand: no further
    from it than twice the two-launch chain (the gate/up GEMM's bf16 activations, then the down
    projection) + 1e-3 * max|block|. y16 and statistics against the fused output itself, and a
    second run repeats the bits. The expert's shape (50 rows, 720 -> 2048 -> 720) at one and two
    observations, a 64-row block without the norm, and a 7-row block with one hidden slice."""
    from so101_smolvla_edge_b200.ops import linear, mlp, rms_stats

    eps, m = 1e-5, rows * batch
    ss = torch.zeros(m, 64, device="cuda")
    if use_rms:
        x16 = torch.empty(m, k, device="cuda", dtype=torch.bfloat16)
        rms_stats(rnd(m, k, scale=2.0), x16, ss, 1.0 + 0.1 * rnd(k, seed=3))
        rs = torch.rsqrt(ss[:, :1] / k + eps)
    else:
        x16, rs = rnd(m, k, dtype=torch.bfloat16), torch.ones(m, 1, device="cuda")
    rms = (ss, 1, eps) if use_rms else None
    w_gu = rnd(2 * hidden, k, dtype=torch.bfloat16, scale=k**-0.5, seed=1)
    w_d = rnd(n_out, hidden, dtype=torch.bfloat16, scale=hidden**-0.5, seed=2)
    res = rnd(m, n_out, seed=4)
    scale = 1.0 + 0.1 * rnd(n_out, seed=5)
    tiles = (n_out + 127) // 128
    y = res.clone()
    y16 = torch.zeros(m, n_out, dtype=torch.bfloat16, device="cuda")
    st = torch.full((m, 64), -1.0, device="cuda")
    assert mlp(x16, w_gu, w_d, y, residual=y, rms=rms, rows=rows, y16=y16, y16_scale=scale, stat_ss=st) == tiles
    g, u = ((x16.float() * rs) @ w_gu.float().T).chunk(2, dim=-1)
    want = res + (F.silu(g) * u).to(torch.bfloat16).float() @ w_d.float().T
    chain = res + linear(x16, w_gu, silu_gate=True, rms=rms).float() @ w_d.float().T
    size = (want - res).abs().max().item()
    err, err_chain = (y - want).abs().max().item(), (chain - want).abs().max().item()
    assert err <= 2 * err_chain + 1e-3 * size, (err, err_chain, size)
    assert torch.equal(y16, (y * scale).to(torch.bfloat16))
    sq = F.pad(y * y, (0, tiles * 128 - n_out)).view(m, tiles, 128).sum(-1)
    assert torch.allclose(st[:, :tiles], sq, rtol=1e-5, atol=1e-6)
    assert bool((st[:, tiles:] == -1.0).all())
    y2 = res.clone()
    mlp(x16, w_gu, w_d, y2, residual=y2, rms=rms, rows=rows)
    assert torch.equal(y2, y)


@pytest.mark.parametrize("y", ["bf16", "i8", "f32", "resize"])
def test_preprocess_patches_match_torch(y):
    """so101_preprocess: uint8 HWC frames -> /255 -> *2-1 -> 16 x 16 patch rows, channel-major
    within a patch (`engine.py:236-245` and the patch unfold of `smolvla.py:166-170`). 512^2 frames
    take the per-patch kernel: bf16 and fp32 bit for bit against torch's float32 arithmetic, int8
    within one step of torch's round(v / scale) (exact but at rounding ties). A 480 x 640 frame
    takes the bilinear resize (align_corners False) to 384 x 512, zero-padded at the top before the
    shift: against torch's interpolate within fp32 rounding."""
    from so101_smolvla_edge_b200 import _lib as L

    g = torch.Generator(device="cuda").manual_seed(0)
    n, S, P = 3, 512, 16
    h, w = (480, 640) if y == "resize" else (S, S)
    img = torch.randint(0, 256, (n, h, w, 3), generator=g, device="cuda", dtype=torch.uint8)
    dt = {"bf16": torch.bfloat16, "i8": torch.int8}.get(y, torch.float32)
    code = {"bf16": L.BF16, "i8": L.I8}.get(y, L.F32)
    qs = 0.0123 if y == "i8" else 0.0  # 2 / 255 would put every value on a rounding tie
    rh, rw = (384, 512) if y == "resize" else (S, S)
    out = torch.empty(n * (S // P) ** 2, 3 * P * P, dtype=dt, device="cuda")
    L.check(L.lib().so101_preprocess(img.data_ptr(), n, h, w, rh, rw, S, P, out.data_ptr(), code, qs,
                                     torch.cuda.current_stream().cuda_stream), "so101_preprocess")  # fmt: skip
    # a true division (torch divides by a scalar as a multiply by its reciprocal)
    x = img.float() / torch.full(img.shape, 255.0, device="cuda")
    if y == "resize":
        x = F.interpolate(x.permute(0, 3, 1, 2), size=(rh, rw), mode="bilinear", align_corners=False)
        x = F.pad(x, (S - rw, 0, S - rh, 0)).permute(0, 2, 3, 1)  # zero in [0, 1]: -1 after the shift
    x = x * 2.0 - 1.0
    ref = x.reshape(n, S // P, P, S // P, P, 3).permute(0, 1, 3, 5, 2, 4).reshape(n * (S // P) ** 2, 3 * P * P)
    if y == "i8":
        d = (out.float() - torch.round(ref / qs).clamp(-128, 127)).abs()
        assert d.max().item() <= 1 and (d == 0).float().mean().item() > 0.999
    elif y == "resize":
        assert (out - ref).abs().max().item() <= 1e-5
    else:
        assert torch.equal(out, ref.to(dt))


@pytest.mark.parametrize("n,S,N,extras", [(3, 512, 768, True), (5, 256, 256, True), (20, 512, 768, True),
                                          (2, 512, 512, False)])  # fmt: skip
def test_patch_embed_equals_preprocess_then_gemm(n, S, N, extras):
    """so101_patch_embed (the frames converted inside the patch GEMM's operand producer) gives the
    same bits as so101_preprocess writing the patch rows followed by so101_gemm over them with the
    bias and the position table as a periodic residual, K unsplit. (20, 512): 160 row blocks, more
    than one per CTA; (5, 256): 16 x 16 patches per frame; (2, 512, 512): no bias or positions."""
    import ctypes as C

    from so101_smolvla_edge_b200 import _lib as L

    lib = L.lib()
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(4)
    img = torch.randint(0, 256, (n, S, S, 3), generator=g, device="cuda", dtype=torch.uint8)
    G = S // 16
    M, K = n * G * G, 768
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    bias = torch.randn(N, generator=g, device="cuda") * 0.1 if extras else None
    pos = torch.randn(G * G, N, generator=g, device="cuda") * 0.02 if extras else None
    got = torch.full((M, N), float("nan"), device="cuda")
    L.check(lib.so101_patch_embed(img.data_ptr(), n, S, w.data_ptr(), K, N, _p(bias), _p(pos), G * G,
                                  got.data_ptr(), N, st), "so101_patch_embed")  # fmt: skip
    patches = torch.empty(M, K, dtype=torch.bfloat16, device="cuda")
    L.check(lib.so101_preprocess(img.data_ptr(), n, S, S, S, S, S, 16, patches.data_ptr(), L.BF16, 0.0, st),
            "so101_preprocess")  # fmt: skip
    want = torch.empty(M, N, device="cuda")
    epi = L.Epilogue(epilogue=L.EPI_NONE, bias=_p(bias), residual=_p(pos), ldr=N if extras else 0,
                     r_type=L.F32, r_period=G * G if extras else 0, out_scale=1.0)  # fmt: skip
    from so101_smolvla_edge_b200.ops import workspace

    cfg = L.GemmConfig(0, 256, 1, 0, 0)
    ws = workspace(img.device)
    L.check(lib.so101_gemm(L.BF16, patches.data_ptr(), K, w.data_ptr(), K, want.data_ptr(), N, L.F32, M, N, K,
                           C.byref(epi), C.byref(cfg), ws.partials.data_ptr(), ws.nbytes, ws.tickets.data_ptr(),
                           ws.tickets.numel(), st), "so101_gemm")  # fmt: skip
    torch.cuda.synchronize()
    assert torch.equal(got, want), float((got - want).abs().max())
    assert L.lib().so101_device_status() == 0
    # frames whose 128 consecutive patches are not whole patch rows of one frame are refused
    assert lib.so101_patch_embed(img.data_ptr(), 1, 64, w.data_ptr(), K, N, None, None, 1, got.data_ptr(), N,
                                 st) == L.ERR_ARG  # fmt: skip


def test_rms_stats_matches_torch():
    from so101_smolvla_edge_b200.ops import rms_stats

    x = rnd(137, 720)
    nw = 1.0 + 0.1 * rnd(720, seed=3)
    x16 = torch.empty(137, 720, device="cuda", dtype=torch.bfloat16)
    ss = torch.zeros(137, 64, device="cuda")
    rms_stats(x, x16, ss)
    assert torch.equal(x16, x.bfloat16())
    want = (x.double() ** 2).sum(1)
    assert torch.allclose(ss[:, 0].double(), want, rtol=1e-5)
    rms_stats(x, x16, ss, nw)
    assert torch.equal(x16, (x * nw).bfloat16())
    assert torch.allclose(ss[:, 0].double(), want, rtol=1e-5)


@pytest.mark.parametrize("m,n,k,gate", [(50, 1600, 720, False), (50, 2048, 720, True), (241, 1600, 960, False),
                                        (241, 2560, 960, True), (3200, 1600, 720, False), (3200, 2048, 720, True),
                                        (10, 448, 128, False), (10, 160, 128, True), (16, 448, 320, False),
                                        (16, 256, 320, True)])  # fmt: skip
def test_rmsnorm_in_gemm(m, n, k, gate):
    """rstd * (bf16(x * w) @ W^T) against float32 rmsnorm(x) * w @ W^T and against the two-launch
    chain (rms_norm, then the GEMM): the swap tiles with and without a cluster split, the 64-wide
    normal tiles and the persistent kernel all apply the scale; one bf16 rounding of x * w, as the
    rms_norm launch rounds its output once."""
    from so101_smolvla_edge_b200.ops import linear, rms_norm, rms_stats

    eps = 1e-5
    x = rnd(m, k, scale=2.0)
    nw = 1.0 + 0.1 * rnd(k, seed=3)
    w = rnd(2 * n if gate else n, k, dtype=torch.bfloat16, scale=k**-0.5, seed=1)
    x16 = torch.empty(m, k, device="cuda", dtype=torch.bfloat16)
    ss = torch.zeros(m, 64, device="cuda")
    rms_stats(x, x16, ss, nw)
    got = linear(x16, w, silu_gate=gate, rms=(ss, 1, eps))
    want = gemm_ref(_rms_ref(x, nw, eps), w, silu_gate=gate)
    chain = linear(rms_norm(x, nw, eps), w, silu_gate=gate)
    scale = want.abs().max().item()
    err = (got.float() - want).abs().max().item()
    err_chain = (chain.float() - want).abs().max().item()
    assert err <= 1e-2 * scale, err
    assert err <= 2 * err_chain + 1e-3 * scale, (err, err_chain)


@pytest.mark.parametrize("m,n,k,config", [(50, 720, 960, None), (50, 720, 2048, None), (241, 960, 2560, None),
                                          (3200, 720, 960, None), (3200, 720, 960, (0, 256, 1, 0, 8))])
def test_residual_gemm_statistics(m, n, k, config):
    """A residual GEMM's statistics (sums of squares over disjoint column ranges) and bf16(output
    * next norm weight) feed the next norm's GEMM: the slots sum to the rows' sums of squares,
    bit-stable."""
    from so101_smolvla_edge_b200.ops import gemm_stat_slots, linear

    x = rnd(m, k, dtype=torch.bfloat16)
    w = rnd(n, k, dtype=torch.bfloat16, scale=k**-0.5, seed=1)
    e = rnd(m, n, seed=2)
    nw = 1.0 + 0.1 * rnd(n, seed=3)
    slots = gemm_stat_slots(m, n, k, config)
    assert 1 <= slots <= 64
    outs = []
    for _ in range(2):
        r = e.clone()
        ss = torch.zeros(m, 64, device="cuda")
        x16 = torch.zeros(m, n, device="cuda", dtype=torch.bfloat16)
        linear(x, w, residual=r, out=r, stat=(ss, x16, nw), config=config)
        outs.append((r, ss, x16))
    r, ss, x16 = outs[0]
    assert torch.equal(r, outs[1][0]) and torch.equal(ss, outs[1][1])
    ok, err = close(r, gemm_ref(x, w, residual=e), torch.float32)
    assert ok, err
    assert torch.equal(x16, (r * nw).bfloat16())
    want = (r.double() ** 2).sum(1)
    assert torch.allclose(ss[:, :slots].double().sum(1), want, rtol=1e-4)
    assert torch.count_nonzero(ss[:, slots:]) == 0
