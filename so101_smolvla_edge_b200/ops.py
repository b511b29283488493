"""The kernels as torch-tensor operators, with the reference's operator API.

    linear     kernels/gemm.py:350-398        y = x @ w.T with fused bias / residual / SiLU gate
                                              (+ GELU, int8 operands, row remap for the engine)
    attention  kernels/attention.py:110-153   GQA over the kv heads, RoPE on q, computed mask
    rope_kv    kernels/rope.py:481-506        RoPE on the keys + K/V cache write
    rms_norm   kernels/norm.py:423-440        fp32 statistics, one rounding

Every call goes through the C ABI of libso101_b200.so on the tensors' current CUDA stream.
Preconditions the kernels cannot meet raise ValueError, as the reference's wrappers do.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L

DTYPE = {torch.bfloat16: L.BF16, torch.float32: L.F32, torch.int8: L.I8}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and t.device.type != "cuda":
            raise ValueError("the B200 kernels take CUDA tensors only")


class Workspace:
    """Split-K partials and tickets for one device. Every GEMM on the device's stream shares it
    (they run one after another); it must exist before a CUDA graph is captured, as the
    reference's split-K counters must (kernels/gemm.py:335-347)."""

    def __init__(self, device: torch.device, nbytes: int = 64 << 20, n_tickets: int = 1 << 16):
        self.partials = torch.empty(nbytes // 4, dtype=torch.float32, device=device)
        self.tickets = torch.zeros(n_tickets, dtype=torch.int32, device=device)

    @property
    def nbytes(self) -> int:
        return self.partials.numel() * 4


_WS: dict[torch.device, Workspace] = {}


def workspace(device: torch.device | str) -> Workspace:
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    ws = _WS.get(device)
    if ws is None:
        ws = _WS[device] = Workspace(device)
    return ws


def gemm_config(m: int, n: int, k: int, *, silu_gate=False, int8=False) -> tuple[int, int, int, int]:
    """(swap, bn, splits, stages) the library picks for this problem."""
    cfg = L.GemmConfig()
    epi = L.EPI_SILU_GATE if silu_gate else L.EPI_NONE
    L.check(L.lib().so101_gemm_pick(L.I8 if int8 else L.BF16, m, n, k, epi, C.byref(cfg)), "gemm_pick")
    return cfg.as_tuple()


def linear(
    x: torch.Tensor,
    w: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    silu_gate: bool = False,
    gelu: bool = False,
    out_dtype: torch.dtype | None = None,
    out: torch.Tensor | None = None,
    config: tuple[int, int, int, int] | None = None,
    out_scale: float = 1.0,
    residual_period: int = 0,
    x_scale: float | None = None,
    w_scale: torch.Tensor | None = None,
    y_qscale: float | None = None,
    rms: tuple[torch.Tensor, int, float] | None = None,
    stat: tuple[torch.Tensor, torch.Tensor] | None = None,
) -> torch.Tensor:
    """Compute x (..., K) @ w (N, K).T with a fused epilogue on tcgen05.

    With `silu_gate`, w is (2F, K) = [gate; up] and the result (..., F). `residual` (..., N) is
    added in float32 and the result takes its dtype unless `out_dtype` says otherwise; `out` may
    be the residual itself. A float32 x is rounded to bf16 first, as `SmolVLA.lin` casts it.
    int8 operands: x and w int8 with `x_scale` (per tensor) and `w_scale` (N,) dequantizing the
    int32 accumulator. out_dtype int8 quantizes the result by `y_qscale`.

    RMSNorm finished in the GEMM (not in the reference, which launches rms_norm before the GEMM):
    rms=(ss, slots, eps) with x = bf16(residual stream * norm weight) scales row m by
    rsqrt(sum(ss[m, :slots]) / K + eps). stat=(ss, x16[, norm_w]) makes this (residual) GEMM write
    its rows' sums of squares into ss (`gemm_stat_slots` tells how many slots) and bf16(output *
    norm_w) into x16, the next such GEMM's x.
    """
    _cuda(x, w, bias, residual, out)
    if silu_gate and (residual is not None or bias is not None or gelu):
        raise ValueError("silu_gate takes neither a residual, a bias nor gelu")
    k = x.shape[-1]
    int8 = w.dtype == torch.int8
    if int8:
        if x.dtype != torch.int8 or w_scale is None or x_scale is None:
            raise ValueError("int8 weights need int8 x, x_scale and w_scale")
    elif x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    if w.dtype not in (torch.bfloat16, torch.int8):
        raise ValueError(f"w must be bf16 or int8, not {w.dtype}")
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1 or w.stride(-1) != 1:
        raise ValueError("x and w need unit column stride")
    m = x2.shape[0]
    n = w.shape[0] // 2 if silu_gate else w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"x has {k} features, w {tuple(w.shape)}")
    if out_dtype is None:
        out_dtype = residual.dtype if residual is not None else (
            torch.bfloat16 if int8 else w.dtype)  # fmt: skip
    y = out.view(m, n) if out is not None else torch.empty(m, n, dtype=out_dtype, device=x.device)
    r2 = None
    if residual is not None:
        r2 = residual.reshape(-1, n) if residual_period == 0 else residual
        if r2.stride(-1) != 1:
            raise ValueError("residual needs unit column stride")
    epi = L.Epilogue(
        epilogue=L.EPI_SILU_GATE if silu_gate else (L.EPI_GELU if gelu else L.EPI_NONE),
        bias=_ptr(bias), residual=_ptr(r2), ldr=r2.stride(0) if r2 is not None else 0,
        r_type=DTYPE[r2.dtype] if r2 is not None else 0, r_period=residual_period,
        out_scale=out_scale, w_scale=_ptr(w_scale), x_scale=x_scale or 0.0,
        y_qscale=y_qscale or 0.0, row_group=0, row_stride=0,
    )  # fmt: skip
    if rms is not None:
        ss, slots, eps = rms
        epi.rms_ss, epi.rms_slots, epi.rms_ld, epi.rms_n, epi.rms_eps = ss.data_ptr(), slots, ss.stride(0), float(k), eps
    if stat is not None:
        ss, x16, nw = stat if len(stat) == 3 else (*stat, None)
        epi.stat_ss, epi.stat_ld, epi.y16, epi.ld16 = ss.data_ptr(), ss.stride(0), x16.data_ptr(), x16.stride(0)
        epi.y16_scale = _ptr(nw)
    cfg = None
    if config is not None:
        cfg = L.GemmConfig(*config)
    ws = workspace(x.device)
    rc = L.lib().so101_gemm(
        L.I8 if int8 else L.BF16, x2.data_ptr(), x2.stride(0), w.data_ptr(), w.stride(0),
        y.data_ptr(), y.stride(0), DTYPE[y.dtype], m, n, k, C.byref(epi),
        C.byref(cfg) if cfg is not None else None, ws.partials.data_ptr(), ws.nbytes,
        ws.tickets.data_ptr(), ws.tickets.numel(), _stream(x.device),
    )  # fmt: skip
    L.check(rc, "so101_gemm")
    return y.view(*x.shape[:-1], n)


def linear_f32(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None, bias2: torch.Tensor | None = None,
               silu: bool = False) -> torch.Tensor:
    """y = x @ w.T (+ bias + bias2), then SiLU when `silu`, all in float32 on CUDA cores: the
    action / time MLP of the velocity (pkg/model/smolvla.py:282-285). Sequential fmaf over k for
    every output, so any row tiling gives the same bits."""
    _cuda(x, w, bias, bias2)
    m, k = x.shape
    n = w.shape[0]
    y = torch.empty(m, n, dtype=torch.float32, device=x.device)
    L.check(L.lib().so101_linear_f32(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0), _ptr(bias), _ptr(bias2),
                                     y.data_ptr(), y.stride(0), m, n, k, 2 if silu else 0, _stream(x.device)),
            "linear_f32")  # fmt: skip
    return y


def gemm_stat_slots(m: int, n: int, k: int, config=None) -> int:
    """Statistics slots a bf16 GEMM of this shape writes with `stat` (ValueError if none)."""
    got = C.c_int()
    cfg = L.GemmConfig(*config) if config is not None else None
    L.check(L.lib().so101_gemm_stat_slots(L.BF16, m, n, k, L.EPI_NONE, C.byref(cfg) if cfg else None,
                                          C.byref(got)), "gemm_stat_slots")  # fmt: skip
    return got.value


def rms_stats(x: torch.Tensor, x16: torch.Tensor, ss: torch.Tensor, w: torch.Tensor | None = None) -> None:
    """Slot 0 of ss = per-row sums of squares of the fp32 rows x; x16 = bf16(x * w) (w: the norm
    weight, fp32, None: 1)."""
    _cuda(x, x16, ss)
    L.check(L.lib().so101_rms_stats(x.data_ptr(), x.stride(0), x.shape[0], x.shape[1], _ptr(w), x16.data_ptr(),
                                    x16.stride(0), ss.data_ptr(), ss.stride(0), _stream(x.device)),
            "rms_stats")  # fmt: skip


def attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    n_heads: int,
    n_kv: int,
    *,
    cos: torch.Tensor | None = None,
    sin: torch.Tensor | None = None,
    causal_from: int | None = None,
    q_offset: int = 0,
    out: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    out_qscale: float | None = None,
    own: tuple | None = None,
) -> torch.Tensor:
    """Attention of q's heads over k and v, written as (Lq, n_heads * hd).

    q is (Lq, >= n_heads * hd) with head h in columns [h * hd, (h + 1) * hd) and any row stride,
    so it can be a slice of the fused qkv output; k and v are (Lk, n_kv * hd). A leading batch
    dimension on all three runs independent problems. cos and sin (Lq, hd / 2) rotate q; None
    means no RoPE. Key j is visible to query i iff j < causal_from or j <= i + q_offset; None
    means every key is visible. own=(k_own, v_own, own_from, k_cos, k_sin): keys j >= own_from and
    their values come from row j - own_from of k_own / v_own (e.g. the fused qkv rows), the keys
    rotated by k_cos / k_sin as the RoPE cache write would (so101_attention_rows).
    """
    _cuda(q, k, v, out)
    batched = q.dim() == 3
    qb, kb, vb = (q, k, v) if batched else (q[None], k[None], v[None])
    bsz, lq, lk = qb.shape[0], qb.shape[1], kb.shape[1]
    hd = kb.shape[2] // n_kv
    for name, t in (("q", qb), ("k", kb), ("v", vb)):
        if t.stride(-1) != 1:
            raise ValueError(f"{name} needs unit column stride, has {t.stride()}")
        if t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be bf16")
    if out is None:
        out = torch.empty(bsz, lq, n_heads * hd, dtype=out_dtype, device=q.device)
    ob = out if out.dim() == 3 else out[None]
    if cos is not None:
        cos = cos.reshape(lq, hd // 2).float().contiguous()
        sin = sin.reshape(lq, hd // 2).float().contiguous()
    ck = lk if causal_from is None else causal_from
    args = (qb.data_ptr(), qb.stride(1), kb.data_ptr(), kb.stride(1), vb.data_ptr(), vb.stride(1),
            ob.data_ptr(), ob.stride(1), DTYPE[ob.dtype], out_qscale or 0.0, lq, lk, n_heads, n_kv, hd,
            ck, q_offset, _ptr(cos), _ptr(sin), bsz, qb.stride(0), kb.stride(0), vb.stride(0),
            ob.stride(0))  # fmt: skip
    if own is None:
        L.check(L.lib().so101_attention(*args, _stream(q.device)), "so101_attention")
    else:
        k_own, v_own, own_from, k_cos, k_sin = own
        ko = k_own if k_own.dim() == 3 else k_own[None]
        vo = v_own if v_own.dim() == 3 else v_own[None]
        if ko.stride(1) != vo.stride(1) or ko.stride(0) != vo.stride(0):
            raise ValueError("k_own and v_own need the same strides (views of one fused buffer)")
        L.check(L.lib().so101_attention_rows(*args, ko.data_ptr(), vo.data_ptr(), ko.stride(1), ko.stride(0),
                                             own_from, k_cos.data_ptr(), k_sin.data_ptr(), _stream(q.device)),
                "so101_attention_rows")  # fmt: skip
    return out


def attention_o(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    n_heads: int,
    n_kv: int,
    w_o: torch.Tensor,
    y: torch.Tensor,
    *,
    residual: torch.Tensor | None = None,
    cos: torch.Tensor | None = None,
    sin: torch.Tensor | None = None,
    causal_from: int | None = None,
    q_offset: int = 0,
    own: tuple | None = None,
    y16: torch.Tensor | None = None,
    y16_scale: torch.Tensor | None = None,
    stat_ss: torch.Tensor | None = None,
) -> int:
    """y = residual + attention(q, k, v) @ w_o^T in one launch (so101_attention_o).

    q, k, v, cos, sin, causal_from, q_offset and own as `attention` (head_dim 64, at most 16 query
    heads); y and residual fp32 (rows b * Lq + i, residual may be y); w_o (N, n_heads * 64) bf16.
    y16 (bf16) receives y * y16_scale per column and stat_ss[row, t] the row's sum of squares over
    output features [128 t, 128 t + 128). Returns the number of statistics slots, ceil(N / 128).
    """
    _cuda(q, k, v, w_o, y, residual, y16, y16_scale, stat_ss)
    batched = q.dim() == 3
    qb, kb, vb = (q, k, v) if batched else (q[None], k[None], v[None])
    bsz, lq, lk = qb.shape[0], qb.shape[1], kb.shape[1]
    hd = kb.shape[2] // n_kv
    for name, t in (("q", qb), ("k", kb), ("v", vb), ("w_o", w_o)):
        if t.stride(-1) != 1:
            raise ValueError(f"{name} needs unit column stride, has {t.stride()}")
        if t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be bf16")
    n_out = w_o.shape[0]
    y2 = y.reshape(-1, n_out) if y.dim() == 3 else y
    r2 = None if residual is None else (residual.reshape(-1, n_out) if residual.dim() == 3 else residual)
    for name, t in (("y", y2), ("residual", r2), ("stat_ss", stat_ss)):
        if t is not None and t.dtype != torch.float32:
            raise ValueError(f"{name} must be float32")
    if y16 is not None and y16.dtype != torch.bfloat16:
        raise ValueError("y16 must be bf16")
    if cos is not None:
        cos = cos.reshape(lq, hd // 2).float().contiguous()
        sin = sin.reshape(lq, hd // 2).float().contiguous()
    if y16_scale is not None:
        y16_scale = y16_scale.float().contiguous()
    ck = lk if causal_from is None else causal_from
    own_args: tuple = (None, None, 0, 0, 0, None, None)
    if own is not None:
        k_own, v_own, own_from, k_cos, k_sin = own
        ko = k_own if k_own.dim() == 3 else k_own[None]
        vo = v_own if v_own.dim() == 3 else v_own[None]
        if ko.stride(1) != vo.stride(1) or ko.stride(0) != vo.stride(0):
            raise ValueError("k_own and v_own need the same strides (views of one fused buffer)")
        own_args = (ko.data_ptr(), vo.data_ptr(), ko.stride(1), ko.stride(0), own_from, k_cos.data_ptr(),
                    k_sin.data_ptr())  # fmt: skip
    y16_2 = None if y16 is None else y16.reshape(-1, n_out) if y16.dim() == 3 else y16
    rc = L.lib().so101_attention_o(
        qb.data_ptr(), qb.stride(1), kb.data_ptr(), kb.stride(1), vb.data_ptr(), vb.stride(1), lq, lk, n_heads,
        n_kv, hd, ck, q_offset, _ptr(cos), _ptr(sin), bsz, qb.stride(0), kb.stride(0), vb.stride(0), *own_args,
        w_o.data_ptr(), w_o.stride(0), n_out, y2.data_ptr(), y2.stride(0), _ptr(r2), 0 if r2 is None else r2.stride(0),
        _ptr(y16_2), 0 if y16_2 is None else y16_2.stride(0), _ptr(y16_scale), _ptr(stat_ss),
        0 if stat_ss is None else stat_ss.stride(0), _stream(q.device),
    )  # fmt: skip
    L.check(rc, "so101_attention_o")
    return (n_out + 127) // 128


def mlp(
    x: torch.Tensor,
    w_gate_up: torch.Tensor,
    w_down: torch.Tensor,
    y: torch.Tensor,
    *,
    residual: torch.Tensor | None = None,
    rms: tuple[torch.Tensor, int, float] | None = None,
    rows: int | None = None,
    y16: torch.Tensor | None = None,
    y16_scale: torch.Tensor | None = None,
    stat_ss: torch.Tensor | None = None,
) -> int:
    """y = residual + (silu(x @ gate^T) * (x @ up^T)) @ w_down^T in one launch (so101_mlp).

    x (B * rows, K) bf16 with at most 64 rows per observation (rows defaults to all of x: one
    observation); w_gate_up (2 * mlp, K) is [gate; up]; w_down (N, mlp). rms=(ss, slots, eps)
    finishes the RMSNorm of x as `linear` does. y, residual, y16, y16_scale and stat_ss as
    `attention_o`. Returns the number of statistics slots, ceil(N / 128).
    """
    _cuda(x, w_gate_up, w_down, y, residual, y16, y16_scale, stat_ss)
    for name, t in (("x", x), ("w_gate_up", w_gate_up), ("w_down", w_down)):
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1:
            raise ValueError(f"{name} must be bf16 with unit column stride")
    rows = x.shape[0] if rows is None else rows
    if x.shape[0] % rows:
        raise ValueError("x's rows are not a whole number of observations")
    n_out, hidden = w_down.shape
    if w_gate_up.shape[0] != 2 * hidden:
        raise ValueError("w_gate_up needs 2 * mlp rows for w_down's mlp columns")
    for name, t in (("y", y), ("residual", residual), ("stat_ss", stat_ss)):
        if t is not None and t.dtype != torch.float32:
            raise ValueError(f"{name} must be float32")
    if y16_scale is not None:
        y16_scale = y16_scale.float().contiguous()
    ss, slots, eps = rms if rms is not None else (None, 0, 0.0)
    rc = L.lib().so101_mlp(
        x.data_ptr(), x.stride(0), rows, x.shape[0] // rows, x.shape[1], _ptr(ss), slots,
        0 if ss is None else ss.stride(0), eps, w_gate_up.data_ptr(), w_gate_up.stride(0), hidden,
        w_down.data_ptr(), w_down.stride(0), n_out, y.data_ptr(), y.stride(0), _ptr(residual),
        0 if residual is None else residual.stride(0), _ptr(y16), 0 if y16 is None else y16.stride(0),
        _ptr(y16_scale), _ptr(stat_ss), 0 if stat_ss is None else stat_ss.stride(0), _stream(x.device),
    )  # fmt: skip
    L.check(rc, "so101_mlp")
    return (n_out + 127) // 128


def rope_kv(
    qkv: torch.Tensor,
    n_heads: int,
    n_kv: int,
    cos: torch.Tensor,
    sin: torch.Tensor,
    k_out: torch.Tensor,
    v_out: torch.Tensor | None = None,
) -> None:
    """Rotate the key columns of qkv into k_out and copy its value columns into v_out.

    qkv is (R, (n_heads + 2 * n_kv) * hd), k_out and v_out (R, n_kv * hd) and may be row slices
    of a larger cache, cos and sin (R, hd / 2).
    """
    _cuda(qkv, k_out, v_out)
    r = qkv.shape[0]
    hd = qkv.shape[1] // (n_heads + 2 * n_kv)
    for name, t in (("qkv", qkv), ("k_out", k_out), ("v_out", v_out)):
        if t is not None and t.stride(-1) != 1:
            raise ValueError(f"{name} needs unit column stride")
    cos = cos.reshape(r, hd // 2).float().contiguous()
    sin = sin.reshape(r, hd // 2).float().contiguous()
    rc = L.lib().so101_rope_kv(
        qkv.data_ptr(), qkv.stride(0), n_heads, n_kv, hd, cos.data_ptr(), sin.data_ptr(),
        k_out.data_ptr(), k_out.stride(0), _ptr(v_out), v_out.stride(0) if v_out is not None else 0,
        r, 1, 0, 0, 0, _stream(qkv.device),
    )  # fmt: skip
    L.check(rc, "so101_rope_kv")


def rms_norm(
    x: torch.Tensor,
    w: torch.Tensor,
    eps: float,
    out_dtype: torch.dtype = torch.bfloat16,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Normalize x (..., N), float32 or bf16, by w (N,) into `out_dtype`."""
    _cuda(x, w, out)
    n = x.shape[-1]
    x2 = x.reshape(-1, n)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    y = out if out is not None else torch.empty(x2.shape, dtype=out_dtype, device=x.device)
    w = w.float().contiguous()
    rc = L.lib().so101_rms_norm(
        x2.data_ptr(), x2.stride(0), DTYPE[x2.dtype], w.data_ptr(), y.data_ptr(), y.stride(0),
        DTYPE[y.dtype], x2.shape[0], n, eps, _stream(x.device),
    )  # fmt: skip
    L.check(rc, "so101_rms_norm")
    return y.view(*x.shape[:-1], n)


def layer_norm(x, w, b, eps, out_dtype=torch.bfloat16, out_qscale=None, shuffle=1,
               tokens_per_image=0, out=None):  # fmt: skip
    """LayerNorm of float32 rows (+ the SmolVLM pixel shuffle of each image's tokens)."""
    _cuda(x, w, b, out)
    n = x.shape[-1]
    x2 = x.reshape(-1, n)
    rows = x2.shape[0]
    if out is None:
        shape = (rows // shuffle**2, n * shuffle**2) if shuffle > 1 else (rows, n)
        out = torch.empty(shape, dtype=out_dtype, device=x.device)
    rc = L.lib().so101_layer_norm(
        x2.data_ptr(), x2.stride(0), w.data_ptr(), b.data_ptr(), out.data_ptr(), out.stride(0),
        DTYPE[out.dtype], out_qscale or 0.0, rows, n, eps, shuffle, tokens_per_image,
        _stream(x.device),
    )  # fmt: skip
    L.check(rc, "so101_layer_norm")
    return out


def quantize_weight(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel symmetric int8 (w_q, scale) of a float32 or bf16 (N, K) matrix."""
    _cuda(w)
    w = w.contiguous()
    n, k = w.shape
    wq = torch.empty(n, k, dtype=torch.int8, device=w.device)
    s = torch.empty(n, dtype=torch.float32, device=w.device)
    rc = L.lib().so101_quantize_weight(w.data_ptr(), DTYPE[w.dtype], n, k, wq.data_ptr(),
                                       s.data_ptr(), _stream(w.device))  # fmt: skip
    L.check(rc, "so101_quantize_weight")
    return wq, s


def device_status() -> int:
    return L.lib().so101_device_status()


def set_pdl(enable: bool) -> None:
    """Launch GEMMs with programmatic dependent launch (they start streaming weights while the
    previous kernel on the stream drains)."""
    L.check(L.lib().so101_set_pdl(1 if enable else 0), "so101_set_pdl")
