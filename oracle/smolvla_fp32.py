"""CPU float32 oracle for the SmolVLA chunk path. TEST INFRASTRUCTURE ONLY.

Only tests, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg may import this module,
and only as the checker or the timed CPU baseline. The product path (the CUDA engine in
`so101_smolvla_edge_b200`) never imports or calls it.

It restates, in float32 torch on the CPU, what the reference's float32 engine computes
(`Engine(device="cpu", dtype="fp32", cuda_graph=False)`, which `scripts/standin_bundle.py:150`
uses to write its golden actions). Each function cites the reference lines it follows; paths are
relative to the reference project, `pkg/` = `src/so101_smolvla_edge/`.

Parity is pinned: `tests/golden/make_golden.py` ran the reference itself on seeded bundles and
stored its actions and intermediates; `tests/test_oracle.py` checks this module against them.

W8A8 vision (`act_clip` given) follows the int8 arithmetic the reference pins in
`tests/test_ov_engine.py:222-236` for its TensorRT/OpenVINO int8 graphs: per-output-channel
symmetric weights `Wq = clamp(round(W / s_w), -127, 127)`, `s_w = max|W_row| / 127`; per-tensor
activations `xq = clamp(round(x / s_x), -128, 127)`, `s_x = clip / 127`; the product in float32.
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from so101_smolvla_edge_b200.bundle import Bundle
from so101_smolvla_edge_b200.spec import ModelSpec

Tensor = torch.Tensor


class Oracle:
    """The float32 chunk for one bundle: `actions(images, state, noise)`."""

    def __init__(self, bundle: Bundle, act_clip: dict[str, float] | None = None,
                 threads: int | None = None):  # fmt: skip
        if threads:
            torch.set_num_threads(threads)
        self.b = bundle
        self.s: ModelSpec = bundle.spec
        self.w = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in bundle.tensors.items()}
        self.act_clip = act_clip
        self.record: dict[str, list[float]] | None = None  # calibration: max |x| per linear
        s = self.s
        L, H = s.prefix_len, s.chunk
        self.cos_p, self.sin_p = rope_tables(torch.arange(L), s.head_dim, s.rope_wavelength)
        self.cos_s, self.sin_s = rope_tables(torch.arange(L, L + H), s.head_dim,
                                             s.rope_wavelength)  # fmt: skip
        self.cos_c, self.sin_c = rope_tables(torch.arange(H), s.head_dim, s.rope_wavelength)
        self.time_proj = time_projection(s, self.w)

    # -------------------------------------------------------------------- linears
    def lin(self, x: Tensor, name: str, bias: str | None = None, qname: str | None = None):
        """x @ W.T (+ b) in float32; W8A8 fake quant when `qname` has an activation clip."""
        W = self.w[name]
        b = None if bias is None else self.w[bias]
        if qname is not None and self.record is not None:
            self.record[qname] = max(self.record.get(qname, 0.0), float(x.abs().max()))
        if qname is not None and self.act_clip is not None and qname in self.act_clip:
            xs = self.act_clip[qname] / 127.0
            x = torch.clamp(torch.round(x / xs), -128, 127) * xs
            ws = (W.abs().amax(1, keepdim=True) / 127.0).clamp(min=1e-8)
            W = torch.clamp(torch.round(W / ws), -127, 127) * ws
        y = x @ W.T
        return y if b is None else y + b

    # -------------------------------------------------------------------- vision
    def preprocess(self, images: dict[str, np.ndarray]) -> Tensor:
        """uint8 HWC frames -> px (n, 3, S, S) in [-1, 1]: bilinear resize keeping the aspect,
        zero padding on the left and top (`pkg/model/engine.py:236-245`)."""
        S = self.s.image_size
        img = torch.stack([torch.from_numpy(np.ascontiguousarray(images[c])) for c in self.b.cameras])
        x = img.permute(0, 3, 1, 2).float() / 255.0
        h, w = x.shape[2:]
        ratio = max(w / S, h / S)
        rh, rw = int(h / ratio), int(w / ratio)
        x = F.interpolate(x, size=(rh, rw), mode="bilinear", align_corners=False)
        x = F.pad(x, (S - rw, 0, S - rh, 0), value=0.0)
        return x * 2.0 - 1.0

    def vision(self, px: Tensor) -> Tensor:
        """SigLIP + post-LN + pixel shuffle + connector -> rows (n * 64, text_dim) * sqrt(text_dim)
        (`pkg/model/smolvla.py:159-190`)."""
        s, w = self.s, self.w
        n, g, P, d = px.shape[0], s.grid, s.patch, s.vis_dim
        # (n, 3, gy, P, gx, P) -> (n, gy, gx, 3, P, P): feature = c*P*P + py*P + px
        patches = px.reshape(n, 3, g, P, g, P).permute(0, 2, 4, 1, 3, 5).reshape(n, g * g, 3 * P * P)
        x = self.lin(patches, "vis.patch.w", "vis.patch.b", "patch") + w["vis.pos"]
        nh, hd = s.vis_heads, d // s.vis_heads
        for i in range(s.vis_layers):
            p = f"vis.{i}."
            h = layer_norm(x, w[p + "ln1.w"], w[p + "ln1.b"], s.vis_eps)
            qkv = self.lin(h, p + "qkv.w", p + "qkv.b", p[:-1] + ".qkv").reshape(n, -1, 3, nh, hd)
            q, k, v = (qkv[:, :, j].transpose(1, 2) for j in range(3))  # (n, heads, L, hd)
            a = softmax_attention(q, k, v, None).transpose(1, 2).reshape(n, -1, d)
            x = x + self.lin(a, p + "out.w", p + "out.b", p[:-1] + ".out")
            h = layer_norm(x, w[p + "ln2.w"], w[p + "ln2.b"], s.vis_eps)
            h = gelu_tanh(self.lin(h, p + "fc1.w", p + "fc1.b", p[:-1] + ".fc1"))
            x = x + self.lin(h, p + "fc2.w", p + "fc2.b", p[:-1] + ".fc2")
        x = layer_norm(x, w["vis.post_ln.w"], w["vis.post_ln.b"], s.vis_eps)
        x = self.lin(shuffle_tokens(x, s.shuffle), "conn.w", None, "conn")
        return (x * math.sqrt(s.text_dim)).reshape(-1, s.text_dim)

    # -------------------------------------------------------------------- prefix
    def prefix_rows(self, img_rows: Tensor, state: Tensor) -> Tensor:
        """[image rows; task tokens; state row] (`pkg/model/engine.py:247-252`)."""
        s, w = self.s, self.w
        st = (state - w["norm.state.mean"]) / (w["norm.state.std"] + 1e-8)
        st = F.pad(st, (0, s.max_state - st.shape[0]))
        st_row = (st @ w["state.w"].T + w["state.b"])[None]
        return torch.cat([img_rows, w["lang.emb"], st_row], dim=0)

    def prefix(self, rows: Tensor) -> dict[str, list]:
        """The VLM layers over the prefix rows; returns every layer's rotated K and V (L, n_kv*hd)
        and the expert's caches (`pkg/model/smolvla.py:193-257`,
        `pkg/model/smolvla_triton.py:78-103`)."""
        s, w = self.s, self.w
        L, nq, nk, hd = rows.shape[0], s.n_heads, s.n_kv, s.head_dim
        x = rows.clone()
        ks, vs, kx, vx = [], [], [], []
        for i in range(s.n_layers):
            t = f"txt.{i}."
            h = rms_norm(x, w[t + "ln_in"], s.rms_eps)
            qkv = self.lin(h, t + "qkv")
            q, k, v = qkv.split([nq * hd, nk * hd, nk * hd], dim=-1)
            k = rope(k.reshape(L, nk, hd), self.cos_p, self.sin_p).reshape(L, nk * hd)
            ks.append(k)
            vs.append(v)
            if s.is_self_attn(i):
                kx.append(None)
                vx.append(None)
            else:
                kx.append(self.lin(k, f"exp.{i}.k"))
                vx.append(self.lin(v, f"exp.{i}.v"))
            if i == s.n_layers - 1:
                break
            q = rope(q.reshape(L, nq, hd), self.cos_p, self.sin_p)
            vis = prefix_visibility(L)
            a = gqa(q, k.reshape(L, nk, hd), v.reshape(L, nk, hd), vis)
            x = x + self.lin(a, t + "o")
            h = rms_norm(x, w[t + "ln_post"], s.rms_eps)
            gu = self.lin(h, t + "gate_up")
            g, u = gu.chunk(2, dim=-1)
            x = x + self.lin(F.silu(g) * u, t + "down")
        return {"k": ks, "v": vs, "kx": kx, "vx": vx}

    # -------------------------------------------------------------------- denoising
    def velocity(self, x_t: Tensor, k_step: int, cache: dict[str, list]) -> Tensor:
        """Flow velocity (H, max_action) for noisy actions x_t (H, max_action)
        (`pkg/model/smolvla.py:260-309`)."""
        s, w = self.s, self.w
        L, H = s.prefix_len, x_t.shape[0]
        nq, nk, hd = s.n_heads, s.n_kv, s.head_dim
        a_emb = x_t @ w["act.in.w"].T + w["act.in.b"]
        h = a_emb @ w["act.time_in.w_action"].T + self.time_proj[k_step]
        e = F.silu(h) @ w["act.time_out.w"].T + w["act.time_out.b"]
        for i in range(s.n_layers):
            p = f"exp.{i}."
            h = rms_norm(e, w[p + "ln_in"], s.rms_eps)
            if s.is_self_attn(i):
                q, k, v = self.lin(h, p + "qkv").split([nq * hd, nk * hd, nk * hd], dim=-1)
                q = rope(q.reshape(H, nq, hd), self.cos_s, self.sin_s)
                k = rope(k.reshape(H, nk, hd), self.cos_s, self.sin_s)
                kk = torch.cat([cache["k"][i].reshape(L, nk, hd), k], dim=0)
                vv = torch.cat([cache["v"][i].reshape(L, nk, hd), v.reshape(H, nk, hd)], dim=0)
                a = gqa(q, kk, vv, suffix_visibility(L, H))
            else:
                q = rope(self.lin(h, p + "q").reshape(H, nq, hd), self.cos_c, self.sin_c)
                a = gqa(q, cache["kx"][i].reshape(L, nk, hd), cache["vx"][i].reshape(L, nk, hd),
                        None)  # fmt: skip
            e = e + self.lin(a, p + "o")
            h = rms_norm(e, w[p + "ln_post"], s.rms_eps)
            g, u = self.lin(h, p + "gate_up").chunk(2, dim=-1)
            e = e + self.lin(F.silu(g) * u, p + "down")
        e = rms_norm(e, w["exp.norm"], s.rms_eps)
        return e @ w["act.out.w"].T + w["act.out.b"]

    def finish(self, x_t: Tensor, state: Tensor) -> Tensor:
        """Undo the action representation and normalisation (`pkg/model/engine.py:281-291`)."""
        s, w, meta = self.s, self.w, self.b.meta
        a = x_t
        if meta["action_repr"] != "absolute":
            st = (state - w["norm.state.mean"]) / (w["norm.state.std"] + 1e-8)
            st = F.pad(st, (0, s.max_state - st.shape[0]))
            a = a * w["repr.std"] + w["repr.mean"]
            a = a + st[None] if meta["action_repr"] == "delta" else st[None] + torch.cumsum(a, 0)
        return a[:, : meta["action_dim"]] * w["norm.action.std"] + w["norm.action.mean"]

    # -------------------------------------------------------------------- whole chunk
    @torch.no_grad()
    def run(self, images, state, noise, keep: bool = False) -> dict:
        """One chunk. Returns {"actions": (H, action_dim)} and, with keep, the intermediates."""
        s = self.s
        st = torch.as_tensor(np.asarray(state, np.float32))
        px = self.preprocess(images)
        rows_img = self.vision(px)
        rows = self.prefix_rows(rows_img, st)
        cache = self.prefix(rows)
        x_t = torch.as_tensor(np.asarray(noise, np.float32)).reshape(s.chunk, s.max_action)
        v0 = None
        dt = -1.0 / s.n_steps
        for k in range(s.n_steps):
            v = self.velocity(x_t, k, cache)
            if k == 0:
                v0 = v
            x_t = x_t + dt * v
        out = {"actions": self.finish(x_t, st)}
        if keep:
            out.update(px=px, img_rows=rows_img, rows=rows, cache=cache, v0=v0, x_final=x_t)
        return out

    def actions(self, images, state, noise) -> np.ndarray:
        return self.run(images, state, noise)["actions"].numpy()

    @torch.no_grad()
    def calibrate(self, observations) -> dict[str, float]:
        """max |input| of every vision linear over the observations' images, the calibration
        the reference's int8 test runs (`tests/test_ov_engine.py:222-225`)."""
        self.record = {}
        try:
            for images in observations:
                self.vision(self.preprocess(images))
            return dict(self.record)
        finally:
            self.record = None


# ------------------------------------------------------------------------ building blocks
def rope_tables(pos: Tensor, head_dim: int, wavelength: float) -> tuple[Tensor, Tensor]:
    """cos/sin (L, head_dim/2) for integer positions, float32 throughout
    (`pkg/model/smolvla.py:77-85`)."""
    half = head_dim // 2
    exps = (2.0 / head_dim) * torch.arange(half, dtype=torch.float32)
    ang = pos.float()[:, None] / (wavelength**exps)[None, :]
    return torch.cos(ang), torch.sin(ang)


def rope(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """Rotate halves: [x1 c - x2 s, x2 c + x1 s] for x (L, heads, hd) (`pkg/model/smolvla.py:88-94`)."""
    half = x.shape[-1] // 2
    c, s_ = cos[:, None, :], sin[:, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s_, x2 * c + x1 * s_], dim=-1)


def rms_norm(x: Tensor, w: Tensor, eps: float) -> Tensor:
    """x * rsqrt(mean(x^2) + eps) * w (`pkg/model/smolvla.py:72-74`)."""
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def layer_norm(x: Tensor, w: Tensor, b: Tensor, eps: float) -> Tensor:
    mu = x.mean(-1, keepdim=True)
    var = (x - mu).pow(2).mean(-1, keepdim=True)
    return (x - mu) * torch.rsqrt(var + eps) * w + b


def gelu_tanh(x: Tensor) -> Tensor:
    """GELU, tanh approximation: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))."""
    return 0.5 * x * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x**3)))


def softmax_attention(q: Tensor, k: Tensor, v: Tensor, visible: Tensor | None) -> Tensor:
    """softmax(q k^T / sqrt(hd), masked) v over the last two dims."""
    sc = (q @ k.transpose(-1, -2)) / math.sqrt(q.shape[-1])
    if visible is not None:
        sc = sc.masked_fill(~visible, float("-inf"))
    return torch.softmax(sc, dim=-1) @ v


def gqa(q: Tensor, k: Tensor, v: Tensor, visible: Tensor | None) -> Tensor:
    """Grouped-query attention: q (Lq, nq, hd), k/v (Lk, nk, hd); query head h reads kv head
    h // (nq / nk) (`pkg/model/smolvla.py:312-325`). Returns (Lq, nq * hd)."""
    nq, nk = q.shape[1], k.shape[1]
    g = nq // nk
    kk = k.transpose(0, 1).repeat_interleave(g, dim=0)
    vv = v.transpose(0, 1).repeat_interleave(g, dim=0)
    a = softmax_attention(q.transpose(0, 1), kk, vv, visible)
    return a.transpose(0, 1).reshape(q.shape[0], -1)


def prefix_visibility(L: int) -> Tensor:
    """Prefix-LM mask: images and task tokens see each other, the last (state) token sees all,
    nothing else sees it (`pkg/model/engine.py:72-77`)."""
    i = torch.arange(L)[:, None]
    j = torch.arange(L)[None, :]
    return (j < L - 1) | (i == L - 1)


def suffix_visibility(L: int, H: int) -> Tensor:
    """Action rows see the whole prefix and are causal among themselves
    (`pkg/model/engine.py:80-84`)."""
    i = torch.arange(H)[:, None]
    j = torch.arange(L + H)[None, :]
    return (j < L) | (j - L <= i)


def shuffle_tokens(x: Tensor, s: int) -> Tensor:
    """SmolVLM pixel shuffle (n, N, d) -> (n, N/s^2, d s^2): output token (hj, wj), feature
    (hs, ws, c) reads input token (hj*s + hs, wj*s + ws), channel c
    (`pkg/model/smolvla.py:105-114`)."""
    n, N, d = x.shape
    side = int(round(N**0.5))
    x = x.reshape(n, side // s, s, side // s, s, d)  # (n, hj, hs, wj, ws, d)
    x = x.permute(0, 1, 3, 2, 4, 5)  # (n, hj, wj, hs, ws, d)
    return x.reshape(n, N // (s * s), d * s * s)


def time_projection(s: ModelSpec, w: dict[str, Tensor]) -> Tensor:
    """time_in's time half, bias included, for t = 1, 1 - 1/n, ..., 1/n (n_steps, exp_dim)
    (`pkg/model/engine.py:137-141`, sinusoid `pkg/model/smolvla.py:97-102`)."""
    dt = -1.0 / s.n_steps
    # the step times are a float32 tensor upcast for the sinusoid, as the engine builds them
    t = torch.tensor([1.0 + k * dt for k in range(s.n_steps)], dtype=torch.float32).double()
    frac = torch.linspace(0.0, 1.0, s.exp_dim // 2, dtype=torch.float64)
    period = s.min_period * (s.max_period / s.min_period) ** frac
    ang = t[:, None] * (2 * math.pi / period)[None, :]
    temb = torch.cat([torch.sin(ang), torch.cos(ang)], dim=-1).float()
    return temb @ w["act.time_in.w_time"].T + w["act.time_in.b"]
