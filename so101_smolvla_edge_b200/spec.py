"""SmolVLA architecture constants and parameter table.

The field names, defaults and parameter names are the bundle format of so101-smolvla-edge
(`src/so101_smolvla_edge/model/smolvla.py:25-69` for `ModelSpec`, `:328-397` for the parameter
table), so a bundle written by that project loads here unchanged and the reverse.
"""

from __future__ import annotations

from dataclasses import dataclass, fields


@dataclass
class ModelSpec:
    """SmolVLA on SmolVLM2-500M with a 0.75x action expert (defaults), or a bundle's own sizes."""

    n_cams: int = 3
    image_size: int = 512
    patch: int = 16
    vis_dim: int = 768
    vis_layers: int = 12
    vis_heads: int = 12
    vis_mlp: int = 3072
    vis_eps: float = 1e-6
    shuffle: int = 4
    text_dim: int = 960
    n_layers: int = 16
    n_heads: int = 15
    n_kv: int = 5
    head_dim: int = 64
    text_mlp: int = 2560
    rms_eps: float = 1e-5
    exp_dim: int = 720
    exp_mlp: int = 2048
    self_attn_every: int = 2
    rope_wavelength: float = 10_000.0
    chunk: int = 50
    max_state: int = 32
    max_action: int = 32
    n_steps: int = 10
    min_period: float = 4e-3
    max_period: float = 4.0
    lang_len: int = 0

    @classmethod
    def from_dict(cls, d: dict) -> "ModelSpec":
        known = {f.name for f in fields(cls)}
        return cls(**{k: v for k, v in d.items() if k in known})

    def to_dict(self) -> dict:
        return {f.name: getattr(self, f.name) for f in fields(self)}

    @property
    def grid(self) -> int:
        """Patches per image side."""
        return self.image_size // self.patch

    @property
    def n_patches(self) -> int:
        return self.grid**2

    @property
    def img_tokens(self) -> int:
        """Prefix rows per camera after the pixel shuffle."""
        return self.n_patches // (self.shuffle**2)

    @property
    def prefix_len(self) -> int:
        """Image rows, task-token rows and the one state row."""
        return self.n_cams * self.img_tokens + self.lang_len + 1

    @property
    def qkv_dim(self) -> int:
        return (self.n_heads + 2 * self.n_kv) * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv * self.head_dim

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    def is_self_attn(self, layer: int) -> bool:
        """Expert layer `layer` attends to the prefix and its own rows (else: cross-attends)."""
        return self.self_attn_every > 0 and layer % self.self_attn_every == 0


F32 = "f32"
W = "w"  # the big matrices: stored in the bundle's precision, computed in bf16


def param_shapes(s: ModelSpec) -> dict[str, tuple[tuple[int, ...], str]]:
    """(shape, kind) of every model parameter by bundle name; kind is "w" for the matrices the
    engine runs in bf16 and "f32" for norms, biases, the position table and the small MLPs."""
    out: dict[str, tuple[tuple[int, ...], str]] = {
        "vis.patch.w": ((s.vis_dim, 3 * s.patch * s.patch), W),
        "vis.patch.b": ((s.vis_dim,), F32),
        "vis.pos": ((s.n_patches, s.vis_dim), F32),
        "vis.post_ln.w": ((s.vis_dim,), F32),
        "vis.post_ln.b": ((s.vis_dim,), F32),
        "conn.w": ((s.text_dim, s.vis_dim * s.shuffle**2), W),
        "state.w": ((s.text_dim, s.max_state), F32),
        "state.b": ((s.text_dim,), F32),
        "act.in.w": ((s.exp_dim, s.max_action), F32),
        "act.in.b": ((s.exp_dim,), F32),
        "act.time_in.w_action": ((s.exp_dim, s.exp_dim), F32),
        "act.time_in.w_time": ((s.exp_dim, s.exp_dim), F32),
        "act.time_in.b": ((s.exp_dim,), F32),
        "act.time_out.w": ((s.exp_dim, s.exp_dim), F32),
        "act.time_out.b": ((s.exp_dim,), F32),
        "act.out.w": ((s.max_action, s.exp_dim), F32),
        "act.out.b": ((s.max_action,), F32),
        "exp.norm": ((s.exp_dim,), F32),
    }
    for i in range(s.vis_layers):
        p = f"vis.{i}."
        out.update(
            {
                p + "ln1.w": ((s.vis_dim,), F32),
                p + "ln1.b": ((s.vis_dim,), F32),
                p + "ln2.w": ((s.vis_dim,), F32),
                p + "ln2.b": ((s.vis_dim,), F32),
                p + "qkv.w": ((3 * s.vis_dim, s.vis_dim), W),
                p + "qkv.b": ((3 * s.vis_dim,), F32),
                p + "out.w": ((s.vis_dim, s.vis_dim), W),
                p + "out.b": ((s.vis_dim,), F32),
                p + "fc1.w": ((s.vis_mlp, s.vis_dim), W),
                p + "fc1.b": ((s.vis_mlp,), F32),
                p + "fc2.w": ((s.vis_dim, s.vis_mlp), W),
                p + "fc2.b": ((s.vis_dim,), F32),
            }
        )
    for i in range(s.n_layers):
        t, e = f"txt.{i}.", f"exp.{i}."
        out.update(
            {
                t + "ln_in": ((s.text_dim,), F32),
                t + "ln_post": ((s.text_dim,), F32),
                t + "qkv": ((s.qkv_dim, s.text_dim), W),
                t + "o": ((s.text_dim, s.q_dim), W),
                t + "gate_up": ((2 * s.text_mlp, s.text_dim), W),
                t + "down": ((s.text_dim, s.text_mlp), W),
                e + "ln_in": ((s.exp_dim,), F32),
                e + "ln_post": ((s.exp_dim,), F32),
                e + "o": ((s.exp_dim, s.q_dim), W),
                e + "gate_up": ((2 * s.exp_mlp, s.exp_dim), W),
                e + "down": ((s.exp_dim, s.exp_mlp), W),
            }
        )
        if s.is_self_attn(i):
            out[e + "qkv"] = ((s.qkv_dim, s.exp_dim), W)
        else:
            out[e + "q"] = ((s.q_dim, s.exp_dim), W)
            out[e + "k"] = ((s.kv_dim, s.kv_dim), W)
            out[e + "v"] = ((s.kv_dim, s.kv_dim), W)
    return out


def vision_linear_names(s: ModelSpec) -> list[str]:
    """Names of the vision stage's linears in graph order, as the int8 activation-clip files key
    them (`src/so101_smolvla_edge/model/trt_vision.py:89-99`)."""
    out = ["patch"]
    for i in range(s.vis_layers):
        out += [f"vis.{i}.qkv", f"vis.{i}.out", f"vis.{i}.fc1", f"vis.{i}.fc2"]
    return out + ["conn"]
