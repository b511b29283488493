"""ctypes binding of libso101_b200.so (the C ABI declared in include/so101_b200.h).

The library is required: `lib()` raises if the shared object is missing or fails to load, and
there is no other implementation to fall back to. `build.py` produces it in-tree.
"""

from __future__ import annotations

import ctypes as C
import functools
import re
from pathlib import Path

from .build import LIB

HEADER = Path(__file__).resolve().parents[1] / "include" / "so101_b200.h"

OK, ERR_ARG, ERR_LAUNCH, ERR_WORKSPACE, ERR_TIMEOUT, ERR_DRIVER = range(6)
BF16, F32, I8 = 0, 1, 2
EPI_NONE, EPI_GELU, EPI_SILU_GATE = 0, 1, 2
ERRORS = {
    ERR_ARG: "unsupported size, stride, alignment or dtype",
    ERR_LAUNCH: "CUDA launch failed",
    ERR_WORKSPACE: "split-K workspace or tickets too small",
    ERR_TIMEOUT: "a device wait timed out",
    ERR_DRIVER: "cuTensorMapEncodeTiled unavailable",
}


class Epilogue(C.Structure):
    _fields_ = [
        ("epilogue", C.c_int),
        ("bias", C.c_void_p),
        ("residual", C.c_void_p),
        ("ldr", C.c_int64),
        ("r_type", C.c_int),
        ("r_period", C.c_int64),
        ("out_scale", C.c_float),
        ("w_scale", C.c_void_p),
        ("x_scale", C.c_float),
        ("y_qscale", C.c_float),
        ("row_group", C.c_int64),
        ("row_stride", C.c_int64),
        ("rms_ss", C.c_void_p),
        ("rms_slots", C.c_int),
        ("rms_ld", C.c_int64),
        ("rms_n", C.c_float),
        ("rms_eps", C.c_float),
        ("stat_ss", C.c_void_p),
        ("stat_ld", C.c_int64),
        ("y16", C.c_void_p),
        ("ld16", C.c_int64),
        ("y16_scale", C.c_void_p),
    ]


GEMM_GLOBAL_SPLITK, GEMM_PERSISTENT, GEMM_ONE_TILE_PER_CTA, GEMM_PAIR = 1, 2, 4, 8


class GemmConfig(C.Structure):
    _fields_ = [("swap", C.c_int), ("bn", C.c_int), ("splits", C.c_int), ("stages", C.c_int),
                ("flags", C.c_int)]

    def as_tuple(self) -> tuple[int, int, int, int, int]:
        return (self.swap, self.bn, self.splits, self.stages, self.flags)


P, I, I64, F, S = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_void_p  # S: cudaStream_t

EXPERT_MAX_LAYERS = 16


class ExpertLayer(C.Structure):
    """`so101_expert_layer`: one expert layer's weights, norms and K/V rows."""

    _fields_ = [("w_attn", P), ("w_o", P), ("w_gate_up", P), ("w_down", P), ("ln_in", P),
                ("ln_post", P), ("k", P), ("v", P), ("self_attn", C.c_int)]  # fmt: skip


class ExpertStep(C.Structure):
    """`so101_expert_step`: the persistent expert-step kernel's problem."""

    _fields_ = [(n, C.c_int) for n in ("n_layers", "rows", "prefix_len", "exp_dim", "q_dim", "kv_dim",
                                       "n_heads", "n_kv", "head_dim", "mlp_dim")] + [
        ("eps", C.c_float), ("layer", ExpertLayer * EXPERT_MAX_LAYERS), ("e", P), ("q", P), ("attn", P),
        ("act", P), ("cos_self", P), ("sin_self", P), ("cos_cross", P), ("sin_cross", P),
        ("workspace", P), ("workspace_bytes", C.c_int64)]  # fmt: skip

SIGNATURES = {
    "so101_gemm": [I, P, I64, P, I64, P, I64, I, I64, I64, I64, C.POINTER(Epilogue),
                   C.POINTER(GemmConfig), P, I64, P, I64, S],
    "so101_gemm_pick": [I, I64, I64, I64, I, C.POINTER(GemmConfig)],
    "so101_gemm_workspace": [I, I64, I64, I64, I, C.POINTER(GemmConfig), C.POINTER(C.c_int64),
                             C.POINTER(C.c_int64)],
    "so101_attention": [P, I64, P, I64, P, I64, P, I64, I, F, I64, I64, I, I, I, I64, I64, P, P, I,
                        I64, I64, I64, I64, S],
    "so101_attention_rows": [P, I64, P, I64, P, I64, P, I64, I, F, I64, I64, I, I, I, I64, I64, P, P, I,
                             I64, I64, I64, I64, P, P, I64, I64, I64, P, P, S],
    "so101_attention_o": [P, I64, P, I64, P, I64, I64, I64, I, I, I, I64, I64, P, P, I, I64, I64, I64,
                          P, P, I64, I64, I64, P, P, P, I64, I64, P, I64, P, I64, P, I64, P, P, I64, S],
    "so101_mlp": [P, I64, I64, I, I64, P, I, I64, F, P, I64, I64, P, I64, I64, P, I64, P, I64, P, I64, P, P,
                  I64, S],
    "so101_rms_norm": [P, I64, I, P, P, I64, I, I64, I64, F, S],
    "so101_layer_norm": [P, I64, P, P, P, I64, I, F, I64, I64, F, I, I64, S],
    "so101_rope_kv": [P, I64, I, I, I, P, P, P, I64, P, I64, I64, I, I64, I64, I64, S],
    "so101_preprocess": [P, I, I, I, I, I, I, I, P, I, F, S],
    "so101_patchify": [P, I, I, I, P, I, F, S],
    "so101_patch_embed": [P, I, I, P, I64, I64, P, P, I64, P, I64, S],
    "so101_linear_f32": [P, I64, P, I64, P, P, P, I64, I64, I64, I64, I, S],
    "so101_split_bf16x3": [P, I64, I64, I64, P, I64, S],
    "so101_expert_out": [P, I64, P, F, P, P, P, I64, I64, I64, I64, F, S],
    "so101_prefix_tail": [P, I, P, P, P, I, P, P, I, I, P, I64, I64, I64, I, S],
    "so101_finish": [P, I, P, I, P, P, P, P, P, P, P, I, I, I, I, S],
    "so101_absmax": [P, I64, I, I64, I64, P, S],
    "so101_quantize_weight": [P, I, I64, I64, P, P, S],
    "so101_device_status": [],
    "so101_clear_device_status": [],
    "so101_set_pdl": [I],
    "so101_gemm_stat_slots": [I, I64, I64, I64, I, C.POINTER(GemmConfig), C.POINTER(C.c_int)],
    "so101_rms_stats": [P, I64, I64, I64, P, P, I64, P, I64, S],
    "so101_expert_step_workspace": [C.POINTER(ExpertStep), C.POINTER(C.c_int64)],
    "so101_expert_step_run": [C.POINTER(ExpertStep), S],
    "so101_expert_step_test_hooks": [I64, I],
}  # fmt: skip


def header_symbols() -> list[str]:
    """Every function the C header declares."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"SO101_API\s+[\w\s\*]*?\b(so101_\w+)\s*\(", text)))


@functools.cache
def lib() -> C.CDLL:
    """Load the library (raises OSError/RuntimeError if it is missing: there is no fallback)."""
    if not LIB.exists():
        raise RuntimeError(
            f"{LIB} is missing: build it with `python -m so101_smolvla_edge_b200.build`"
        )
    dll = C.CDLL(str(LIB))
    for name, args in SIGNATURES.items():
        fn = getattr(dll, name)
        fn.argtypes = args
        fn.restype = C.c_int
    dll.so101_version.restype = C.c_char_p
    dll.so101_version.argtypes = []
    dll.so101_last_error.restype = C.c_char_p
    dll.so101_last_error.argtypes = []
    return dll


class KernelError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    """Raise on a non-zero status: ValueError for argument errors (as the reference's
    precondition checks), RuntimeError otherwise (as its TensorRT enqueue failure)."""
    if rc == OK:
        return
    msg = f"{what}: {ERRORS.get(rc, f'status {rc}')}"
    if rc == ERR_LAUNCH and LIB.exists():
        cause = lib().so101_last_error().decode()
        if cause:
            msg += f" ({cause})"
    if rc == ERR_ARG:
        raise ValueError(msg)
    raise KernelError(msg)
