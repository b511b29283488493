"""so101_gemm_static, the GEMM entry point for callers that cannot allocate device memory.

Hosts inside CUDA-graph capture, real-time loops that forbid allocation after start-up, and
foreign-language runtimes that reach the GPU only through this library cannot hand so101_gemm a
workspace. so101_gemm_static keeps its split-K scratch in a file-scope device array instead. This
test calls it through the C ABI twice in a row and checks each result against so101_gemm with a
caller-allocated workspace, on split-K plans that use the scratch, and checks that a plan larger
than the array is refused. It lives in its own file, collected last, and passes alone in a fresh
process or after the rest of the suite.
"""

from __future__ import annotations

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def _bind():
    from so101_smolvla_edge_b200 import _lib as L

    lib = L.lib()
    fn = lib.so101_gemm_static
    fn.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_int64,
                   C.c_int, C.c_int64, C.c_int64, C.c_int64, C.POINTER(L.Epilogue),
                   C.POINTER(L.GemmConfig), C.c_void_p]  # fmt: skip
    fn.restype = C.c_int
    return L, lib, fn


def _close(got, want):
    """The GEMM tests' bound: one rounding to the output dtype plus fp32 accumulation noise."""
    eps = 2**-8 if got.dtype == torch.bfloat16 else 1e-5
    err = (got.float() - want.float()).abs()
    return bool(err.max() <= 2 * eps * want.float().abs().max() + 1e-4)


# flags 1 = SO101_GEMM_GLOBAL_SPLITK: reduce through scratch memory rather than a cluster
@pytest.mark.parametrize("m,n,k,cfg,gate", [
    (50, 720, 2048, (1, 64, 4, 0, 1), False),     # the expert's down projection, split 4 ways
    (50, 2048, 720, (1, 64, 3, 0, 1), True),      # gate_up with the SiLU gate, split 3 ways
    (241, 960, 2560, (0, 128, 5, 0, 1), False),   # prefix down, tokens on the MMA M side
])  # fmt: skip
def test_static_scratch_gemm_matches_workspace_gemm(m, n, k, cfg, gate):
    L, lib, static = _bind()
    from so101_smolvla_edge_b200.ops import workspace

    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * n if gate else n, k, device="cuda", generator=g) * k**-0.5).to(torch.bfloat16)
    r = torch.randn(m, n, device="cuda", generator=g)
    out_dtype = torch.bfloat16 if gate else torch.float32
    epi = L.Epilogue(epilogue=L.EPI_SILU_GATE if gate else L.EPI_NONE,
                     residual=None if gate else r.data_ptr(), ldr=0 if gate else n,
                     r_type=L.F32, out_scale=1.0)  # fmt: skip
    c = L.GemmConfig(*cfg)
    need, tick = C.c_int64(), C.c_int64()
    L.check(lib.so101_gemm_workspace(L.BF16, m, n, k, epi.epilogue, C.byref(c), C.byref(need),
                                     C.byref(tick)), "workspace")  # fmt: skip
    assert need.value > 0, "the plan must use split-K scratch"
    stream = torch.cuda.current_stream().cuda_stream
    ws = workspace(x.device)
    want = torch.empty(m, n, dtype=out_dtype, device="cuda")
    L.check(lib.so101_gemm(L.BF16, x.data_ptr(), k, w.data_ptr(), k, want.data_ptr(), n,
                           L.BF16 if gate else L.F32, m, n, k, C.byref(epi), C.byref(c),
                           ws.partials.data_ptr(), ws.nbytes, ws.tickets.data_ptr(),
                           ws.tickets.numel(), stream), "so101_gemm")  # fmt: skip
    for _ in range(2):  # the scratch keeps the last call's contents: a second call must not care
        got = torch.full((m, n), float("nan"), dtype=out_dtype, device="cuda")
        rc = static(L.BF16, x.data_ptr(), k, w.data_ptr(), k, got.data_ptr(), n,
                    L.BF16 if gate else L.F32, m, n, k, C.byref(epi), C.byref(c), stream)
        assert rc == L.OK
        torch.cuda.synchronize()
        assert _close(got, want)
    assert lib.so101_device_status() == 0


def _both(L, lib, static, a_type, x, w, m, n, k, epi, cfg, out_dtype, y_type):
    """so101_gemm with a caller workspace, then so101_gemm_static twice: (want, [got, got])."""
    from so101_smolvla_edge_b200.ops import workspace

    stream = torch.cuda.current_stream().cuda_stream
    ws = workspace(x.device)
    cp = C.byref(cfg) if cfg is not None else None
    want = torch.empty(m, n, dtype=out_dtype, device="cuda")
    L.check(lib.so101_gemm(a_type, x.data_ptr(), k, w.data_ptr(), k, want.data_ptr(), n, y_type, m, n,
                           k, C.byref(epi), cp, ws.partials.data_ptr(), ws.nbytes,
                           ws.tickets.data_ptr(), ws.tickets.numel(), stream), "so101_gemm")  # fmt: skip
    got = []
    for _ in range(2):
        y = torch.full((m, n), float("nan"), dtype=out_dtype, device="cuda")
        rc = static(a_type, x.data_ptr(), k, w.data_ptr(), k, y.data_ptr(), n, y_type, m, n, k,
                    C.byref(epi), cp, stream)  # fmt: skip
        assert rc == L.OK
        torch.cuda.synchronize()
        got.append(y)
    return want, got


@pytest.mark.parametrize("m,n,k", [(50, 720, 2048), (241, 320, 960), (3072, 768, 768)])
def test_static_scratch_gemm_picks_its_own_plan(m, n, k):
    """cfg = NULL: both entry points pick the plan themselves (the picks reduce split-K inside a
    thread-block cluster, so the scratch is not touched, but the call must still match)."""
    L, lib, static = _bind()
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda", generator=g) * k**-0.5).to(torch.bfloat16)
    epi = L.Epilogue(epilogue=L.EPI_NONE, out_scale=1.0)
    want, got = _both(L, lib, static, L.BF16, x, w, m, n, k, epi, None, torch.float32, L.F32)
    for y in got:
        assert _close(y, want)
    assert lib.so101_device_status() == 0


def test_static_scratch_int8_split_k():
    """W8A8 operands with per-channel weight scales: int32 partials through the static scratch."""
    L, lib, static = _bind()
    m, n, k = 256, 768, 3072  # int8 operands take the tokens-on-M tiles
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randint(-128, 128, (m, k), device="cuda", generator=g, dtype=torch.int32).to(torch.int8)
    w = torch.randint(-127, 128, (n, k), device="cuda", generator=g, dtype=torch.int32).to(torch.int8)
    ws = torch.rand(n, device="cuda", generator=g) * 1e-3 + 1e-4
    epi = L.Epilogue(epilogue=L.EPI_NONE, out_scale=1.0, w_scale=ws.data_ptr(), x_scale=0.02)
    cfg = L.GemmConfig(0, 128, 6, 0, L.GEMM_GLOBAL_SPLITK)
    need, tick = C.c_int64(), C.c_int64()
    L.check(lib.so101_gemm_workspace(L.I8, m, n, k, L.EPI_NONE, C.byref(cfg), C.byref(need),
                                     C.byref(tick)), "workspace")  # fmt: skip
    assert need.value > 0 and tick.value > 0, "the plan must use split-K scratch"
    want, got = _both(L, lib, static, L.I8, x, w, m, n, k, epi, cfg, torch.float32, L.F32)
    exact = (x.double() @ w.double().T) * 0.02 * ws.double()
    assert torch.allclose(want.double(), exact, rtol=1e-5, atol=1e-5)
    for y in got:
        assert torch.equal(y, want)  # integer partials: the sum does not depend on the order
    assert lib.so101_device_status() == 0


def test_static_scratch_refuses_plans_beyond_its_size():
    """A split-K plan needing more than the 8 MiB array is refused with SO101_ERR_WORKSPACE."""
    L, lib, static = _bind()
    m, n, k = 3072, 3072, 4096
    x = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(n, k, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    epi = L.Epilogue(epilogue=L.EPI_NONE, out_scale=1.0)
    c = L.GemmConfig(0, 256, 8, 0, 1)  # 288 tiles x 8 splits x 256 x 128 x 4 B: far beyond 8 MiB
    rc = static(L.BF16, x.data_ptr(), k, w.data_ptr(), k, y.data_ptr(), n, L.BF16, m, n, k,
                C.byref(epi), C.byref(c), torch.cuda.current_stream().cuda_stream)
    assert rc == L.ERR_WORKSPACE
