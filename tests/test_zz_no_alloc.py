"""The allocation-free attention-backward entry point, called through its C symbol.

Some callers of this library cannot allocate device memory: they run inside
another runtime's memory arena or a fixed-budget serving process, or they speak
only a C ABI and own no CUDA allocator. ``pb_attn_bwd_noalloc``
(``priml_b200/ops/csrc/attention_noalloc.h``) serves them: they pass their own
inputs and outputs, and the scratch lives in a static device array inside the
library. These tests call the exported C symbol through ctypes and check its
gradients against both the regular entry point (``native().attn_bwd``) and an
fp32 PyTorch oracle of the same op, on two calls in a row. A larger problem runs
first so that the shared array holds stale, non-zero data when the smaller cases
read it. The file sorts last so a run that stops at the first failure has
already run every other test.
"""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, BAD_ARGUMENT, TOO_LARGE, CUDA_ERROR = 0, 1, 2, 3


def _lib() -> ctypes.CDLL:
    from priml_b200.ops import native

    lib = ctypes.CDLL(native().__file__)
    fn = lib.pb_attn_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_void_p] + [ctypes.c_void_p] * 3 + [ctypes.c_int] * 6 + [
        ctypes.c_float,
        ctypes.c_int,
        ctypes.c_int,
        ctypes.c_void_p,
    ]
    lib.pb_attn_bwd_noalloc_status.restype = ctypes.c_int
    lib.pb_attn_bwd_noalloc_status.argtypes = [ctypes.c_void_p]
    return lib


def _err(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6))


def _call(lib: ctypes.CDLL, q, k, v, o, do, lse, causal: bool, window: int, scale: float):  # noqa: ANN001, ANN202
    B, S, H, D = q.shape
    T, Hkv = k.shape[1], k.shape[2]
    dq = torch.full_like(q, float("nan"))
    dk = torch.full_like(k, float("nan"))
    dv = torch.full_like(v, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.pb_attn_bwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, S, T, H, Hkv, D, scale, int(causal), window, stream,
    )  # fmt: skip
    assert rc == OK
    assert lib.pb_attn_bwd_noalloc_status(stream) == 0
    return dq, dk, dv


@pytest.fixture(scope="module")
def lib() -> ctypes.CDLL:
    """The library, after one large call has left non-zero data across most of the shared array."""
    from priml_b200.ops import native

    lib = _lib()
    torch.manual_seed(9)
    B, S, H, Hkv, D = 4, 1024, 64, 8, 64  # 262,144 rows: half of the array
    q = torch.randn(B, S, H, D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, S, Hkv, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, S, Hkv, D, device="cuda", dtype=torch.bfloat16)
    o, lse = native().attn_fwd(q, k, v, 0.125, True, -1)
    _call(lib, q, k, v, o, torch.randn_like(o), lse, True, -1, 0.125)
    torch.cuda.synchronize()
    return lib


CASES = [
    # B, S, T, H, Hkv, D, causal, window
    (2, 256, 256, 4, 2, 64, True, -1),
    (1, 384, 384, 2, 1, 128, True, -1),
    (1, 200, 200, 4, 2, 64, True, -1),  # S not a multiple of 64: tiles read past S
    (1, 198, 198, 2, 2, 128, True, -1),  # S not a multiple of 4: the non-bulk row path
    (2, 192, 192, 4, 4, 64, False, -1),  # full (non-causal) attention
    (1, 128, 320, 4, 2, 64, True, -1),  # cross-attention, T > S, bottom-right causal mask
    (1, 256, 256, 4, 2, 64, True, 64),  # sliding window
    (1, 198, 262, 2, 1, 64, False, 48),  # window without causality, T > S, S % 4 != 0
]


@pytest.mark.parametrize("B,S,T,H,Hkv,D,causal,window", CASES)
def test_noalloc_matches_regular_entry_point_and_oracle(lib, B, S, T, H, Hkv, D, causal, window) -> None:  # noqa: ANN001
    from priml_b200.ops import native, reference

    torch.manual_seed(0)
    q = torch.randn(B, S, H, D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, T, Hkv, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, T, Hkv, D, device="cuda", dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(D)
    o, lse = native().attn_fwd(q, k, v, scale, causal, window)
    do = torch.randn_like(o)
    dq_nat, dk_nat, dv_nat = native().attn_bwd(q, k, v, o, do, lse, scale, causal, window)

    qr, kr, vr = (t.float().requires_grad_() for t in (q, k, v))
    orf = reference.attention(qr, kr, vr, causal=causal, scale=scale, window=None if window < 0 else window)
    orf.backward(do.float())

    for _ in range(2):  # the second call reads the array exactly as the first left it
        dq, dk, dv = _call(lib, q, k, v, o, do, lse, causal, window, scale)
        for got, nat, ref in ((dq, dq_nat, qr.grad), (dk, dk_nat, kr.grad), (dv, dv_nat, vr.grad)):
            assert torch.isfinite(got).all()
            assert _err(got, nat) < 3e-2
            assert _err(got, ref) < 3e-2


def test_noalloc_rejects_oversized_problem(lib) -> None:  # noqa: ANN001
    x = torch.empty(16, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(16, device="cuda", dtype=torch.float32)
    p = x.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    # B * H * S = 8 * 32 * 4096 rows exceeds the 524288-row array: rejected before any launch.
    rc = lib.pb_attn_bwd_noalloc(p, p, p, p, p, lse.data_ptr(), p, p, p, 8, 4096, 4096, 32, 8, 64, 0.125, 1, -1, stream)
    assert rc == TOO_LARGE
    # unsupported head dimension
    rc = lib.pb_attn_bwd_noalloc(p, p, p, p, p, lse.data_ptr(), p, p, p, 1, 16, 16, 1, 1, 96, 0.1, 1, -1, stream)
    assert rc == BAD_ARGUMENT
