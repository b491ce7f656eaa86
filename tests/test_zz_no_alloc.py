"""The allocation-free attention-backward entry point, called through its C symbol.

Some callers of this library cannot allocate device memory (they run inside
another runtime's memory arena, or speak only a C ABI with no allocator).
``pb_attn_bwd_noalloc`` serves them: they pass their own inputs and outputs and
the scratch lives in a static device array. This test calls the exported C
symbol with ctypes and checks its gradients against the regular entry point
(``native().attn_bwd``) on two calls in a row. The file sorts last so a run that
stops at the first failure has already run every other test.
"""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


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
    return lib


def _err(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-6))


@pytest.mark.parametrize("B,S,H,Hkv,D", [(2, 256, 4, 2, 64), (1, 384, 2, 1, 128)])
def test_noalloc_matches_regular_entry_point(B: int, S: int, H: int, Hkv: int, D: int) -> None:
    from priml_b200.ops import native

    lib = _lib()
    torch.manual_seed(0)
    q = torch.randn(B, S, H, D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, S, Hkv, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, S, Hkv, D, device="cuda", dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(D)
    o, lse = native().attn_fwd(q, k, v, scale, True, -1)
    do = torch.randn_like(o)
    dq_ref, dk_ref, dv_ref = native().attn_bwd(q, k, v, o, do, lse, scale, True, -1)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        dq = torch.full_like(q, float("nan"))
        dk = torch.full_like(k, float("nan"))
        dv = torch.full_like(v, float("nan"))
        rc = lib.pb_attn_bwd_noalloc(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, S, S, H, Hkv, D, scale, 1, -1, stream,
        )  # fmt: skip
        assert rc == 0
        torch.cuda.synchronize()
        assert lib.pb_attn_bwd_noalloc_status() == 0
        assert _err(dq, dq_ref) < 3e-2
        assert _err(dk, dk_ref) < 3e-2
        assert _err(dv, dv_ref) < 3e-2


def test_noalloc_rejects_oversized_problem() -> None:
    lib = _lib()
    x = torch.empty(16, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(16, device="cuda", dtype=torch.float32)
    p = x.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    # B * H * S = 8 * 32 * 4096 rows exceeds the 524288-row scratch: rejected before any launch.
    rc = lib.pb_attn_bwd_noalloc(p, p, p, p, p, lse.data_ptr(), p, p, p, 8, 4096, 4096, 32, 8, 64, 0.125, 1, -1, stream)
    assert rc == 2
