"""Newton-Schulz / Polar-Express orthogonalization on the tcgen05 GEMMs.

Muon and NorMuon (``priml/optimizers/normuon.py:309-392``,
``priml/math/numeric.py:299-341``) replace a momentum matrix ``X`` by an
approximation of the orthogonal factor ``U V^T`` of ``X = U S V^T`` through a
few odd-polynomial steps on the wide orientation (``m <= n``):

    A  = Y Y^T                      (m x m, contraction n)
    B  = c A A + b A                (m x m, contraction m)
    Y' = B Y + a Y                  (m x n, contraction m)

On CUDA each step is three launches of the 2-CTA GEMM: the first with a plain
bf16 store, the other two with the scaled-add epilogue (``C = alpha * acc + beta
* X``), so no elementwise pass touches HBM between them and ``A A`` needs no
transpose (``A`` is symmetric, so it is its own K-major ``B`` operand). The
iterate ping-pongs between two buffers because every tile of the next GEMM
still reads the previous one.

A stack of matrices runs as one batched launch per GEMM when both sides are
multiples of 256 (the 2-CTA tile): the tiles of every matrix share one
persistent grid, so a stack of small matrices fills the GPU. Other shapes run
one chain per matrix, spread over a few CUDA streams.

Shapes the 2-CTA tiles cannot take (a side under 256, or not a multiple of 8) and
CPU tensors run the same polynomial in torch.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
from torch import Tensor

__all__ = ["newton_schulz_steps", "newton_schulz_reference"]


def newton_schulz_reference(y: Tensor, coefficients: Sequence[tuple[float, float, float]]) -> Tensor:
    """The polynomial steps in torch on ``[..., m, n]`` (any orientation), in ``y``'s dtype."""
    tall = y.size(-2) > y.size(-1)
    for a, b, c in coefficients:
        if tall:
            gram = y.mT @ y
            y = a * y + y @ (b * gram + c * (gram @ gram))
        else:
            gram = y @ y.mT
            y = a * y + (b * gram + c * (gram @ gram)) @ y
    return y


def native_module():  # noqa: ANN201
    from priml_b200.ops._loader import native

    return native()


def _native_ok(y: Tensor) -> bool:
    from priml_b200.ops._loader import native

    m, n = sorted(y.shape[-2:])
    return (
        y.is_cuda
        and y.dtype == torch.bfloat16
        and m >= 256
        and m % 8 == 0
        and n % 8 == 0
        and hasattr(native(), "gemm_axpby")
    )


def _chain(y: Tensor, coefficients: Sequence[tuple[float, float, float]]) -> Tensor:
    """Steps on one contiguous wide ``[m, n]`` bf16 matrix; returns the final iterate (a new buffer)."""
    from priml_b200.ops._loader import native

    nat = native()
    m = y.shape[0]
    gram = torch.empty(m, m, device=y.device, dtype=torch.bfloat16)
    poly = torch.empty_like(gram)
    cur, nxt = y, torch.empty_like(y)
    for a, b, c in coefficients:
        nat.gemm(cur, cur, gram, False, False, 0)  # A = Y Y^T
        nat.gemm_axpby(gram, gram, gram, poly, False, False, float(c), float(b))  # B = c A A + b A
        nat.gemm_axpby(poly, cur, cur, nxt, False, True, 1.0, float(a))  # Y' = B Y + a Y
        cur, nxt = nxt, cur
    return cur


def _chain_batched(y: Tensor, coefficients: Sequence[tuple[float, float, float]]) -> Tensor:
    """Steps on a contiguous ``[B, m, n]`` stack (m, n multiples of 256): every GEMM is one launch for the stack."""
    from priml_b200.ops._loader import native

    nat = native()
    b, m, _ = y.shape
    gram = torch.empty(b, m, m, device=y.device, dtype=torch.bfloat16)
    poly = torch.empty_like(gram)
    cur, nxt = y, torch.empty_like(y)
    for a, bb, c in coefficients:
        nat.gemm_batched(cur, cur, gram, False, False)  # A = Y Y^T
        nat.gemm_batched(gram, gram, poly, False, False, gram, float(c), float(bb))  # B = c A A + b A
        nat.gemm_batched(poly, cur, nxt, False, True, cur, 1.0, float(a))  # Y' = B Y + a Y
        cur, nxt = nxt, cur
    return cur


def newton_schulz_steps(y: Tensor, coefficients: Sequence[tuple[float, float, float]]) -> Tensor:
    """Apply the ``(a, b, c)`` steps to each matrix of an already normalised ``[..., m, n]`` tensor.

    bf16 CUDA input whose shorter side is at least 256 (both sides multiples of 8)
    runs the tcgen05 GEMM chain; anything else runs :func:`newton_schulz_reference`.
    Returns a new tensor of ``y``'s shape and dtype; ``y`` is left as it was.
    """
    if not _native_ok(y):
        return newton_schulz_reference(y, coefficients)
    shape = y.shape
    tall = shape[-2] > shape[-1]
    mats = y.reshape(-1, *shape[-2:])
    wide = mats.transpose(-2, -1).contiguous() if tall else mats.clone()  # the chain overwrites its input
    out = torch.empty_like(wide)
    m, n = wide.shape[-2:]
    if m % 256 == 0 and n % 256 == 0 and hasattr(native_module(), "gemm_batched"):
        out = _chain_batched(wide, coefficients)
        if tall:
            out = out.transpose(-2, -1)
        return out.reshape(shape)
    pair_tiles = ((m + 255) // 256) * ((n + 255) // 256)
    sms = torch.cuda.get_device_properties(y.device).multi_processor_count
    lanes = max(1, min(len(wide), 8, (sms // 2) // max(1, pair_tiles)))
    if lanes == 1:
        for i in range(len(wide)):
            out[i] = _chain(wide[i], coefficients)
    else:
        main = torch.cuda.current_stream(y.device)
        streams = [torch.cuda.Stream(y.device) for _ in range(lanes)]
        for s in streams:
            s.wait_stream(main)
        for i in range(len(wide)):
            with torch.cuda.stream(streams[i % lanes]):
                out[i].copy_(_chain(wide[i], coefficients))
        for s in streams:
            main.wait_stream(s)
    if tall:
        out = out.transpose(-2, -1)
    return out.reshape(shape)
