"""Kernel micro-benchmarks: ``python -m priml_b200.ops.bench_kernels [--json out.json]``.

Times each kernel with CUDA events on its launching stream after warm-up,
flushing L2 (a 512 MiB write) outside the timed window before every timed
launch, and reports achieved TFLOP/s or GB/s against the measured peaks in
``MEASURED_PEAKS.json`` when present. Shapes are the Llama-1B training step
(16384 tokens = micro-batch 4 x seq 4096, d_model 2048, GQA 32/8 x 64, SwiGLU 8192,
vocab 32768).
"""

from __future__ import annotations

import argparse
import json
from collections.abc import Callable
from pathlib import Path

import torch

PEAKS_FILE = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"


def _peaks() -> tuple[float, float]:
    try:
        d = json.loads(PEAKS_FILE.read_text())
        return float(d["bf16_tflops"]), float(d["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0


def time_fn(fn: Callable[[], object], iters: int = 10, warmup: int = 3) -> float:
    """Median milliseconds per call, L2 flushed before each timed call."""
    flush = torch.empty(512 * 1024 * 1024 // 4, device="cuda", dtype=torch.float32)
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def gemm_cases(tokens: int = 16384) -> list[tuple[str, int, int, int, bool, bool]]:
    """(name, M, N, K, a_mn, b_mn) for the forward, dgrad and wgrad GEMMs."""
    d, hid, vocab, qkv = 2048, 8192, 32768, 3072
    cases = []
    for name, n, k in (("qkv", qkv, d), ("o", d, d), ("up", 2 * hid, d), ("down", d, hid), ("lm_head", vocab, d)):
        cases.append((f"{name}.fwd", tokens, n, k, False, False))
        cases.append((f"{name}.dgrad", tokens, k, n, False, True))
        cases.append((f"{name}.wgrad", n, k, tokens, True, True))
    return cases


def bench_gemms(tokens: int = 16384) -> list[dict]:
    from priml_b200.ops import native

    peak_tf, _ = _peaks()
    n = native()
    rows = []
    for name, m, nn, k, a_mn, b_mn in gemm_cases(tokens):
        a = torch.randn((k, m) if a_mn else (m, k), device="cuda", dtype=torch.bfloat16)
        b = torch.randn((k, nn) if b_mn else (nn, k), device="cuda", dtype=torch.bfloat16)
        wgrad = name.endswith("wgrad")
        c = torch.empty(m, nn, device="cuda", dtype=torch.float32 if wgrad else torch.bfloat16)
        epi = 1 if wgrad else 0
        ours = time_fn(lambda a=a, b=b, c=c, a_mn=a_mn, b_mn=b_mn, epi=epi: n.gemm(a, b, c, a_mn, b_mn, epi))
        at = a.T if a_mn else a
        bt = b if b_mn else b.T
        cub = time_fn(lambda at=at, bt=bt: torch.matmul(at, bt))
        flops = 2.0 * m * nn * k
        rows.append(
            {
                "case": name,
                "M": m,
                "N": nn,
                "K": k,
                "ours_ms": round(ours, 4),
                "ours_tflops": round(flops / ours / 1e9, 1),
                "frac_of_measured_peak": round(flops / ours / 1e9 / peak_tf, 3),
                "cublas_ms": round(cub, 4),
                "speedup_vs_cublas": round(cub / ours, 3),
            }
        )
        del a, b, c
    # fused SwiGLU up-projections (h = silu(x Wg^T) * (x Wu^T), pre-activations kept for backward):
    # the Llama-1B FFN and the 512-wide, K = 512 puzzle-solver FFN (384 x 81 tokens)
    for name, m, h, k in (("up.swiglu", tokens, 8192, 2048), ("puzzle.up.swiglu", 31104, 1536, 512)):
        x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(2 * h, k, device="cuda", dtype=torch.bfloat16) * k**-0.5  # unit-scale pre-activations
        hh = torch.empty(m, h, device="cuda", dtype=torch.bfloat16)
        gu = torch.empty(m, 2 * h, device="cuda", dtype=torch.bfloat16)
        ours = time_fn(lambda x=x, w=w, hh=hh, gu=gu: n.gemm_swiglu(x, w, hh, gu))
        cub = time_fn(lambda x=x, w=w: torch.matmul(x, w.T))
        flops = 2.0 * m * 2 * h * k
        rows.append({"case": name, "M": m, "N": 2 * h, "K": k, "ours_ms": round(ours, 4),
                     "ours_tflops": round(flops / ours / 1e9, 1),
                     "frac_of_measured_peak": round(flops / ours / 1e9 / peak_tf, 3),
                     "out_gb_per_s": round(m * 3 * h * 2 / ours / 1e6, 1),
                     "cublas_ms": round(cub, 4), "speedup_vs_cublas": round(cub / ours, 3)})  # fmt: skip
        del x, w, hh, gu
    # fused SwiGLU backward: dgu = swiglu'(gu) * (dy @ W_down), reading gu and writing dgu ([M, 2H] each)
    for name, m, h, c in (("down.dgrad.swiglu", tokens, 8192, 2048), ("puzzle.down.dgrad.swiglu", 31104, 1536, 512)):
        dy = torch.randn(m, c, device="cuda", dtype=torch.bfloat16)
        wd = torch.randn(c, h, device="cuda", dtype=torch.bfloat16) * c**-0.5
        gu = torch.randn(m, 2 * h, device="cuda", dtype=torch.bfloat16)
        dgu = torch.empty(m, 2 * h, device="cuda", dtype=torch.bfloat16)
        ours = time_fn(lambda dy=dy, wd=wd, gu=gu, dgu=dgu: n.gemm_swiglu_bwd(dy, wd, gu, dgu))
        cub = time_fn(lambda dy=dy, wd=wd: torch.matmul(dy, wd))
        flops = 2.0 * m * h * c
        rows.append({"case": name, "M": m, "N": h, "K": c, "ours_ms": round(ours, 4),
                     "ours_tflops": round(flops / ours / 1e9, 1),
                     "frac_of_measured_peak": round(flops / ours / 1e9 / peak_tf, 3),
                     "io_gb_per_s": round(m * 4 * h * 2 / ours / 1e6, 1),
                     "cublas_ms": round(cub, 4), "speedup_vs_cublas": round(cub / ours, 3)})  # fmt: skip
        del dy, wd, gu, dgu
    for name, m, nn, k in (("puzzle.qkv", 31104, 1536, 512), ("puzzle.down", 31104, 512, 1536)):
        a = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(nn, k, device="cuda", dtype=torch.bfloat16)
        c = torch.empty(m, nn, device="cuda", dtype=torch.bfloat16)
        ours = time_fn(lambda a=a, b=b, c=c: n.gemm(a, b, c, False, False, 0))
        cub = time_fn(lambda a=a, b=b: torch.matmul(a, b.T))
        flops = 2.0 * m * nn * k
        rows.append({"case": name, "M": m, "N": nn, "K": k, "ours_ms": round(ours, 4),
                     "ours_tflops": round(flops / ours / 1e9, 1),
                     "frac_of_measured_peak": round(flops / ours / 1e9 / peak_tf, 3),
                     "cublas_ms": round(cub, 4), "speedup_vs_cublas": round(cub / ours, 3)})  # fmt: skip
        del a, b, c
    return rows


def _scaled_mm_mx(qa: torch.Tensor, sa: torch.Tensor, qb: torch.Tensor, sb: torch.Tensor) -> Callable[[], object] | None:
    """cuBLASLt MXFP8 through torch._scaled_mm on the same bytes (the library baseline), if this torch has it."""
    try:
        a8, b8 = qa.view(torch.float8_e4m3fn), qb.view(torch.float8_e4m3fn)
        sa8, sb8 = sa.view(torch.float8_e8m0fnu), sb.view(torch.float8_e8m0fnu)

        def run() -> object:
            return torch._scaled_mm(a8, b8.t(), scale_a=sa8, scale_b=sb8, out_dtype=torch.bfloat16)  # noqa: SLF001

        run()
        torch.cuda.synchronize()
        return run
    except Exception:  # noqa: BLE001 -- unsupported build / layout: no baseline
        return None


def bench_mx(tokens: int = 16384) -> list[dict]:
    """MXFP8 GEMMs (operands pre-quantized) on the forward-shaped Llama-1B GEMMs, vs our bf16 GEMM
    and cuBLASLt MXFP8; plus the quantizer's bandwidth."""
    from priml_b200.ops import native

    peak_tf, peak_gbs = _peaks()
    n = native()
    rows = []
    for name, m, nn, k, a_mn, b_mn in gemm_cases(tokens):
        if a_mn or b_mn:
            continue  # every MX GEMM reads K-major operands (transposed ones are quantized transposed)
        a = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(nn, k, device="cuda", dtype=torch.bfloat16)
        qa, sa = n.mx_quantize(a, False)
        qb, sb = n.mx_quantize(b, False)
        c = torch.empty(m, nn, device="cuda", dtype=torch.bfloat16)
        mx = time_fn(lambda: n.mx_gemm(qa, sa, qb, sb, c, 0))
        bf = time_fn(lambda: n.gemm(a, b, c, False, False, 0))
        lib = _scaled_mm_mx(qa, sa, qb, sb)
        lib_ms = time_fn(lib) if lib is not None else None
        quant = time_fn(lambda: n.mx_quantize(a, False))
        flops = 2.0 * m * nn * k
        rows.append(
            {
                "case": f"mx.{name}",
                "M": m, "N": nn, "K": k,
                "mx_ms": round(mx, 4),
                "mx_tflops": round(flops / mx / 1e9, 1),
                "frac_of_2x_measured_bf16": round(flops / mx / 1e9 / (2 * peak_tf), 3),
                "frac_of_nominal_fp8_4500": round(flops / mx / 1e9 / 4500.0, 3),
                "our_bf16_ms": round(bf, 4),
                "speedup_vs_our_bf16": round(bf / mx, 3),
                "cublaslt_mxfp8_ms": None if lib_ms is None else round(lib_ms, 4),
                "quantize_ms": round(quant, 4),
                "quantize_frac_of_measured_hbm": round((m * k * 3 + m * k / 32) / quant / 1e6 / peak_gbs, 3),
            }
        )  # fmt: skip
        del a, b, qa, qb, c
    return rows


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", type=str, default="")
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--attn-only", action="store_true")
    ap.add_argument("--gemm-only", action="store_true")
    ap.add_argument("--profile", type=str, default="")
    ap.add_argument("--mx", action="store_true", help="MXFP8 GEMMs and quantizers only")
    ap.add_argument("--decode", action="store_true", help="decode attention kernel and graph-replayed decode steps")
    ap.add_argument("--ns", action="store_true", help="Newton-Schulz / Polar-Express chains vs the torch path")
    ap.add_argument("--gdn", action="store_true", help="gated delta-rule chunk scan vs the torch chunked path")
    ap.add_argument("--mla-decode", action="store_true", help="latent-space MLA decode kernel vs the einsum order")
    args = ap.parse_args()
    if args.mla_decode:
        for r in bench_mla_decode():
            print(json.dumps(r))
        return
    if args.gdn:
        for r in bench_gated_delta():
            print(json.dumps(r))
        return
    if args.ns:
        for r in bench_newton_schulz():
            print(json.dumps(r))
        return
    if args.decode:
        for r in bench_decode():
            print(json.dumps(r))
        return
    if args.profile:
        profile_case(args.profile)
        return
    if args.mx:
        for r in bench_mx(args.tokens):
            print(json.dumps(r))
        return
    rows = bench_gemms(args.tokens) if not args.attn_only else []
    if not args.gemm_only:
        rows += bench_attention()  # Llama-1B: 32 q / 8 kv heads x 64
        rows += bench_attention(b=1, s=8192, h=32, hkv=8, d=128)  # Llama-3-8B: 32 / 8 heads x 128
        rows += bench_attention(b=2, s=4096, h=16, hkv=16, d=192, dv=128)  # MLA: 16 heads, 128+64 / 128
    for r in rows:
        print(json.dumps(r))
    if args.json:
        Path(args.json).write_text(json.dumps(rows, indent=1))


def bench_attention(b: int = 4, s: int = 4096, h: int = 32, hkv: int = 8, d: int = 64, dv: int | None = None) -> list[dict]:
    """Causal GQA attention fwd / fwd+bwd: ours vs torch SDPA (cuDNN / flash)."""
    dv = d if dv is None else dv
    import math as _m

    import torch.nn.functional as F

    from priml_b200.ops.attention_fn import FlashAttnFn

    q = torch.randn(b, s, h, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(b, s, hkv, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(b, s, hkv, dv, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    do = torch.randn(b, s, h, dv, device="cuda", dtype=torch.bfloat16)
    sc = 1 / _m.sqrt(d)
    flops_f = 2.0 * b * h * s * s * (d + dv) / 2
    rows = []

    def ours_f():
        return FlashAttnFn.apply(q, k, v, True, sc, -1)

    def sdpa_f():
        return F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True,
                                              enable_gqa=True)  # fmt: skip

    for name, f in (("ours", ours_f), ("sdpa", sdpa_f)):
        with torch.no_grad():
            t_f = time_fn(f)
        t_fb = time_fn(lambda f=f: torch.autograd.backward(f(), do if name == "ours" else do.transpose(1, 2)))
        rows.append({"case": f"attn.{name}", "B": b, "S": s, "H": h, "Hkv": hkv, "D": d, "Dv": dv, "fwd_ms": round(t_f, 3),
                     "fwd_tflops": round(flops_f / t_f / 1e9, 1), "fwdbwd_ms": round(t_fb, 3),
                     "bwd_tflops": round(2.5 * flops_f / (t_fb - t_f) / 1e9, 1)})  # fmt: skip
    return rows


def bench_newton_schulz() -> list[dict]:
    """Five Polar-Express steps on stacks of momentum matrices: tcgen05 chain vs torch bf16 matmuls (cuBLAS)."""
    from priml_b200.math.numeric import POLAR_EXPRESS_COEFFICIENTS
    from priml_b200.ops.orthogonalize import newton_schulz_reference, newton_schulz_steps

    peak, _ = _peaks()
    rows = []
    # Llama-1B (16 layers): q/o 2048 x 2048, SwiGLU up 16384 x 2048, down 2048 x 8192; nanochat d20: 1280 x 1280, 1280 x 5120
    for b, m, n in ((16, 2048, 2048), (16, 16384, 2048), (16, 2048, 8192), (20, 1280, 1280), (20, 1280, 5120)):
        x = torch.randn(b, m, n, device="cuda")
        y = (x / (x.norm(dim=(-2, -1), keepdim=True) * 1.02 + 1e-6)).to(torch.bfloat16)
        del x
        lo, hi = min(m, n), max(m, n)
        flops = 5 * b * (4.0 * lo * lo * hi + 2.0 * lo**3)
        t_ours = time_fn(lambda: newton_schulz_steps(y, POLAR_EXPRESS_COEFFICIENTS), iters=5)
        t_torch = time_fn(lambda: newton_schulz_reference(y, POLAR_EXPRESS_COEFFICIENTS), iters=5)
        rows.append({"case": "polar_express_5", "batch": b, "m": m, "n": n, "ours_ms": round(t_ours, 3),
                     "torch_ms": round(t_torch, 3), "ours_tflops": round(flops / t_ours / 1e9, 1),
                     "ours_frac_of_bf16_peak": round(flops / t_ours / 1e9 / peak, 3)})  # fmt: skip
    return rows


def bench_decode() -> list[dict]:
    """Decode attention (ours vs SDPA over the same cache) and Llama-1B decode steps (graph vs eager)."""
    import torch.nn.functional as F

    from priml_b200 import ops

    _, hbm = _peaks()
    rows = []
    for b, h, hkv, t, d in ((1, 32, 8, 4096, 64), (16, 32, 8, 4096, 64), (64, 32, 8, 4096, 64), (16, 32, 8, 8192, 128)):
        q = torch.randn(b, h, d, device="cuda", dtype=torch.bfloat16)
        k = torch.randn(b, hkv, t, d, device="cuda", dtype=torch.bfloat16)
        v = torch.randn(b, hkv, t, d, device="cuda", dtype=torch.bfloat16)
        lengths = torch.full((b,), t, device="cuda", dtype=torch.int32)
        nbytes = 2 * k.numel() * 2
        t_ours = time_fn(lambda: ops.decode_attention(q, k, v, lengths), iters=20)
        t_sdpa = time_fn(lambda: F.scaled_dot_product_attention(q[:, :, None], k, v, enable_gqa=True), iters=20)
        rows.append({"case": "decode_attn", "B": b, "H": h, "Hkv": hkv, "T": t, "D": d, "ours_us": round(1e3 * t_ours, 1),
                     "sdpa_us": round(1e3 * t_sdpa, 1), "ours_gbs": round(nbytes / t_ours / 1e6, 1),
                     "ours_frac_hbm": round(nbytes / t_ours / 1e6 / hbm, 3)})  # fmt: skip

    from priml_b200.inference import Decoder
    from priml_b200.models.presets import llama_1b

    torch.manual_seed(0)
    model = llama_1b().make().cuda().to(torch.bfloat16).eval()
    for batch, ctx in ((1, 1024), (64, 1024)):
        for graph in (True, False):
            dec = Decoder(model, batch=batch, max_seq=ctx + 64, cuda_graph=graph)
            dec.prefill(torch.randint(0, 32768, (batch, ctx), device="cuda"))
            tok = torch.zeros(batch, dtype=torch.long, device="cuda")
            for _ in range(3):
                dec.step(tok)
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n = 32
            s.record()
            for _ in range(n):
                dec.step(tok)
            e.record()
            torch.cuda.synchronize()
            ms = s.elapsed_time(e) / n
            rows.append({"case": "llama1b_decode_step", "batch": batch, "context": ctx, "cuda_graph": graph,
                         "ms_per_step": round(ms, 3), "tokens_per_s": round(batch * 1e3 / ms, 1)})  # fmt: skip
            del dec
    return rows


def bench_mla_decode() -> list[dict]:
    """Latent-space MLA decode (one token per sequence, 512 latent + 64 rotary) against the einsum
    order on the same bf16 cache; bytes = the cache rows read once (c_kv and k_pe)."""
    from priml_b200 import ops
    from priml_b200.ops import reference

    _, hbm = _peaks()
    rows = []
    for b, h, t in ((1, 16, 4096), (16, 16, 4096), (64, 16, 4096), (16, 16, 32768), (16, 128, 4096)):
        q = torch.randn(b, h, 576, device="cuda", dtype=torch.bfloat16)
        c = torch.randn(b, t, 512, device="cuda", dtype=torch.bfloat16)
        r = torch.randn(b, t, 64, device="cuda", dtype=torch.bfloat16)
        scale = 192**-0.5
        nbytes = (c.numel() + r.numel()) * 2
        t_ours = time_fn(lambda: ops.mla_decode(q, c, r, scale=scale), iters=20)
        t_ref = time_fn(lambda: reference.mla_decode(q, c, r, scale=scale), iters=5)
        rows.append({"case": "mla_decode", "B": b, "H": h, "T": t, "ours_us": round(1e3 * t_ours, 1),
                     "einsum_us": round(1e3 * t_ref, 1), "ours_gbs": round(nbytes / t_ours / 1e6, 1),
                     "ours_frac_hbm": round(nbytes / t_ours / 1e6 / hbm, 3)})  # fmt: skip
    return rows


def bench_gated_delta(b: int = 4, s: int = 4096, h: int = 16, d: int = 128) -> list[dict]:
    """Gated delta rule forward and forward + backward: chunk scan kernels against the torch chunked path."""
    from priml_b200.models.gated_delta_net import gated_delta_chunked
    from priml_b200.ops.gated_delta import gated_delta_rule

    torch.manual_seed(0)
    q = torch.randn(b, s, h, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn_like(q, requires_grad=True)
    v = torch.randn_like(q, requires_grad=True)
    g = (-torch.rand(b, s, h, device="cuda") * 2).requires_grad_()
    beta = torch.rand(b, s, h, device="cuda").requires_grad_()
    do = torch.randn_like(q)
    rows = []
    for name, fn in (("kernel", gated_delta_rule), ("torch_chunked", gated_delta_chunked)):
        def fwd() -> object:
            with torch.no_grad():
                return fn(q, k, v, g, beta)

        def fwd_bwd() -> object:
            o = fn(q, k, v, g, beta)
            return torch.autograd.grad(o, (q, k, v, g, beta), do)

        rows.append({"op": "gated_delta", "impl": name, "shape": [b, s, h, d], "fwd_ms": round(time_fn(fwd, iters=5), 3),
                     "fwd_bwd_ms": round(time_fn(fwd_bwd, iters=5), 3)})  # fmt: skip
    return rows


def profile_case(name: str) -> None:
    """Run one small instance of a kernel a few times (for an external profiler)."""
    from priml_b200.ops import native
    from priml_b200.ops.attention_fn import FlashAttnFn

    n = native()
    if name == "gdn":
        # one forward and one backward chunk scan: 64 batch-heads x 32 chunks of 128 tokens
        from priml_b200.ops.gated_delta import gated_delta_rule

        q = torch.randn(4, 4096, 16, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        g = -torch.rand(4, 4096, 16, device="cuda")
        beta = torch.rand(4, 4096, 16, device="cuda")
        for _ in range(2):
            o = gated_delta_rule(q, q, q, g, beta)
            o.backward(torch.ones_like(o))
    elif name == "mla_decode":
        # latent-space MLA decode: 64 sequences x 4096 cached tokens, 16 heads (302 MB of cache)
        from priml_b200 import ops

        q = torch.randn(64, 16, 576, device="cuda", dtype=torch.bfloat16)
        c = torch.randn(64, 4096, 512, device="cuda", dtype=torch.bfloat16)
        r = torch.randn(64, 4096, 64, device="cuda", dtype=torch.bfloat16)
        for _ in range(3):
            ops.mla_decode(q, c, r, scale=192**-0.5)
    elif name == "gemm":
        a = torch.randn(8192, 2048, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(8192, 2048, device="cuda", dtype=torch.bfloat16)
        c = torch.empty(8192, 8192, device="cuda", dtype=torch.bfloat16)
        for _ in range(3):
            n.gemm(a, b, c, False, False, 0)
    elif name == "mx_gemm":
        a = torch.randn(8192, 2048, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(8192, 2048, device="cuda", dtype=torch.bfloat16)
        c = torch.empty(8192, 8192, device="cuda", dtype=torch.bfloat16)
        qa, sa = n.mx_quantize(a, False)
        qb, sb = n.mx_quantize(b, False)
        for _ in range(3):
            n.mx_gemm(qa, sa, qb, sb, c, 0)
    elif name == "swiglu_bwd":
        # the SwiGLU-backward GEMM of a 512-wide FFN over 16384 tokens (K = 512: epilogue-bound)
        dy = torch.randn(16384, 512, device="cuda", dtype=torch.bfloat16)
        wd = torch.randn(512, 1536, device="cuda", dtype=torch.bfloat16) * 512**-0.5
        gu = torch.randn(16384, 3072, device="cuda", dtype=torch.bfloat16)
        dgu = torch.empty(16384, 3072, device="cuda", dtype=torch.bfloat16)
        for _ in range(3):
            n.gemm_swiglu_bwd(dy, wd, gu, dgu)
    elif name == "memory":
        # the memory-bound kernels of a training / decode step, each twice, on inputs larger than L2
        from priml_b200 import ops
        from priml_b200.models.rope import RoPE
        from priml_b200.ops import functional as fn

        x = torch.randn(65536, 2048, device="cuda", dtype=torch.bfloat16, requires_grad=True)  # 256 MiB
        d = torch.randn_like(x, requires_grad=True)
        w = torch.ones(2048, device="cuda", requires_grad=True)
        for _ in range(2):
            h, y = ops.add_rms_norm(x, d, w, 1e-5)
            torch.autograd.backward((h, y), (torch.ones_like(h), torch.ones_like(y)))
        del x, d, h, y
        q = torch.randn(16, 4096, 32, 64, device="cuda", dtype=torch.bfloat16)  # 256 MiB
        k = torch.randn(16, 4096, 8, 64, device="cuda", dtype=torch.bfloat16)
        cos, sin = RoPE.Config(64, base=5e5).make().to("cuda").table(4096, torch.device("cuda"))
        for _ in range(2):
            ops.rotary(q, k, cos, sin)
        del q, k
        logits = torch.randn(16384, 32768, device="cuda", dtype=torch.bfloat16, requires_grad=True)  # 1 GiB
        t = torch.randint(0, 32768, (16384,), device="cuda")
        for _ in range(2):
            ops.cross_entropy(logits, t).sum().backward()
        del logits
        xm = torch.randn(16384, 8192, device="cuda", dtype=torch.bfloat16)
        for _ in range(2):
            n.mx_quantize(xm, False)
        del xm
        qd = torch.randn(64, 32, 64, device="cuda", dtype=torch.bfloat16)
        kc = torch.randn(64, 8, 4096, 64, device="cuda", dtype=torch.bfloat16)  # 2 x 256 MiB
        vc = torch.randn_like(kc)
        lengths = torch.full((64,), 4096, device="cuda", dtype=torch.int32)
        for _ in range(2):
            ops.decode_attention(qd, kc, vc, lengths)
        del kc, vc
        e, rows, c, hid = 8, 16384, 2048, 1024
        xs = torch.randn(rows, c, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        up = (torch.randn(e, 2 * hid, c, device="cuda") * c**-0.5).requires_grad_()
        down = (torch.randn(e, c, hid, device="cuda") * hid**-0.5).requires_grad_()
        offsets = torch.arange(0, rows + 1, rows // e, device="cuda", dtype=torch.int32)
        for _ in range(2):
            fn.grouped_swiglu_mlp(xs, up, down, offsets).sum().backward()
        del xs, up, down
        from priml_b200.optimizers import FusedAdamW

        params = [torch.nn.Parameter(torch.randn(4096, 4096, device="cuda")) for _ in range(4)]  # 64 M params
        for p in params:
            p.grad = torch.randn_like(p)
        opt = FusedAdamW(params, lr=1e-3)
        for _ in range(2):
            opt.step()
    elif name in ("attn_fwd", "attn_bwd"):
        q = torch.randn(1, 4096, 32, 64, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        k = torch.randn(1, 4096, 8, 64, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        v = torch.randn(1, 4096, 8, 64, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        for _ in range(2):
            o = FlashAttnFn.apply(q, k, v, True, 0.125, -1)
            if name == "attn_bwd":
                o.backward(torch.ones_like(o))
    torch.cuda.synchronize()


if __name__ == "__main__":
    main()
