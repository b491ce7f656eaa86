"""Math library against independent oracles (SciPy, NumPy, explicit loops)."""

from __future__ import annotations

import math

import numpy as np
import pytest
import scipy.fft as sfft
import scipy.special as sp
import scipy.stats as st
import torch

import priml_b200.math.diffusion as D
from priml_b200.math import advantage as A
from priml_b200.math import frequency as Fq
from priml_b200.math import numeric as N
from priml_b200.math import pixel as Px
from priml_b200.math import pooling as Pl
from priml_b200.math import probability as P
from priml_b200.math import stats as S
from priml_b200.math import tensor as Tn
from priml_b200.testing import run_ranks

f64 = torch.float64


def test_gae_and_q_lambda_match_sequential_loops() -> None:
    g = torch.Generator().manual_seed(0)
    T, E, K = 37, 5, 4
    r = torch.randn(T, E, generator=g, dtype=f64)
    v = torch.randn(T, E, generator=g, dtype=f64)
    d = (torch.rand(T, E, generator=g) < 0.15).to(f64)
    last = torch.randn(E, generator=g, dtype=f64)
    adv, tgt = A.generalized_advantage(rewards=r, values=v, dones=d, last_value=last, discount=0.97, trace_decay=0.9)
    ref = torch.zeros_like(v)
    running = torch.zeros(E, dtype=f64)
    nxt = last
    for t in range(T - 1, -1, -1):
        delta = r[t] + 0.97 * nxt * (1 - d[t]) - v[t]
        running = delta + 0.97 * 0.9 * (1 - d[t]) * running
        ref[t] = running
        nxt = v[t]
    assert torch.allclose(adv, ref, atol=1e-12) and torch.allclose(tgt, ref + v)

    q = torch.randn(T + 1, E, K, generator=g, dtype=f64)
    got = A.q_lambda_targets(rewards=r, q_values=q, dones=d, discount=0.99, trace_decay=0.65)
    greedy = q.max(-1).values
    want = torch.zeros_like(r)
    carried = r[-1] + 0.99 * (1 - d[-1]) * greedy[-1]
    want[-1] = carried
    for t in range(T - 2, -1, -1):
        boot = r[t] + 0.99 * (1 - d[t]) * greedy[t + 1]
        carried = boot + 0.99 * 0.65 * (1 - d[t]) * (carried - greedy[t + 1])
        want[t] = torch.where(d[t].bool(), r[t], carried)
        carried = want[t]
    assert torch.allclose(got, want, atol=1e-12)
    with pytest.raises(ValueError):
        A.q_lambda_targets(rewards=r, q_values=q[:-1], dones=d, discount=0.9, trace_decay=0.5)
    assert float(A.explained_variance(v, v)) == 1.0
    assert float(A.explained_variance(v, torch.ones_like(v))) == 0.0


def test_stats_against_numpy_and_scipy() -> None:
    g = torch.Generator().manual_seed(1)
    x = torch.randn(50, 4, generator=g, dtype=f64)
    y = torch.randn(50, 3, generator=g, dtype=f64)
    assert np.allclose(S.cov(x).numpy(), np.cov(x.numpy(), rowvar=False, bias=True))
    assert np.allclose(S.cov(x, bias=False).numpy(), np.cov(x.numpy(), rowvar=False))
    full = np.cov(np.concatenate([x.numpy(), y.numpy()], 1), rowvar=False, bias=True)
    assert np.allclose(S.cov(x, y).numpy(), full[:4, 4:])
    assert abs(float(S.cov(x[:, 0])) - float(np.var(x[:, 0].numpy()))) < 1e-12
    logits = torch.randn(6, 9, generator=g, dtype=f64)
    p = torch.softmax(logits, -1)
    assert np.allclose(S.entropy_logits(logits).numpy(), st.entropy(p.numpy(), axis=-1))
    assert np.allclose(S.entropy_probs(p).numpy(), st.entropy(p.numpy(), axis=-1))
    lp = torch.log_softmax(torch.randn(3, 6, 9, generator=g, dtype=f64), -1)
    j = S.jsd(lp, ensemble_dim=0, event_dim=-1)
    assert j.shape == (6,) and bool((j >= -1e-12).all())
    assert float(S.jsd(torch.stack([lp[0], lp[0]]), ensemble_dim=0).abs().max()) < 1e-12
    data = torch.randn(400, 5, generator=g, dtype=f64) @ torch.randn(5, 5, generator=g, dtype=f64)
    vals, vecs = S.pca(data)
    ref = np.linalg.eigvalsh(np.cov(data.numpy(), rowvar=False, bias=True))
    assert np.allclose(vals.numpy(), ref, rtol=1e-4)
    v2, _ = S.pca(data, decompose=S.pca_svd)
    v3, _ = S.pca(data, decompose=S.pca_power)
    assert np.allclose(v2.numpy(), ref, rtol=1e-4) and np.allclose(v3.numpy(), ref, rtol=1e-3)
    _, w = S.pca(data, whiten=True, eps=0.0)
    centered = (data - data.mean(0)).float()
    assert torch.allclose(torch.cov((centered @ w).T, correction=0), torch.eye(5), atol=1e-3)
    qn = S.quantile_normalize(torch.randn(1000, generator=g))
    assert float(qn.min()) == 0.0 and float(qn.max()) == 1.0
    win = S.SlidingWindow(window_sec=10.0, pseudocount=0.0, pseudotime=0.0)
    for t in range(20):
        win.add(float(t), 5.0 * t)
    assert abs(win.compute_rate(19.0, 95.0) - 5.0) < 1e-9


def test_probability_against_scipy() -> None:
    x = torch.linspace(-4, 4, 17, dtype=f64)
    assert np.allclose(P.pdf_normal(x, 0.5, 2.0).numpy(), st.norm.pdf(x.numpy(), 0.5, 2.0))
    assert np.allclose(P.cdf_normal(x, 0.5, 2.0).numpy(), st.norm.cdf(x.numpy(), 0.5, 2.0))
    pr = torch.linspace(0.01, 0.99, 9, dtype=f64)
    assert np.allclose(P.quantile_normal(pr, loc=0.5, scale=2.0).numpy(), st.norm.ppf(pr.numpy(), 0.5, 2.0))
    u = torch.linspace(0.02, 0.98, 9, dtype=f64)
    logit = np.log(u.numpy() / (1 - u.numpy()))
    assert np.allclose(P.cdf_logit_normal(u, 0.3, 0.7).numpy(), st.norm.cdf(logit, 0.3, 0.7))
    assert np.allclose(P.pdf_logit_normal(u, 0.3, 0.7).numpy(),
                       st.norm.pdf(logit, 0.3, 0.7) / (u.numpy() * (1 - u.numpy())))  # fmt: skip
    assert np.allclose(P.quantile_logit_normal(P.cdf_logit_normal(u, 0.3, 0.7), 0.3, 0.7).numpy(), u.numpy())
    a, b = (-1.0 - 0.3) / 1.5, (2.0 - 0.3) / 1.5
    tn = st.truncnorm(a, b, loc=0.3, scale=1.5)
    z = torch.linspace(-0.9, 1.9, 8, dtype=f64)
    assert np.allclose(P.cdf_truncated_normal(z, loc=0.3, scale=1.5, low=-1.0, high=2.0).numpy(), tn.cdf(z.numpy()))
    assert np.allclose(P.log_cdf_truncated_normal(z, loc=0.3, scale=1.5, low=-1.0, high=2.0).numpy(),
                       tn.logcdf(z.numpy()))  # fmt: skip
    assert np.allclose(P.quantile_truncated_normal(pr, loc=0.3, scale=1.5, low=-1.0, high=2.0).numpy(),
                       tn.ppf(pr.numpy()))  # fmt: skip
    # far tail: scipy's truncnorm with both bounds in the upper tail
    tail = st.truncnorm(6.0, 9.0)
    assert np.allclose(P.cdf_truncated_normal(torch.tensor([6.5, 7.0], dtype=f64), low=6.0, high=9.0).numpy(),
                       tail.cdf([6.5, 7.0]))  # fmt: skip
    xs = torch.tensor([0.3, 2.0, 9.0, 50.0, 400.0], dtype=f64)
    ys = torch.tensor([0.7, 10.0, 12.0, 60.0, 3.0], dtype=f64)
    assert np.allclose(P.lbeta(xs, ys).numpy(), sp.betaln(xs.numpy(), ys.numpy()), rtol=1e-12, atol=1e-12)
    big = torch.tensor([8.0, 30.0, 1e4], dtype=f64)
    assert np.allclose(P.log_gamma_difference(torch.tensor([0.5, 3.0, 7.0], dtype=f64), big).numpy(),
                       sp.gammaln(big.numpy()) - sp.gammaln(big.numpy() + [0.5, 3.0, 7.0]), rtol=1e-12)  # fmt: skip
    corr = P.log_gamma_correction(big)
    stirling = (big - 0.5) * torch.log(big) - big + 0.5 * math.log(2 * math.pi)
    assert np.allclose((stirling + corr).numpy(), sp.gammaln(big.numpy()), rtol=1e-14)
    assert np.allclose(P.ndtri(P.ndtr(x)).numpy(), x.numpy())


def test_samplers_have_the_right_moments() -> None:
    torch.manual_seed(0)
    g = P.random_gamma(200_000, concentration=torch.tensor([0.5, 3.0]), rate=2.0)
    assert g.shape == (200_000, 2)
    assert torch.allclose(g.mean(0), torch.tensor([0.25, 1.5]), rtol=0.02)
    c = P.random_chi2(200_000, df=4.0)
    assert abs(float(c.mean()) - 4.0) < 0.05
    t = P.random_student_t(200_000, df=10.0, loc=1.0, scale=2.0)
    assert abs(float(t.mean()) - 1.0) < 0.03 and abs(float(t.var()) - 4.0 * 10 / 8) < 0.15
    k = P.random_categorical(100_000, probs=torch.tensor([0.2, 0.5, 0.3]))
    freq = torch.bincount(k, minlength=3).float() / k.numel()
    assert torch.allclose(freq, torch.tensor([0.2, 0.5, 0.3]), atol=0.01)
    with pytest.raises(ValueError):
        P.random_categorical(3)
    ln = P.random_logit_normal(100_000, loc=0.0, scale=1.0)
    assert abs(float(ln.mean()) - 0.5) < 0.01


def test_numeric_helpers() -> None:
    x = torch.tensor([-1e-10, -0.3, -0.7, -30.0], dtype=f64)
    assert np.allclose(N.log1mexp(x).numpy(), np.log(-np.expm1(x.numpy())))
    assert np.allclose(N.logsubexp(torch.tensor(2.0, dtype=f64), torch.tensor(1.0, dtype=f64)).numpy(),
                       math.log(math.e**2 - math.e))  # fmt: skip
    v, s = N.logsubexp(torch.tensor(1.0), torch.tensor(2.0), return_sign=True)
    assert float(s) == -1.0
    y = torch.tensor([-40.0, -3.0, 0.0, 2.0, 30.0], dtype=f64)
    assert np.allclose(N.log_arctan_exp(y).numpy()[1:], np.log(np.arctan(np.exp(y.numpy()[1:]))))
    assert abs(float(N.log_arctan_exp(y)[0]) + 40.0) < 1e-12
    w = torch.tensor([-30.0, -2.0, 0.0, 0.4], dtype=f64)
    assert np.allclose(N.log_tan_exp(w).numpy()[1:], np.log(np.tan(np.exp(w.numpy()[1:]))))
    assert np.allclose(N.logerfc(torch.tensor([-2.0, 0.0, 3.0, 30.0], dtype=f64)).numpy(),
                       np.log(sp.erfc([-2.0, 0.0, 3.0])).tolist() + [math.log(sp.erfcx(30.0)) - 900.0])  # fmt: skip
    z = torch.linspace(-5, 5, 11, dtype=f64)
    assert np.allclose(N.log_cosh(z).numpy(), np.log(np.cosh(z.numpy())))
    assert np.allclose(torch.nn.functional.softplus(N.softplus_inverse(torch.tensor([0.1, 2.0, 9.0]))).numpy(),
                       [0.1, 2.0, 9.0], rtol=1e-5)  # fmt: skip
    assert np.allclose(N.log1psquare(z).numpy(), np.log1p(z.numpy() ** 2))
    assert np.allclose(N.smoothstep(N.smoothstep_inverse(torch.linspace(0, 1, 11, dtype=f64))).numpy(),
                       np.linspace(0, 1, 11))  # fmt: skip
    assert float(N.kahan_sum(torch.tensor([1e8, 1.0, -1e8], dtype=torch.float32))) == 1.0
    assert N.mesh_arange((2, 3)).tolist() == [[0, 0], [0, 1], [0, 2], [1, 0], [1, 1], [1, 2]]
    assert torch.allclose(N.softmax_centered_inverse(N.softmax_centered(z[:4])), z[:4])
    assert torch.allclose(N.sinh_arcsinh_inverse(N.sinh_arcsinh(z, 0.3, 1.7), 0.3, 1.7), z)
    assert torch.allclose(N.power_transform_inverse(N.power_transform(z[5:], 0.5), 0.5), z[5:])
    xr = torch.tensor([0.4, 1.6], requires_grad=True)
    N.ste_round(xr).sum().backward()
    assert torch.equal(xr.grad, torch.ones(2))
    q = torch.tensor([-1.0, 0.0, 4.0], requires_grad=True)
    out = N.safe_sqrt(q) + N.safe_log(q.clamp_min(0.0) + 1.0)
    out.sum().backward()
    assert torch.isfinite(q.grad).all()
    assert N.safe_pow(torch.tensor([0.0, 0.0, -2.0, 4.0]), torch.tensor([0.0, 2.0, 0.5, 0.5])).tolist() == [1.0, 0.0, 0.0, 2.0]
    assert N.safe_rsqrt(torch.tensor([0.0, -1.0, 4.0])).tolist() == [math.inf, 0.0, 0.5]


def test_dct_against_scipy() -> None:
    x = torch.randn(4, 6, 10, dtype=f64)
    assert np.allclose(Fq.dct1d(x).numpy(), sfft.dct(x.numpy(), type=2))
    assert np.allclose(Fq.dct1d(x, normalize=True).numpy(), sfft.dct(x.numpy(), type=2, norm="ortho"))
    assert np.allclose(Fq.idct1d(Fq.dct1d(x)).numpy(), x.numpy())
    assert np.allclose(Fq.dctnd(x, axis=(1, 2), normalize=True).numpy(),
                       sfft.dctn(x.numpy(), type=2, axes=(1, 2), norm="ortho"))  # fmt: skip
    assert np.allclose(Fq.idctnd(Fq.dctnd(x)).numpy(), x.numpy())


def test_pooling_pad_and_tensor_helpers() -> None:
    torch.manual_seed(0)
    x = torch.randn(64, 2, 12, 9)
    assert torch.allclose(Pl.adaptive_avg_pool2d(x, (5, 4)), torch.nn.functional.adaptive_avg_pool2d(x, (5, 4)))
    vp = Pl.adaptive_avg_pool2d(x, (5, 4), variance_preserving=True)
    assert abs(float(vp.var()) - 1.0) < 0.1
    even = Pl.adaptive_avg_pool2d(x[..., :8], (4, 4), variance_preserving=True)
    assert torch.allclose(even, torch.nn.functional.avg_pool2d(x[..., :8], (3, 2)) * math.sqrt(6), atol=1e-6)
    v3 = Pl.adaptive_avg_pool3d(torch.randn(2, 3, 7, 6, 5), (3, 2, 2), variance_preserving=True)
    assert v3.shape == (2, 3, 3, 2, 2)
    short = torch.arange(3.0)[None, None]
    padded = Tn.pad(short, [5, 5], mode="reflect_replicate")
    assert padded.shape[-1] == 13 and padded[0, 0, 5:8].tolist() == [0.0, 1.0, 2.0]
    long = torch.arange(10.0)[None, None]
    assert torch.equal(Tn.pad(long, [3, 2], mode="reflect_replicate"),
                       torch.nn.functional.pad(long, [3, 2], mode="reflect"))  # fmt: skip
    assert Tn.as_batch_tensor(torch.zeros(3, 4)).shape == (1, 1, 3, 4)
    assert Tn.as_batch_tensor(torch.zeros(2, 3, 4, 5, 6, 7)).shape == (6, 4, 5, 6, 7)
    sc = Tn.scale_and_shift(torch.tensor([0, 255], dtype=torch.uint8), torch.tensor(-1.0), torch.tensor(2 / 255))
    assert torch.allclose(sc, torch.tensor([-1.0, 1.0]))


def test_pixel_helpers() -> None:
    import einops

    x = torch.randn(2, 3, 4, 6, 8)
    assert torch.equal(Px.patchify(x, (2, 3, 2)),
                       einops.rearrange(x, "b c (f a) (h p) (w q) -> b (c a p q) f h w", a=2, p=3, q=2))  # fmt: skip
    assert torch.equal(Px.unpatchify(Px.patchify(x, (2, 2)), (2, 2)), x)
    img = torch.tensor([0.0, 127.5, 255.0])
    assert torch.allclose(Px.rgb2float(img), torch.tensor([-1.0, 0.0, 1.0]))
    assert Px.float2rgb(Px.rgb2float(img)).tolist() == [0, 127, 255]
    shapes = Px.compute_video_shapes()
    assert shapes.pixel_full.height == 1080 and shapes.pixel_full.width == 1920
    assert shapes.latent == Px.VideoShape(19, 68, 120)
    assert Px.interpolate(torch.randn(7, 3, 16, 16), "linear", size=(8, 8)).shape == (7, 3, 8, 8)
    assert Px.interpolate(torch.randn(2, 5, 3, 8, 8, 8), "linear", scale_factor=(2, 1, 1)).shape == (2, 5, 3, 16, 8, 8)
    cl = Px.interpolate(torch.randn(2, 8, 8, 3), "nearest", size=(4, 4), channels_last=True)
    assert cl.shape == (2, 4, 4, 3)


def test_diffusion_schedules_targets_and_sampler() -> None:
    ls = torch.linspace(-6, 6, 7, dtype=f64)
    for to_sigma, from_sigma in (
        (D.log_sigma_from_log_snr_per_variance_preserving, D.log_snr_from_log_sigma_per_variance_preserving),
        (D.log_sigma_from_log_snr_per_rectified_flow, D.log_snr_from_log_sigma_per_rectified_flow),
    ):
        assert torch.allclose(from_sigma(log_sigma=to_sigma(ls)), ls)
        assert torch.allclose(from_sigma(sigma=to_sigma(ls).exp()), ls)
    # alpha^2 + sigma^2 = 1 and alpha + sigma = 1
    a_vp = D.compute_log_alpha(ls, D.log_sigma_from_log_snr_per_variance_preserving(ls)).exp()
    assert torch.allclose(a_vp**2 + D.log_sigma_from_log_snr_per_variance_preserving(ls).exp() ** 2,
                          torch.ones_like(ls))  # fmt: skip
    lsr = D.log_sigma_from_log_snr_per_rectified_flow(ls)
    assert torch.allclose(D.compute_log_alpha(ls, lsr).exp() + lsr.exp(), torch.ones_like(ls))
    lt = torch.linspace(-6, -0.05, 12, dtype=f64)
    for fwd, inv in ((D.log_snr_from_log_time_per_logit, D.log_time_from_log_snr_per_logit),
                     (D.log_snr_from_log_time_per_logtan, D.log_time_from_log_snr_per_logtan),
                     (D.log_snr_from_log_time_per_truncnormicdf, D.log_time_from_log_snr_per_truncnormicdf)):  # fmt: skip
        snr = fwd(lt)
        assert bool((snr[1:] <= snr[:-1]).all()) and bool((snr <= 20).all()) and bool((snr >= -20).all())
        assert torch.allclose(inv(snr), lt, atol=1e-9)
    torch.manual_seed(0)
    x, eps = torch.randn(3, 5, dtype=f64), torch.randn(3, 5, dtype=f64)
    lsnr = torch.tensor(0.7, dtype=f64)
    for corrupt, tfn, make in (
        (D.log_sigma_from_log_snr_per_rectified_flow, D.target_rectified_flow, lambda a, s: eps - x),
        (D.log_sigma_from_log_snr_per_variance_preserving, D.target_v, lambda a, s: a * eps - s * x),
        (D.log_sigma_from_log_snr_per_variance_preserving, D.target_eps, lambda a, s: eps),
        (D.log_sigma_from_log_snr_per_variance_preserving, D.target_x, lambda a, s: x),
    ):
        lsg = corrupt(lsnr)
        a, s = D.compute_log_alpha(lsnr, lsg).exp(), lsg.exp()
        xt = a * x + s * eps
        res = tfn(make(a, s), xt, lsnr, lsg, x_original=x, eps_original=eps)
        assert torch.allclose(res.x_clean, x) and torch.allclose(res.eps_clean, eps)
        assert torch.allclose(res.target, res.predict)
    # A perfect rectified-flow model makes DDIM land exactly on x.
    log_t = torch.linspace(0, -8, 9, dtype=f64)
    sched = D.log_snr_from_log_time_per_logit(log_t, low=-30, high=30)

    def model_fn(xc, l0, it, n, l1):  # noqa: ANN001, ANN202
        del it, n, l1
        lsg = D.log_sigma_from_log_snr_per_rectified_flow(l0)
        a, s = D.compute_log_alpha(l0, lsg).exp(), lsg.exp()
        e = (xc - a * x) / s
        return e - x

    x0 = torch.randn(3, 5, dtype=f64) * 0 + eps
    out = D.sample(sched[1:], model_fn, x0, D.ddim)
    assert torch.allclose(out.x_clean, x, atol=1e-8)
    steps = list(D.sample_iter(sched[1:], model_fn, x0, D.ddpm))
    assert len(steps) == sched.shape[0] - 2
    g, u = torch.randn(2, 3, 4), torch.randn(2, 3, 4) * 3
    full = D.rescale_classifier_free_guidance(g, u, strength=1.0)
    assert torch.allclose(full.std(dim=(1, 2)), u.std(dim=(1, 2)), rtol=1e-5)
    assert torch.equal(D.rescale_classifier_free_guidance(g, u), g)


def _lse(rank: int, world: int) -> list[float]:
    from priml_b200.math.distributed import logmeanexp_all_to_all, logsumexp_all_to_all

    x = torch.arange(6, dtype=torch.float64).reshape(2, 3) + 10 * rank
    return [logsumexp_all_to_all(x, dim=-1).tolist(), logmeanexp_all_to_all(x, dim=(0, 1)).item()]


def test_distributed_log_reductions_gloo() -> None:
    out = run_ranks(_lse, 2)
    full = torch.cat([torch.arange(6, dtype=f64).reshape(2, 3), torch.arange(6, dtype=f64).reshape(2, 3) + 10], 1)
    assert np.allclose(out[0][0], torch.logsumexp(full, -1).tolist())
    assert abs(out[1][1] - (float(torch.logsumexp(full.reshape(-1), 0)) - math.log(12))) < 1e-12
