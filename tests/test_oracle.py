"""The oracle (oracle/race_oracle.py) reproduces the reference's torch modules.

Golden vectors come from the reference's own ``BatchedACE`` classes run under
autograd in float64 (tests/golden/make_golden.py).  These tests pin the oracle
before any GPU test trusts it.
"""
import math

import numpy as np
import pytest

from oracle import race_oracle as O
from tests import golden_util as G


@pytest.mark.parametrize("path", G.golden_files(), ids=lambda p: p.split("/")[-1][:-4])
def test_oracle_matches_reference_modules(path):
    g = G.load(path)
    q, k, v = G.inputs_as_streams(g)
    P = G.stream_planes(g)
    M, B, H = g["M"], g["B"], g["H"]
    scale = float(g["scale"])
    out = O.forward(q, k, v, P, g["K"], g["L"], scale, g["causal"])
    np.testing.assert_allclose(G.from_streams(out, M, B, H), g["out"], rtol=1e-10, atol=1e-12)

    dout = G.to_streams(g["dout"])
    dq, dk, dv, dscale = O.backward(q, k, v, P, g["K"], g["L"], scale, g["causal"], dout)
    # the reference expands q/k/v over M ensembles, so its gradients are sums over m
    red = lambda x: G.from_streams(x, M, B, H).sum(0)
    np.testing.assert_allclose(red(dq), g["dq"], rtol=1e-9, atol=1e-11)
    np.testing.assert_allclose(red(dk), g["dk"], rtol=1e-9, atol=1e-11)
    np.testing.assert_allclose(red(dv), g["dv"], rtol=1e-9, atol=1e-11)
    if not g["causal"]:
        # d logit_temp = d scale * scale while exp(logit_temp) is inside the clamp
        assert math.isclose(dscale * scale, float(g["dlogit_temp"]), rel_tol=1e-9, abs_tol=1e-12)


def test_causal_last_token_equals_noncausal():
    rng = np.random.default_rng(0)
    N, T, D, K, L = 2, 19, 16, 2, 3
    q, k, v = (rng.standard_normal((N, T, D)) for _ in range(3))
    P = rng.standard_normal((N, K * L, D))
    c = O.causal_forward(q, k, v, P, K, L, 1.3)
    nc = O.noncausal_forward(q, k, v, P, K, L, 1.3)[0]
    np.testing.assert_allclose(c[:, -1], nc[:, -1], rtol=1e-12)


def test_backward_matches_finite_differences():
    rng = np.random.default_rng(1)
    N, T, D, K, L = 1, 7, 8, 2, 2
    q, k, v = (rng.standard_normal((N, T, D)) for _ in range(3))
    P = rng.standard_normal((N, K * L, D))
    dout = rng.standard_normal((N, T, D))
    for causal in (False, True):
        f = lambda q_, k_, v_, s_: float((O.forward(q_, k_, v_, P, K, L, s_, causal) * dout).sum())
        dq, dk, dv, ds = O.backward(q, k, v, P, K, L, 0.7, causal, dout)
        h = 1e-6
        for arr, grad, which in ((q, dq, 0), (k, dk, 1), (v, dv, 2)):
            idx = (0, 3, 5)
            a1, a2 = arr.copy(), arr.copy()
            a1[idx] += h
            a2[idx] -= h
            args1 = [q, k, v]
            args2 = [q, k, v]
            args1[which], args2[which] = a1, a2
            num = (f(*args1, 0.7) - f(*args2, 0.7)) / (2 * h)
            assert math.isclose(num, grad[idx], rel_tol=1e-5, abs_tol=1e-7)
        num = (f(q, k, v, 0.7 + h) - f(q, k, v, 0.7 - h)) / (2 * h)
        assert math.isclose(num, ds, rel_tol=1e-5, abs_tol=1e-7)


def test_oracle_prefix_mean_matches_reference_cpp():
    """Pin the causal restatement on the reference's own compiled C++ kernel."""
    from oracle.ref_loader import load_race_pref
    rp = load_race_pref()
    if rp is None:
        pytest.skip("oracle/_ref/race_pref not built (make -C oracle)")
    import torch
    g = torch.Generator().manual_seed(0)
    NS, T, D = 12, 300, 16
    w = torch.rand(NS, T, generator=g)
    V = torch.randn(NS, T, D, generator=g)
    gE = torch.randn(NS, T, D, generator=g)
    E = rp.race_prefix_mean_flat(w, V, 1e-6)
    np.testing.assert_allclose(E.numpy(), O.prefix_mean_flat(w.numpy(), V.numpy()), rtol=2e-6, atol=2e-6)
    gw, gV = rp.race_prefix_mean_flat_bw(w, V, gE, 1e-6)
    ow, oV = O.prefix_mean_flat_backward(w.numpy(), V.numpy(), gE.numpy())
    assert O.rel_l2(gw.numpy(), ow) < 1e-6
    assert O.rel_l2(gV.numpy(), oV) < 1e-6


def test_streamed_causal_matches_dense():
    """The chunk-streamed causal oracle (used at full sequence length) equals the dense one."""
    rng = np.random.default_rng(5)
    N, T, D, K, L = 2, 301, 16, 2, 3
    q, k, v, dout = (rng.standard_normal((N, T, D)) for _ in range(4))
    P = rng.standard_normal((N, K * L, D))
    ref = (O.causal_forward(q, k, v, P, K, L, 0.9),) + O.causal_backward(q, k, v, P, K, L, 0.9, dout)
    for chunk in (1, 64, 1000):
        got = O.causal_streamed(q, k, v, P, K, L, 0.9, dout, chunk=chunk)
        for a, b in zip(got[:4], ref[:4]):
            np.testing.assert_allclose(a, b, rtol=1e-9, atol=1e-12)
        assert math.isclose(got[4], ref[4], rel_tol=1e-9)
    np.testing.assert_allclose(O.causal_streamed(q, k, v, P, K, L, 0.9, chunk=50), ref[0], rtol=1e-9, atol=1e-12)


def _probs_streams(g, name):
    """[B,T,H,d] input of a probs golden -> [N,T,d] streams in (m, b, h) order."""
    M, B, T, H, d = (int(v) for v in g["meta"][:5])
    x = np.asarray(g[name], np.float64)
    xs = np.broadcast_to(x.transpose(0, 2, 1, 3)[None], (M, B, H, T, d)).reshape(M * B * H, T, d)
    return xs, (M, B, T, H, d)


@pytest.mark.parametrize("path", G.probs_files(), ids=lambda p: p.split("/")[-1][:-4])
def test_oracle_matches_reference_probs_export(path):
    """soft_hash / soft_hash_backward reproduce race_bucket_probs_from_qk
    (misc/arxiv_64K.py:1580-1642) run under autograd in float64."""
    g = np.load(path)
    K, L = int(g["meta"][5]), int(g["meta"][6])
    scale = float(g["scale"])
    planes = np.asarray(g["planes"], np.float64)
    dl = 0.0
    for name, pname, gname, dname in (("q", "probs_q", "gq", "dq"), ("k", "probs_k", "gk", "dk")):
        xs, (M, B, T, H, d) = _probs_streams(g, name)
        P = planes[np.repeat(np.arange(M) if planes.shape[0] == M else np.zeros(M, int), B * H)]
        p, h = O.soft_hash(xs, P, K, L, scale)
        np.testing.assert_allclose(p, g[pname].reshape(M * B * H, T, -1), rtol=1e-10, atol=1e-12)
        dp = np.asarray(g[gname], np.float64).reshape(M * B * H, T, -1)
        dx, ds = O.soft_hash_backward(dp, p, h, P, K, L, scale)
        dx = dx.reshape(M, B, H, T, d).sum(0).transpose(0, 2, 1, 3)   # -> [B,T,H,d]
        np.testing.assert_allclose(dx, g[dname], rtol=1e-9, atol=1e-11)
        dl += ds * scale
    assert math.isclose(dl, float(g["dlogit_temp"]), rel_tol=1e-9, abs_tol=1e-12)


@pytest.mark.parametrize("path", G.global_files(), ids=lambda p: p.split("/")[-1][:-4])
def test_oracle_matches_reference_global_causal(path):
    """causal_global reproduces the reference's CausalRACEAttention torch path
    (misc/elsaa_causal_complete.py:520-571: chunked, padded, table-averaged,
    optionally masked and chunk-grouped) run under autograd in float64: out,
    d_token and the gradients of Q, K, V and log_beta."""
    g = G.load_global(path)
    B, H, L, K = g["B"], g["H"], g["L"], g["K"]
    scale = 1.0 / float(g["beta"])
    # the torch path averages num and den over the L tables before its
    # clamp_min(1e-6): the same as a floor of L * 1e-6 on the table sum
    eps = L * 1e-6
    keep = g["keep_s"]
    out, den, dq, dk, dv, ds = O.causal_global(
        g["qs"], g["ks"], g["vs"], g["planes_s"], K, L, scale, dout=g["douts"] * keep,
        dden=g["dden"], eps=eps)
    rel = lambda a, b: float(np.abs(a - b).max() / np.abs(b).max())
    assert rel(G.merge_heads(out * keep, B, H), g["out"]) < 1e-13
    d_token = np.maximum(den.reshape(B, H, -1).mean(1) / L, 1e-6)
    assert rel(d_token, g["d_token"][..., 0]) < 1e-13
    assert rel(G.merge_heads(dv * keep, B, H), g["dv"]) < 1e-13
    # the hash gradients pass through 1 - tanh^2 of projections up to ~17,
    # where that factor (~1e-14) carries a relative rounding error of ~1e-2 in
    # either implementation: 1e-7 of the largest element bounds the gap
    assert rel(G.merge_heads(dq, B, H), g["dq"]) < 1e-7
    assert rel(G.merge_heads(dk * keep, B, H), g["dk"]) < 1e-7
    assert math.isclose(-ds * scale, float(g["dlog_beta"]), rel_tol=1e-7)


def test_l2_normalize_matches_torch():
    """The oracle's normalisation (used by the normalize_qk flag) against
    torch.nn.functional.normalize and its autograd, zero rows included."""
    import torch
    rng = np.random.default_rng(3)
    x = rng.standard_normal((3, 17, 64))
    x[1, 4] = 0.0
    g = rng.standard_normal(x.shape)
    xt = torch.tensor(x, requires_grad=True)
    y = torch.nn.functional.normalize(xt, dim=-1)
    y.backward(torch.tensor(g))
    assert np.allclose(O.l2_normalize(x), y.detach().numpy(), rtol=1e-12, atol=1e-14)
    assert np.allclose(O.l2_normalize_backward(x, g), xt.grad.numpy(), rtol=1e-10, atol=1e-12)
