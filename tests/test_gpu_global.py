"""Global-normalised causal mode on the GPU vs the reference's fixtures and the oracle.

The mode is the reference's CausalRACEAttention (misc/elsaa_causal_complete.py:
438-571, misc/race_kernel.py): one denominator per token summed over all
buckets.  Tolerances as for the per-bucket paths: relative L2 1e-4 for float32
inputs, 2e-2 for bfloat16 inputs (the oracle then sees the same rounded inputs).
"""
import math

import numpy as np
import pytest
import torch
from torch import nn

from oracle import race_oracle as O
from tests import golden_util as G
from tests.cuda_util import bf16_round

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from race_attention_b200 import _lib
    _lib.load()   # fails loudly when the extension is missing


def _c(t):
    return t.detach().double().cpu().numpy()


@pytest.mark.parametrize("path", G.global_files(), ids=lambda p: p.split("/")[-1][:-4])
def test_golden_functional(path):
    """race_attention(normalize='global') against the reference module's own
    float64 out, d_token and gradients (the torch path's L * 1e-6 floor)."""
    from race_attention_b200 import race_attention
    g = G.load_global(path)
    B, T, H, dk, K, L = (g[x] for x in ("B", "T", "H", "hd", "K", "L"))
    dev = "cuda"
    q, k, v = (torch.tensor(g[x], device=dev, requires_grad=True) for x in ("q", "k", "v"))
    keep = torch.tensor(g["mask"] if g["masked"] else np.ones((B, T), np.float32), device=dev)
    lb = torch.tensor(math.log(float(g["beta"])), dtype=torch.float32, device=dev,
                      requires_grad=True)
    heads = lambda z: z.view(B, T, H, dk)
    kk = heads(k) * keep[:, :, None, None]
    vv = heads(v) * keep[:, :, None, None]
    planes = torch.tensor(g["planes"], device=dev).reshape(1, L * K, dk)
    out, den = race_attention(heads(q), kk, vv, planes, K, L, 1.0 / lb.exp(), causal=True,
                              eps=L * 1e-6, normalize="global", return_den=True)
    out = out.reshape(B, T, H * dk) * keep[..., None]
    d_token = (den.mean(dim=1) / L).unsqueeze(-1).clamp_min(1e-6)
    loss = (out * torch.tensor(g["dout"], device=dev)).sum() + \
        (d_token * torch.tensor(g["gtok"], device=dev)).sum()
    loss.backward()
    assert O.rel_l2(_c(out), g["out"]) < 1e-4
    assert O.rel_l2(_c(d_token), g["d_token"]) < 1e-4
    assert O.rel_l2(_c(q.grad), g["dq"]) < 1e-4
    assert O.rel_l2(_c(k.grad), g["dk"]) < 1e-4
    assert O.rel_l2(_c(v.grad), g["dv"]) < 1e-4
    assert math.isclose(float(lb.grad), float(g["dlog_beta"]), rel_tol=1e-4, abs_tol=1e-6)


class _Const(nn.Module):
    def __init__(self, t):
        super().__init__()
        self.t = t

    def forward(self, x):
        return self.t


@pytest.mark.parametrize("path", G.global_files(), ids=lambda p: p.split("/")[-1][:-4])
def test_golden_module(path):
    """The drop-in CausalRACEAttention module, wired as the fixture generator
    wired the reference's (projections replaced by the inputs, o = identity)."""
    from race_attention_b200.elsaa import CausalRACEAttention
    g = G.load_global(path)
    B, T, H, dk, K, L = (g[x] for x in ("B", "T", "H", "hd", "K", "L"))
    dev = "cuda"
    att = CausalRACEAttention(H * dk, H, 0.0, num_bits=K, num_tables=L, chunk_size=g["C"],
                              device=dev, den_floor=L * 1e-6).to(dev)
    with torch.no_grad():
        att.planes.copy_(torch.tensor(g["planes"]))
        att.log_beta.fill_(math.log(float(g["beta"])))
    q, k, v = (torch.tensor(g[x], device=dev, requires_grad=True) for x in ("q", "k", "v"))
    att.q, att.k, att.v, att.o = _Const(q), _Const(k), _Const(v), nn.Identity()
    mask = torch.tensor(g["mask"], device=dev) if g["masked"] else None
    out, d_token = att(torch.zeros(B, T, H * dk, device=dev), mask=mask, return_den=True)
    ((out * torch.tensor(g["dout"], device=dev)).sum()
     + (d_token * torch.tensor(g["gtok"], device=dev)).sum()).backward()
    assert O.rel_l2(_c(out), g["out"]) < 1e-4
    assert O.rel_l2(_c(d_token), g["d_token"]) < 1e-4
    assert O.rel_l2(_c(att.last_den), g["d_token"]) < 1e-4
    for name, t in (("dq", q), ("dk", k), ("dv", v)):
        assert O.rel_l2(_c(t.grad), g[name]) < 1e-4, name
    assert math.isclose(float(att.log_beta.grad), float(g["dlog_beta"]), rel_tol=1e-4,
                        abs_tol=1e-6)


CASES = [
    # N, T, d, K, L, dtype, chunk
    (2, 5, 64, 2, 5, torch.float32, 0),
    (3, 33, 32, 3, 3, torch.float32, 0),
    (2, 1000, 64, 2, 5, torch.float32, 0),
    (2, 1000, 64, 2, 5, torch.float32, 64),
    (1, 3001, 64, 4, 2, torch.float32, 0),
    (2, 2048, 64, 2, 5, torch.bfloat16, 0),
    (2, 777, 32, 1, 8, torch.bfloat16, 0),
]


@pytest.mark.parametrize("N,T,d,K,L,dtype,chunk", CASES)
def test_vs_oracle(N, T, d, K, L, dtype, chunk):
    """Seeded streams (several token ranges per stream at T >= 1000) with an
    incoming d(den) as well as d(out): out, den, dq, dk, dv, dscale."""
    from race_attention_b200 import race_attention
    rng = np.random.default_rng(1000 * N + T + d + K)
    x = lambda: rng.standard_normal((N, T, d)).astype(np.float32)
    q, k, v, dout = x(), x(), x(), x()
    if dtype == torch.bfloat16:
        q, k, v, dout = (bf16_round(a) for a in (q, k, v, dout))
    planes = rng.standard_normal((1, L * K, d)).astype(np.float32)
    dden = rng.standard_normal((N, T)).astype(np.float32) * 0.1
    scale = 0.8
    dev = "cuda"
    to = lambda a: torch.tensor(a, device=dev).to(dtype).unsqueeze(0).unsqueeze(3)
    qt, kt, vt = (to(a).requires_grad_(True) for a in (q, k, v))
    sc = torch.tensor(scale, device=dev, requires_grad=True)
    out, den = race_attention(qt, kt, vt, torch.tensor(planes, device=dev), K, L, sc,
                              causal=True, chunk=chunk, normalize="global", return_den=True)
    assert den.shape == (1, N, 1, T) and den.dtype == torch.float32
    torch.autograd.backward([out, den], [to(dout), torch.tensor(dden, device=dev)[None, :, None]])
    ro, rden, rdq, rdk, rdv, rds = O.causal_global(q, k, v, np.broadcast_to(planes, (N,) + planes.shape[1:]),
                                                   K, L, scale, dout=dout, dden=dden)
    f = lambda t: _c(t).squeeze(3).squeeze(0)
    tol = TOL[dtype]
    assert O.rel_l2(f(out), ro) < tol
    assert O.rel_l2(_c(den)[0, :, 0], rden) < (1e-5 if dtype == torch.float32 else 1e-3)
    assert O.rel_l2(f(qt.grad), rdq) < tol
    assert O.rel_l2(f(kt.grad), rdk) < tol
    assert O.rel_l2(f(vt.grad), rdv) < tol
    assert math.isclose(float(sc.grad), rds, rel_tol=tol, abs_tol=1e-5)


def test_bucket_mode_unchanged_and_rejects():
    """The default per-bucket mode ignores the new field; global is causal-only."""
    from race_attention_b200 import race_attention
    dev = "cuda"
    q = torch.randn(1, 1, 64, 2, 64, device=dev)
    with pytest.raises(ValueError):
        race_attention(q, q, q, torch.randn(1, 10, 64, device=dev), 2, 5, 1.0, causal=False,
                       normalize="global")
    with pytest.raises(ValueError):
        race_attention(q, q, q, torch.randn(1, 10, 64, device=dev), 2, 5, 1.0, causal=True,
                       return_den=True)
