"""Bucket-probability export on the GPU (needs a B200).

``bucket_probs`` / ``race_bucket_probs_from_qk`` against the reference's own
race_bucket_probs_from_qk run in float64 (tests/golden/probs_*.npz) and
against the oracle on seeded inputs; gradients in x and the temperature
included.  Bars: 1e-4 relative L2 for float32 inputs, 2e-2 for bfloat16.
"""
import math

import numpy as np
import pytest
import torch

from oracle import race_oracle as O
from tests import golden_util as G
from tests.cuda_util import bf16_round

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from race_attention_b200 import _lib
    _lib.load()


@pytest.mark.parametrize("path", G.probs_files(), ids=lambda p: p.split("/")[-1][:-4])
def test_probs_golden(path):
    from race_attention_b200.functional import bucket_probs
    g = np.load(path)
    M, B, T, H, d, K, L, share = (int(v) for v in g["meta"])
    dev = "cuda"
    lt = torch.tensor(math.log(float(g["scale"])), device=dev, dtype=torch.float64,
                      requires_grad=True)
    scale = lt.exp().clamp(1e-2, 20.0).float()
    planes = torch.tensor(g["planes"], device=dev)
    dl = 0.0
    for name, pname, gname, dname in (("q", "probs_q", "gq", "dq"), ("k", "probs_k", "gk", "dk")):
        x = torch.tensor(g[name], device=dev, requires_grad=True)
        xp = x.unsqueeze(0).expand(M, -1, -1, -1, -1)
        p = bucket_probs(xp, planes, K, L, scale, shared_planes=bool(share))
        assert tuple(p.shape) == tuple(g[pname].shape)
        assert O.rel_l2(p.detach().double().cpu().numpy(), g[pname]) < 1e-4
        p.backward(torch.tensor(g[gname], device=dev), retain_graph=True)
        assert O.rel_l2(x.grad.double().cpu().numpy(), g[dname]) < 1e-4
    assert math.isclose(float(lt.grad), float(g["dlogit_temp"]), rel_tol=1e-4, abs_tol=1e-6)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("N,T,d,K,L", [(2, 1, 64, 2, 5), (3, 1000, 64, 3, 3), (2, 333, 32, 5, 1),
                                       (1, 4100, 64, 1, 16), (2, 777, 64, 4, 2)])
def test_probs_vs_oracle(N, T, d, K, L, dtype):
    from race_attention_b200.functional import bucket_probs
    rng = np.random.default_rng(N * 131 + T + K * 7 + L)
    x = rng.standard_normal((N, T, d)).astype(np.float32)
    dp = rng.standard_normal((N, T, L << K)).astype(np.float32)
    planes = rng.standard_normal((1, K * L, d)).astype(np.float32)
    scale = 0.9
    if dtype == torch.bfloat16:
        x = bf16_round(x)
    dev = "cuda"
    xt = torch.tensor(x, device=dev).to(dtype).unsqueeze(0).unsqueeze(3).requires_grad_(True)
    sc = torch.tensor(scale, device=dev, requires_grad=True)
    p = bucket_probs(xt, torch.tensor(planes, device=dev), K, L, sc)      # [1, N, 1, T, L, R]
    p.backward(torch.tensor(dp, device=dev).reshape(p.shape))
    P = np.broadcast_to(planes, (N,) + planes.shape[1:])
    ref_p, h = O.soft_hash(x, P, K, L, scale)
    ref_dx, ref_ds = O.soft_hash_backward(dp, ref_p, h, P, K, L, scale)
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    got_p = p.detach().double().cpu().numpy().reshape(N, T, -1)
    assert O.rel_l2(got_p, ref_p) < 1e-4          # computed in fp32 from the (rounded) inputs
    got_dx = xt.grad.float().double().cpu().numpy().reshape(N, T, d)
    assert O.rel_l2(got_dx, ref_dx) < tol
    assert math.isclose(float(sc.grad), ref_ds, rel_tol=tol, abs_tol=1e-3 * tol), (float(sc.grad), ref_ds)


def test_probs_from_qk_module():
    """race_bucket_probs_from_qk with the drop-in RACEAttention module."""
    from race_attention_b200.vit import RACEAttention, race_bucket_probs_from_qk
    torch.manual_seed(3)
    attn = RACEAttention(128, 128, 0.0, 2, L=5, K=2, N_M=2, device="cuda").cuda()
    with torch.no_grad():
        attn.ace.logit_temp.fill_(math.log(1.7))
    Bq, T = 2, 200
    Q = torch.randn(Bq, T, 2, 64, device="cuda")
    Kt = torch.randn(Bq, T, 2, 64, device="cuda")
    pq, pk = race_bucket_probs_from_qk(attn, Q, Kt)
    assert tuple(pq.shape) == (2, Bq, 2, T, 5, 4)
    planes = attn.ace.planes().detach().cpu().numpy()           # [M or 1, LK, d]
    scale = float(attn.ace.scale())
    for got, x in ((pq, Q), (pk, Kt)):
        xs = x.cpu().numpy().transpose(0, 2, 1, 3).reshape(Bq * 2, T, 64)
        for m in range(2):
            Pm = planes[m if planes.shape[0] == 2 else 0]
            ref, _ = O.soft_hash(xs, np.broadcast_to(Pm, (Bq * 2,) + Pm.shape), 2, 5, scale)
            g = got[m].detach().double().cpu().numpy().reshape(Bq * 2, T, -1)
            assert O.rel_l2(g, ref) < 1e-4
