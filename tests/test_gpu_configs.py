"""The benchmark configurations' own shapes on the GPU (needs a B200).

BASELINE's ViT config (C3: batch 256, 6 heads, 785 tokens, d 64, K 4 L 4,
i.e. 64 buckets, 1536 streams), its causal bf16 language-model config (C2:
batch 4, 12 heads, 16384 tokens: 48 streams) and its long causal decoder
(C4: 12 heads, 65536 tokens).  Each runs whole on the device through the
autograd API in the [B, T, H, d] layout of the modules; streams are
independent, so a seeded sample of them is checked against the float64
oracle at the path's bars (1e-4 relative L2 for float32, 2e-2 for bfloat16).
Inputs are synthetic N(0, 1) draws standing in for the reference's datasets.
"""
import numpy as np
import pytest
import torch

from oracle import race_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _run(B, T, H, d, K, L, causal, dtype, scale, seed, sample):
    from race_attention_b200 import race_attention
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(seed)
    mk = lambda: torch.randn(B, T, H, d, generator=g, device=dev).to(dtype)
    q, k, v, do = mk(), mk(), mk(), mk()
    for t in (q, k, v):
        t.requires_grad_(True)
    planes = torch.randn(1, K * L, d, generator=g, device=dev)
    out = race_attention(q, k, v, planes, K, L, scale, causal=causal)
    out.backward(do)
    torch.cuda.synchronize()
    rng = np.random.default_rng(seed)
    picks = rng.choice(B * H, size=sample, replace=False)
    f = lambda t, b, h: t[b, :, h, :].detach().float().cpu().numpy().astype(np.float64)
    P = planes.cpu().numpy()
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    for s in picks:
        b, h = divmod(int(s), H)
        qs, ks, vs, ds = (f(t, b, h)[None] for t in (q, k, v, do))
        if causal and T > 20000:
            ref, dq, dk, dv, _ = O.causal_streamed(qs, ks, vs, P, K, L, scale, ds)
        else:
            ref = O.forward(qs, ks, vs, P, K, L, scale, causal)
            dq, dk, dv, _ = O.backward(qs, ks, vs, P, K, L, scale, causal, ds)
        for name, a, r in (("out", out, ref), ("dq", q.grad, dq), ("dk", k.grad, dk),
                           ("dv", v.grad, dv)):
            err = O.rel_l2(f(a, b, h)[None], r)
            assert err < tol, (name, b, h, err)


def test_c3_vit_shape_64_buckets():
    _run(256, 785, 6, 64, 4, 4, False, torch.float32, 1.0, 31, sample=12)


def test_c3_vit_shape_64_buckets_bf16():
    _run(256, 785, 6, 64, 4, 4, False, torch.bfloat16, 1.0, 32, sample=12)


def test_c2_causal_bf16_shape():
    _run(4, 16384, 12, 64, 2, 5, True, torch.bfloat16, 8.0, 33, sample=4)


def test_c4_long_causal_shape():
    _run(1, 65536, 12, 64, 2, 5, True, torch.float32, 8.0, 34, sample=2)
