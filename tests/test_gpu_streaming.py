"""Host-buffer forward + backward (race_attention_b200.streaming) against the
device-tensor autograd path on the same values (relative L2 1e-4 in float32,
2e-2 in bfloat16: the chunked path sums the bucket states in another order)."""
import numpy as np
import pytest
import torch

from oracle import race_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from race_attention_b200 import _lib
    _lib.load()


@pytest.mark.parametrize("causal,dtype,T,H,chunks", [
    (False, torch.float32, 5000, 2, 8),
    (True, torch.float32, 5000, 2, 8),
    (False, torch.bfloat16, 3001, 1, 3),
    (True, torch.bfloat16, 3001, 1, 3),
    (True, torch.float32, 100, 1, 8),
    (False, torch.float32, 0, 1, 4),
])
def test_host_pipeline_matches_device_path(causal, dtype, T, H, chunks):
    from race_attention_b200 import race_attention
    from race_attention_b200.streaming import fwd_bwd_host
    K, L, d = 2, 5, 64
    g = torch.Generator().manual_seed(7 + T)
    host = [torch.randn(1, 1, T, H, d, generator=g).to(dtype).pin_memory() for _ in range(4)]
    planes = torch.randn(1, K * L, d, generator=g)
    scale = torch.tensor(1.3, device="cuda", requires_grad=True)
    out, dq, dk, dv, ds = fwd_bwd_host(*host, planes, K, L, scale.detach(), causal=causal,
                                       chunks=chunks)
    torch.cuda.current_stream().synchronize()
    q, k, v = (h.cuda().requires_grad_(True) for h in host[:3])
    ref = race_attention(q, k, v, planes.cuda(), K, L, scale, causal=causal)
    ref.backward(host[3].cuda())
    if T == 0:
        assert out.numel() == 0 and float(ds) == 0.0
        return
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    c = lambda t: t.detach().double().cpu().numpy()
    for got, want in ((out, ref), (dq, q.grad), (dk, k.grad), (dv, v.grad)):
        assert O.rel_l2(c(got), c(want)) < tol
    assert abs(float(ds) - float(scale.grad)) <= tol * max(1.0, abs(float(scale.grad)))
