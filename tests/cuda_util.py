"""Runs the CUDA path through the public autograd API for parity tests."""
import numpy as np
import torch

from race_attention_b200 import race_attention


def run_streams(q, k, v, planes, K, L, scale, causal, dout, dtype=torch.float32, chunk=0,
                eps=1e-6):
    """q,k,v,dout: [N,T,d] numpy; planes [N or 1, LK, d].  Returns numpy results.

    Streams are laid out as [M=1, B=N, T, H=1, d]; planes must then be shared
    (one set), or given per stream via ensembles -> handled by the caller.
    """
    dev = "cuda"
    to = lambda a: torch.tensor(np.asarray(a), dtype=torch.float32, device=dev).to(dtype)
    qt, kt, vt = (to(a).unsqueeze(0).unsqueeze(3).requires_grad_(True) for a in (q, k, v))
    P = torch.tensor(np.asarray(planes), dtype=torch.float32, device=dev)
    sc = torch.tensor(float(scale), dtype=torch.float32, device=dev, requires_grad=True)
    out = race_attention(qt, kt, vt, P, K, L, sc, causal=causal, eps=eps, chunk=chunk,
                         shared_planes=True)
    out.backward(to(dout).unsqueeze(0).unsqueeze(3))
    f = lambda t: t.detach().float().squeeze(3).squeeze(0).cpu().numpy().astype(np.float64)
    return f(out), f(qt.grad), f(kt.grad), f(vt.grad), float(sc.grad)


def bf16_round(a):
    return torch.tensor(np.asarray(a), dtype=torch.float32).bfloat16().float().numpy()
