"""PyTorch-CPU restatement of the reference's RACE op sequence, for TIMING.

TEST INFRASTRUCTURE / CPU BASELINE ONLY (``bench.py``'s cpu_baseline leg and
``--impl reference`` arm).  It issues the same torch operations, in the same
order and precision, as the reference modules:

  non-causal: misc/vit.py:943-975 -- einsum projection, tanh, /scale,
              @protos_T, softmax, bmm pK^T V, sum, divide, bmm pQ E;
  causal:     misc/race.py:79-138 -- the same soft hash, then the
              per-bucket prefix mean.  The reference materialises the
              [N,T,L,R,d] cumsum (misc/race.py:109), which does not fit a
              bounded sample, so here the identical arithmetic runs in token
              blocks carrying the running sums across blocks.

The reference tree is not importable on the GPU host, hence the restatement.
"""
from __future__ import annotations

import itertools

import torch
import torch.nn.functional as F


def protos_T(K, device="cpu", dtype=torch.float32):
    c = torch.tensor(list(itertools.product([-1.0, 1.0], repeat=K)), device=device, dtype=dtype)
    return c.T


def soft_hash(x, planes_T, K, L, scale, protos):
    """x [N,T,d], planes_T [d, L*K] -> probs [N,T,L*R] (misc/vit.py:943-958)."""
    N, T, _ = x.shape
    proj = (x @ planes_T).view(N, T, L, K)
    logits = proj.tanh().div(scale) @ protos
    return F.softmax(logits, dim=-1).reshape(N, T, -1)


def noncausal(q, k, v, planes_T, K, L, scale, protos, eps=1e-6):
    pK = soft_hash(k, planes_T, K, L, scale, protos)
    pQ = soft_hash(q, planes_T, K, L, scale, protos)
    b_sum = pK.transpose(1, 2).bmm(v)                 # misc/vit.py:967
    A = pK.sum(dim=1)                                 # misc/vit.py:969
    E = b_sum / (A.unsqueeze(-1) + eps)               # misc/vit.py:972
    return pQ.bmm(E)                                  # misc/vit.py:975


def causal(q, k, v, planes_T, K, L, scale, protos, eps=1e-6, block=1024):
    pK = soft_hash(k, planes_T, K, L, scale, protos)
    pQ = soft_hash(q, planes_T, K, L, scale, protos)
    N, T, S = pK.shape
    d = v.shape[-1]
    outs = []
    A0 = torch.zeros(N, 1, S, dtype=v.dtype)
    B0 = torch.zeros(N, 1, S, d, dtype=v.dtype)
    for t0 in range(0, T, block):
        pk, pq, vv = pK[:, t0:t0 + block], pQ[:, t0:t0 + block], v[:, t0:t0 + block]
        A = A0 + pk.cumsum(dim=1)                                         # misc/race.py:108
        Bp = B0 + (pk.unsqueeze(-1) * vv.unsqueeze(2)).cumsum(dim=1)      # misc/race.py:109
        E = Bp / (A.unsqueeze(-1) + eps)                                  # misc/race.py:110
        outs.append(torch.einsum("nts,ntsd->ntd", pq, E))                 # misc/race.py:135-138
        A0, B0 = A[:, -1:], Bp[:, -1:]
    return torch.cat(outs, dim=1)


def fwd_bwd(q, k, v, planes_T, K, L, scale, protos, dout, is_causal):
    """One reference-style fwd+bwd step (loss = <out, dout>), as benchmark_time.py:305-326."""
    for t in (q, k, v):
        t.grad = None
    fn = causal if is_causal else noncausal
    out = fn(q, k, v, planes_T, K, L, scale, protos)
    out.backward(dout)
    return out
