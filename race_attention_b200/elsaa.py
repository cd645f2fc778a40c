"""Drop-in for the reference's global-normalised causal RACE module
(``CausalRACEAttention``, misc/elsaa_causal_complete.py:438-571, the module the
ELSAA, WikiText, NIAH and copy-task scripts build).

Same constructor signature, parameter and buffer names (``q``, ``k``, ``v``,
``o``, ``planes`` [L, K, d_k], ``corners``, ``log_beta``, ``last_den``) and the
same ``forward(x, mask=None, return_den=False)``.  The attention itself --
soft hash, causal prefix sums, per-token global denominator, its backward --
runs in the library's causal walk with ``normalize="global"``; the chunking
the reference needs for memory (``chunk_size``, ``chunk_group_size``) has no
effect on the result and is kept only for signature compatibility.

Semantics kept from the reference:
  * phi = softmax over the 2^K corners of beta * tanh(x . planes), with
    beta = exp(log_beta).clamp(1e-2, 20) (:500-506); the library's divisor is
    1 / beta, so log_beta gets its gradient through autograd.
  * out = sum_l num_l / clamp_min(sum_l den_l, 1e-6) -- the reference's CUDA
    path (:551-557).  Its torch fallback averages num and den over the L
    tables first, i.e. floors the table sum at L * 1e-6 instead; pass
    ``den_floor=num_tables * 1e-6`` to reproduce that path exactly.
  * mask: keys and values of masked tokens are zeroed before hashing and the
    output of masked tokens is zeroed (:524-527, :558-559).
  * d_token = mean over heads of den / L, clamped at 1e-6, returned with
    ``return_den`` and kept (detached) in ``last_den`` (:560-562).
"""
from __future__ import annotations

import itertools
from typing import Optional

import torch
from torch import nn

from .functional import race_attention


class CausalRACEAttention(nn.Module):
    def __init__(self, d, h, drop, num_bits=4, num_tables=4, beta_init=1.0, chunk_size=256,
                 qkv_bias=False, device="cpu", chunk_group_size=64,
                 den_floor: Optional[float] = None):
        super().__init__()
        assert d % h == 0
        self.h = h
        self.dk = d // h
        self.num_bits = num_bits
        self.num_tables = num_tables
        self.R = 1 << num_bits
        self.C = chunk_size
        self.chunk_group_size = chunk_group_size
        self.den_floor = 1e-6 if den_floor is None else float(den_floor)
        self.q = nn.Linear(d, d, bias=qkv_bias)
        self.k = nn.Linear(d, d, bias=qkv_bias)
        self.v = nn.Linear(d, d, bias=qkv_bias)
        self.o = nn.Linear(d, d)
        self.drop = nn.Dropout(drop)
        self.register_buffer("planes", torch.randn(num_tables, num_bits, self.dk, device=device),
                             persistent=False)
        corners = torch.tensor(list(itertools.product([-1.0, 1.0], repeat=num_bits)),
                               device=device, dtype=torch.float32)
        self.register_buffer("corners", corners, persistent=False)
        self.log_beta = nn.Parameter(torch.log(torch.tensor(beta_init, dtype=torch.float32)))
        self.last_den = None

    def beta(self) -> torch.Tensor:
        return self.log_beta.exp().clamp(1e-2, 20.0)

    def forward(self, x, mask=None, return_den=False):
        B, T, _ = x.shape
        H, dk, L = self.h, self.dk, self.num_tables
        Q = self.q(x).view(B, T, H, dk)
        K = self.k(x).view(B, T, H, dk)
        V = self.v(x).view(B, T, H, dk)
        if mask is not None:
            keep = mask[:, :, None, None].to(Q.dtype)
            K = K * keep
            V = V * keep
        planes = self.planes.reshape(1, L * self.num_bits, dk)
        out, den = race_attention(Q, K, V, planes, self.num_bits, L, 1.0 / self.beta(),
                                  causal=True, eps=self.den_floor, normalize="global",
                                  return_den=True)
        out = out.to(x.dtype).reshape(B, T, H * dk)
        out = self.drop(self.o(out))
        if mask is not None:
            out = out * mask.unsqueeze(-1).to(out.dtype)
        d_token = (den.mean(dim=1) / L).unsqueeze(-1).clamp_min(1e-6).to(x.dtype)   # [B, T, 1]
        self.last_den = d_token.detach()
        return (out, d_token) if return_den else out
