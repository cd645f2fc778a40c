"""Drop-in causal RACE modules (the reference's misc/race.py:26-206).

Per-bucket normalised prefix mean with the fixed divisor sqrt(d_k)
(misc/race.py:67) and shared planes by default.  Same constructor
signatures and buffer names as the reference.
"""
from __future__ import annotations

import itertools
import math

import torch
from torch import nn

from .functional import fused_qkv, race_attention


class BatchedACE(nn.Module):
    """Causal BatchedACE (misc/race.py:26-142): inputs/outputs [M, B, T, H, d_k]."""

    def __init__(self, d_k, K, L, M, device="cpu", share_planes: bool = True):
        super().__init__()
        self.d_k, self.K, self.L, self.M = d_k, K, L, M
        self.R = 1 << K
        self.share_planes = share_planes
        if share_planes:
            planes = torch.randn(L, K, d_k, device=device)
            self.register_buffer("planes_T", planes.view(L * K, d_k).T)
        else:
            planes = torch.randn(M, L, K, d_k, device=device)
            planes = planes.view(M, L * K, d_k).transpose(1, 2)
            self.register_buffer("planes_T", planes)
        corners = torch.tensor(list(itertools.product([-1.0, 1.0], repeat=K)), device=device)
        self.register_buffer("protos_T", corners.T)
        self.register_buffer("_scale", torch.tensor(math.sqrt(d_k)), persistent=False)

    def planes(self) -> torch.Tensor:
        pt = self.planes_T
        if pt.dim() == 2:
            pt = pt.unsqueeze(0)
        return pt.transpose(1, 2)

    def forward(self, Khf, Vhf, Qhf, head_major_out: bool = False):
        M, B, T, H, dk = Khf.shape
        assert M == self.M and dk == self.d_k
        return race_attention(Qhf, Khf, Vhf, self.planes(), self.K, self.L, self._scale,
                              causal=True, eps=1e-6, shared_planes=self.share_planes,
                              head_major_out=head_major_out)


class RACEAttention(nn.Module):
    """misc/race.py:144-173.

    Head merge as in the reference, ``mean(0).permute(0, 2, 1, 3)
    .contiguous().view(B, T, -1)`` (misc/race.py:171), by default
    (``merge_heads="reference"``): the rows of the merged tensor hold head
    h's tokens side by side.  ``merge_heads="concat"`` concatenates the heads
    of each token instead (a different model, for new training only).
    """

    def __init__(self, d, h, K, L, M, drop=0.1, qkv_bias=False, device="cpu",
                 merge_heads: str = "reference", fuse_qkv: bool = True):
        super().__init__()
        if merge_heads not in ("reference", "concat"):
            raise ValueError("merge_heads must be 'reference' or 'concat'")
        self.merge_heads = merge_heads
        self.fuse_qkv = fuse_qkv   # one GEMM for q, k, v (same parameters as three)
        assert d % h == 0
        self.h, self.d_k, self.M = h, d // h, M
        self.q = nn.Linear(d, d, bias=qkv_bias)
        self.k = nn.Linear(d, d, bias=qkv_bias)
        self.v = nn.Linear(d, d, bias=qkv_bias)
        self.o = nn.Linear(d, d)
        self.drop = nn.Dropout(drop)
        self.ace = BatchedACE(self.d_k, K, L, M, device=device)

    def forward(self, x):
        B, T, _ = x.shape
        if self.fuse_qkv:
            Q, K, V = fused_qkv(x, self.q, self.k, self.v, self.h, self.d_k)
        else:
            Q = self.q(x).view(B, T, self.h, self.d_k)
            K = self.k(x).view(B, T, self.h, self.d_k)
            V = self.v(x).view(B, T, self.h, self.d_k)
        pack = lambda z: z.unsqueeze(0).expand(self.M, -1, -1, -1, -1)
        ref = self.merge_heads == "reference"
        out_h = self.ace(pack(K), pack(V), pack(Q), head_major_out=ref)
        out = out_h[0] if self.M == 1 else out_h.mean(0)      # [B, T, H, d_k]
        if ref:
            out = out.permute(0, 2, 1, 3)                      # misc/race.py:171
        return self.drop(self.o(out.reshape(B, T, -1)))


class RACEBlock(nn.Module):
    """misc/race.py:176-206."""

    def __init__(self, cfg, device="cpu"):
        super().__init__()
        self.att = RACEAttention(d=cfg["emb_dim"], h=cfg["n_heads"], K=cfg["K"], L=cfg["L"],
                                 M=cfg["M"], drop=cfg["drop_rate"], qkv_bias=cfg["qkv_bias"],
                                 device=device)
        self.norm1 = nn.LayerNorm(cfg["emb_dim"])
        self.norm2 = nn.LayerNorm(cfg["emb_dim"])
        self.ff = nn.Sequential(nn.Linear(cfg["emb_dim"], 4 * cfg["emb_dim"]), nn.GELU(),
                                nn.Linear(4 * cfg["emb_dim"], cfg["emb_dim"]))
        self.drop = nn.Dropout(cfg["drop_rate"])

    def forward(self, x):
        h = x
        x = self.drop(self.att(self.norm1(x))) + h
        h = x
        return self.drop(self.ff(self.norm2(x))) + h
