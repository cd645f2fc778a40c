"""Drop-in non-causal RACE modules (the reference's misc/vit.py:888-1068).

Same constructor signatures, parameter/buffer names and shapes
(``planes_T``, ``protos_T``, ``logit_temp``) as the reference, so existing
model definitions and state_dicts load unchanged.  The forward runs the B200
kernels through ``race_attention``; no PyTorch fallback exists.
"""
from __future__ import annotations

import itertools

import torch
from torch import nn

from .functional import fused_qkv, race_attention


class BatchedACE(nn.Module):
    """Non-causal BatchedACE (misc/vit.py:888-978).

    Inputs Khf, Vhf, Qhf: [M, B, T, H, d_k]; output [M, B, T, H, d_k].
    """

    def __init__(self, d_k, K, L, M, device="cpu", share_planes: bool = False):
        super().__init__()
        self.d_k, self.K, self.L, self.M = d_k, K, L, M
        self.R = 1 << K
        self.share_planes = share_planes
        if share_planes:
            planes = torch.randn(L, K, d_k, device=device)
            self.register_buffer("planes_T", planes.view(L * K, d_k).T)        # [d_k, L*K]
        else:
            planes = torch.randn(M, L, K, d_k, device=device)
            self.register_buffer("planes_T", planes.view(M, L * K, d_k).transpose(1, 2))
        corners = torch.tensor(list(itertools.product([-1.0, 1.0], repeat=K)), device=device)
        self.register_buffer("protos_T", corners.T)                            # [K, R]
        self.logit_temp = nn.Parameter(torch.log(torch.tensor(1.0)))
        self.temp_max = 20.0   # misc/vit.py:923 (mlm.py / benchmark copies use 10.0)

    def planes(self) -> torch.Tensor:
        """Hyperplanes in kernel layout [Mp, L*K, d_k]."""
        pt = self.planes_T
        if pt.dim() == 2:
            pt = pt.unsqueeze(0)
        return pt.transpose(1, 2)

    def scale(self) -> torch.Tensor:
        return self.logit_temp.exp().clamp(1e-2, self.temp_max)

    def forward(self, Khf, Vhf, Qhf, eps: float = 1e-6, head_major_out: bool = False):
        M, B, T, H, dk = Khf.shape
        assert M == self.M and dk == self.d_k
        return race_attention(Qhf, Khf, Vhf, self.planes(), self.K, self.L, self.scale(),
                              causal=False, eps=eps, shared_planes=self.share_planes,
                              head_major_out=head_major_out)


class RACEAttention(nn.Module):
    """misc/vit.py:994-1038: q/k/v projections, RACE, ensemble mean, out-proj.

    Head merge: the reference merges the [B, T, H, d_k] ensemble mean with
    ``permute(0, 2, 1, 3).reshape(B, T, H * d_k)`` (misc/vit.py:1034-1035),
    which lays head h's tokens side by side in the rows of the output rather
    than concatenating the heads of each token.  That is reproduced by
    default (``merge_heads="reference"``), so reference checkpoints give the
    reference's outputs; ``merge_heads="concat"`` selects the per-token
    concatenation (a different model, for new training only).
    """

    def __init__(self, d_in, d_out, dropout, num_heads, L, K, N_M, qkv_bias=False, device="cpu",
                 merge_heads: str = "reference", fuse_qkv: bool = True):
        super().__init__()
        if merge_heads not in ("reference", "concat"):
            raise ValueError("merge_heads must be 'reference' or 'concat'")
        self.merge_heads = merge_heads
        self.fuse_qkv = fuse_qkv   # one GEMM for q, k, v (same parameters as three)
        assert d_in % num_heads == 0
        self.H = num_heads
        self.d_k = d_in // num_heads
        self.M = N_M
        self.L = L
        self.P = K
        self.q_proj = nn.Linear(d_in, d_in, bias=qkv_bias)
        self.k_proj = nn.Linear(d_in, d_in, bias=qkv_bias)
        self.v_proj = nn.Linear(d_in, d_in, bias=qkv_bias)
        self.out = nn.Linear(d_in, d_out)
        self.drop = nn.Dropout(dropout)
        self.ace = BatchedACE(self.d_k, K, L, N_M, device=device)

    def forward(self, x):
        B, T, _ = x.shape
        H, d_k, M = self.H, self.d_k, self.M
        if self.fuse_qkv:
            Q, K, V = fused_qkv(x, self.q_proj, self.k_proj, self.v_proj, H, d_k)
        else:
            Q = self.q_proj(x).view(B, T, H, d_k)
            K = self.k_proj(x).view(B, T, H, d_k)
            V = self.v_proj(x).view(B, T, H, d_k)
        pack = lambda Z: Z.unsqueeze(0).expand(M, -1, -1, -1, -1)
        ref = self.merge_heads == "reference"
        # reference merge: the output is written head-major, so the merge is a view for M = 1
        out_hm = self.ace(pack(K), pack(V), pack(Q), head_major_out=ref)
        out = out_hm[0] if M == 1 else out_hm.mean(dim=0)     # [B, T, H, d_k]
        if ref:
            out = out.permute(0, 2, 1, 3)                      # misc/vit.py:1035
        return self.drop(self.out(out.reshape(B, T, H * d_k)))


class RACEBlock(nn.Module):
    """misc/vit.py:1040-1068: pre-norm transformer block around RACEAttention."""

    def __init__(self, cfg, device="cpu"):
        super().__init__()
        self.att = RACEAttention(d_in=cfg["embed_dim"], d_out=cfg["embed_dim"],
                                 dropout=cfg["drop_rate"], num_heads=cfg["num_heads"],
                                 qkv_bias=cfg["qkv_bias"], L=cfg["L"], K=cfg["K"], N_M=cfg["M"],
                                 device=device)
        self.norm1 = nn.LayerNorm(cfg["embed_dim"])
        self.norm2 = nn.LayerNorm(cfg["embed_dim"])
        self.ff = nn.Sequential(nn.Linear(cfg["embed_dim"], 4 * cfg["embed_dim"]), nn.GELU(),
                                nn.Linear(4 * cfg["embed_dim"], cfg["embed_dim"]))
        self.drop = nn.Dropout(cfg["drop_rate"])

    def forward(self, x):
        h = x
        x = self.drop(self.att(self.norm1(x))) + h
        h = x
        return self.drop(self.ff(self.norm2(x))) + h


def race_bucket_probs_from_qk(attn: RACEAttention, Q: torch.Tensor, K: torch.Tensor):
    """Bucket probabilities of q and k with ``attn``'s planes and temperature,
    for hybrid models (the reference's ``race_bucket_probs_from_qk``,
    misc/arxiv_64K.py:1580-1642): Q, K [B, T, H, d_k] ->
    (probsQ, probsK), each [M, B, H, T, L, R]."""
    from .functional import bucket_probs
    ace = attn.ace
    M = attn.M

    def pack(z):
        return z.unsqueeze(0).expand(M, -1, -1, -1, -1)   # [M, B, T, H, d_k]

    planes = ace.planes()
    scale = ace.scale()
    probsQ = bucket_probs(pack(Q), planes, ace.K, ace.L, scale, shared_planes=ace.share_planes)
    probsK = bucket_probs(pack(K), planes, ace.K, ace.L, scale, shared_planes=ace.share_planes)
    return probsQ, probsK
