"""Generate the golden parity vectors from the reference's own torch modules.

Run in the build container, where the reference project is mounted read-only:

    python tests/golden/make_golden.py /path/to/reference [all|global|modules]

It extracts the class definitions ``BatchedACE`` from ``misc/vit.py``
(non-causal, lines 888-978) and from ``misc/race.py`` (causal, lines 26-142)
with ``ast`` -- the files themselves cannot be imported as-is (``misc/race.py:7``
imports a CPU extension whose loader is broken as shipped) -- runs them in
float64 under autograd on seeded inputs, and writes the inputs, outputs and
gradients to ``tests/golden/*.npz``.  The fixtures are what the committed tests
compare the oracle (and, on a GPU, the CUDA path) against; nothing at test time
reads the reference tree.
"""
from __future__ import annotations

import ast
import itertools
import math
import os
import sys
import types

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

HERE = os.path.dirname(os.path.abspath(__file__))


def load_class(path: str, name: str, extra=None):
    src = open(path).read()
    tree = ast.parse(src)
    for node in tree.body:
        if isinstance(node, ast.ClassDef) and node.name == name:
            seg = ast.get_source_segment(src, node)
            ns = {"torch": torch, "nn": nn, "F": F, "itertools": itertools, "math": math}
            ns.update(extra or {})
            exec(compile(seg, f"{path}:{name}", "exec"), ns)
            return ns[name]
    raise KeyError(name)


def load_function(path: str, name: str, extra=None):
    src = open(path).read()
    tree = ast.parse(src)
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name == name:
            seg = ast.get_source_segment(src, node)
            ns = {"torch": torch, "nn": nn, "F": F, "itertools": itertools, "math": math}
            ns.update(extra or {})
            exec(compile(seg, f"{path}:{name}", "exec"), ns)
            return ns[name]
    raise KeyError(name)


def run_probs_case(fn, cls, *, M, B, T, H, d, K, L, share_planes, logit_temp, seed):
    """The reference's race_bucket_probs_from_qk (misc/arxiv_64K.py:1580-1642)
    on a stand-in attention module holding the reference's BatchedACE."""
    torch.manual_seed(seed)
    ace = cls(d, K, L, M, device="cpu", share_planes=share_planes).double()
    with torch.no_grad():
        ace.logit_temp.fill_(logit_temp)
    attn = types.SimpleNamespace(ace=ace, M=M)
    x = lambda: torch.randn(B, T, H, d, dtype=torch.float32).double()
    q, k = x(), x()
    q.requires_grad_(True)
    k.requires_grad_(True)
    pq, pk = fn(attn, q, k)                                     # [M,B,H,T,L,R] each
    gq = torch.randn(pq.shape, dtype=torch.float32).double()
    gk = torch.randn(pk.shape, dtype=torch.float32).double()
    ((pq * gq).sum() + (pk * gk).sum()).backward()
    planes_T = ace.planes_T.detach()
    if planes_T.dim() == 2:
        planes_T = planes_T.unsqueeze(0)
    planes = planes_T.transpose(1, 2).contiguous()
    scale = float(ace.logit_temp.detach().exp().clamp(1e-2, 20.0))   # as the function computes it
    return dict(
        q=q.detach().float().numpy(), k=k.detach().float().numpy(),
        planes=planes.float().numpy(), probs_q=pq.detach().numpy(),
        probs_k=pk.detach().numpy(), gq=gq.float().numpy(), gk=gk.float().numpy(),
        dq=q.grad.numpy(), dk=k.grad.numpy(), scale=np.float64(scale),
        dlogit_temp=np.float64(ace.logit_temp.grad),
        meta=np.array([M, B, T, H, d, K, L, int(share_planes)], np.int64),
    )


PROBS_CASES = [
    # name, M, B, T, H, d, K, L, share_planes, logit_temp
    ("probs_k2l5_t40", 1, 2, 40, 2, 64, 2, 5, False, 0.0),
    ("probs_k3l3_t29_m2_shared", 2, 1, 29, 3, 32, 3, 3, True, math.log(0.7)),
]


def run_case(cls, *, causal, M, B, T, H, d, K, L, share_planes, logit_temp, seed):
    torch.manual_seed(seed)
    ace = cls(d, K, L, M, device="cpu", share_planes=share_planes).double()  # planes drawn in fp32
    if hasattr(ace, "logit_temp"):
        with torch.no_grad():
            ace.logit_temp.fill_(logit_temp)
    # inputs are drawn in float32 and widened, so the fp32 CUDA path sees the
    # exact same values the float64 reference run saw
    x = lambda: torch.randn(B, T, H, d, dtype=torch.float32).double()
    q, k, v = x(), x(), x()
    for t in (q, k, v):
        t.requires_grad_(True)
    pack = lambda z: z.unsqueeze(0).expand(M, -1, -1, -1, -1)   # misc/vit.py:1022-1028
    out = ace(pack(k), pack(v), pack(q))                        # [M,B,T,H,d]
    dout = torch.randn(out.shape, dtype=torch.float32).double()
    out.backward(dout)
    planes_T = ace.planes_T.detach()
    if planes_T.dim() == 2:
        planes_T = planes_T.unsqueeze(0)
    planes = planes_T.transpose(1, 2).contiguous()              # [Mp, L*K, d]
    if causal:
        scale = math.sqrt(d)                                    # misc/race.py:67
        dlt = 0.0
    else:
        scale = float(torch.tensor(logit_temp).exp().clamp(1e-2, 20.0))   # misc/vit.py:923
        dlt = float(ace.logit_temp.grad)
    return dict(
        q=q.detach().float().numpy(), k=k.detach().float().numpy(),
        v=v.detach().float().numpy(), planes=planes.float().numpy(),
        dout=dout.float().numpy(), out=out.detach().numpy(),
        dq=q.grad.numpy(), dk=k.grad.numpy(), dv=v.grad.numpy(),
        scale=np.float64(scale), dlogit_temp=np.float64(dlt),
        meta=np.array([M, B, T, H, d, K, L, int(share_planes), int(causal)], np.int64),
    )


CASES = [
    # name, causal, M, B, T, H, d, K, L, share_planes, logit_temp
    ("nc_k2l5_t64", False, 1, 1, 64, 2, 64, 2, 5, False, 0.0),
    ("nc_k3l3_t37_m2", False, 2, 2, 37, 1, 64, 3, 3, False, math.log(0.5)),
    ("nc_k2l4_t33_d32_shared", False, 2, 1, 33, 2, 32, 2, 4, True, math.log(3.0)),
    ("c_k2l5_t48", True, 1, 1, 48, 2, 64, 2, 5, True, 0.0),
    ("c_k3l2_t29_m2_indep", True, 2, 1, 29, 2, 64, 3, 2, False, 0.0),
    ("c_k1l8_t17_d32", True, 1, 2, 17, 1, 32, 1, 8, True, 0.0),
]


class _Const(nn.Module):
    """Stands in for a projection: returns a fixed leaf tensor whatever its input."""

    def __init__(self, t):
        super().__init__()
        self.t = t

    def forward(self, x):
        return self.t


def run_global_case(cls, *, B, T, H, dk, K, L, chunk, group, beta, masked, seed):
    """The reference's CausalRACEAttention (misc/elsaa_causal_complete.py:438-571)
    on its torch path, with the q/k/v projections replaced by the inputs
    themselves and the output projection by the identity, so the fixture holds
    the attention alone: out, d_token and the gradients of Q, K, V, log_beta."""
    torch.manual_seed(seed)
    att = cls(H * dk, H, 0.0, num_bits=K, num_tables=L, beta_init=beta, chunk_size=chunk,
              chunk_group_size=group).double()
    x = lambda: torch.randn(B, T, H * dk, dtype=torch.float32).double().requires_grad_(True)
    q, k, v = x(), x(), x()
    att.q, att.k, att.v, att.o = _Const(q), _Const(k), _Const(v), nn.Identity()
    mask = None
    if masked:
        mask = (torch.rand(B, T) > 0.25).double()
        mask[:, 0] = 1.0
    out, d_token = att(torch.zeros(B, T, H * dk, dtype=torch.float64), mask=mask, return_den=True)
    dout = torch.randn(out.shape, dtype=torch.float32).double()
    gtok = torch.randn(d_token.shape, dtype=torch.float32).double()
    ((out * dout).sum() + (d_token * gtok).sum()).backward()
    res = dict(
        q=q.detach().float().numpy(), k=k.detach().float().numpy(), v=v.detach().float().numpy(),
        planes=att.planes.detach().float().numpy(), out=out.detach().numpy(),
        d_token=d_token.detach().numpy(), dout=dout.float().numpy(), gtok=gtok.float().numpy(),
        dq=q.grad.numpy(), dk=k.grad.numpy(), dv=v.grad.numpy(),
        beta=np.float64(att.log_beta.detach().exp().clamp(1e-2, 20.0)),
        dlog_beta=np.float64(att.log_beta.grad),
        meta=np.array([B, T, H, dk, K, L, chunk, int(masked)], np.int64),
    )
    if masked:
        res["mask"] = mask.float().numpy()
    return res


GLOBAL_CASES = [
    # name, B, T, H, dk, K, L, chunk_size, chunk_group_size, beta_init, masked
    ("g_k2l4_t40", 2, 40, 2, 64, 2, 4, 16, None, 1.0, False),
    ("g_k3l3_t37_d32_mask", 1, 37, 3, 32, 3, 3, 8, 2, 0.7, True),
]


def main(ref_root: str):
    vit_cls = load_class(os.path.join(ref_root, "misc/vit.py"), "BatchedACE")
    race_cls = load_class(os.path.join(ref_root, "misc/race.py"), "BatchedACE")
    for i, (name, causal, M, B, T, H, d, K, L, sp, lt) in enumerate(CASES):
        cls = race_cls if causal else vit_cls
        res = run_case(cls, causal=causal, M=M, B=B, T=T, H=H, d=d, K=K, L=L,
                       share_planes=sp, logit_temp=lt, seed=i)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **res)
        print("wrote", path, os.path.getsize(path))
    fn = load_function(os.path.join(ref_root, "misc/arxiv_64K.py"), "race_bucket_probs_from_qk",
                       {"RACEAttention": object})
    for i, (name, M, B, T, H, d, K, L, sp, lt) in enumerate(PROBS_CASES):
        res = run_probs_case(fn, vit_cls, M=M, B=B, T=T, H=H, d=d, K=K, L=L, share_planes=sp,
                             logit_temp=lt, seed=100 + i)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **res)
        print("wrote", path, os.path.getsize(path))


def run_module_case(cls, cfg_or_args, *, kind, B, T, d_model, seed):
    """A reference attention module or block (random init drawn in float32,
    run in float64, dropout 0): x -> out, then the gradients of x and of every
    parameter for a random upstream gradient.  The state_dict is saved under
    ``sd/<name>`` so the drop-in modules load it unchanged."""
    torch.manual_seed(seed)
    if kind == "block":
        mod = cls(cfg_or_args, device="cpu")
    else:
        mod = cls(**cfg_or_args, device="cpu")
    mod = mod.double().eval()
    x = torch.randn(B, T, d_model, dtype=torch.float32).double().requires_grad_(True)
    out = mod(x)
    dout = torch.randn(out.shape, dtype=torch.float32).double()
    out.backward(dout)
    # float32 storage keeps the fixtures small: the state_dict and inputs are
    # float32 values, and rounding the float64 results to float32 (2^-24) is far
    # below the 1e-4 parity bar
    res = dict(x=x.detach().float().numpy(), dout=dout.float().numpy(),
               out=out.detach().float().numpy(), dx=x.grad.float().numpy())
    for name, t in mod.state_dict().items():
        res["sd/" + name] = t.detach().float().numpy()
    for name, prm in mod.named_parameters():
        if prm.grad is not None:
            res["grad/" + name] = prm.grad.float().numpy()
    return res


# name, file, class, kind, constructor args (or block cfg), B, T, d_model
MODULE_CASES = [
    ("mod_vit_attn_h2_m2", "misc/vit.py", "RACEAttention", "attn",
     dict(d_in=64, d_out=64, dropout=0.0, num_heads=2, L=5, K=2, N_M=2), 2, 37, 64),
    ("mod_vit_attn_h3_k4l4", "misc/vit.py", "RACEAttention", "attn",
     dict(d_in=96, d_out=64, dropout=0.0, num_heads=3, L=4, K=4, N_M=1), 2, 29, 96),
    ("mod_vit_block_h2", "misc/vit.py", "RACEBlock", "block",
     dict(embed_dim=64, num_heads=2, drop_rate=0.0, qkv_bias=True, L=5, K=2, M=1), 2, 41, 64),
    ("mod_race_attn_h2_m2", "misc/race.py", "RACEAttention", "attn",
     dict(d=64, h=2, K=2, L=5, M=2, drop=0.0), 2, 33, 64),
    ("mod_race_block_h2", "misc/race.py", "RACEBlock", "block",
     dict(emb_dim=64, n_heads=2, drop_rate=0.0, qkv_bias=False, K=3, L=3, M=1), 1, 45, 64),
]


def main_modules(ref_root: str):
    for i, (name, rel, clsname, kind, args, B, T, dm) in enumerate(MODULE_CASES):
        path = os.path.join(ref_root, rel)
        ace = load_class(path, "BatchedACE")
        extra = {"BatchedACE": ace}
        attn = load_class(path, "RACEAttention", extra)
        extra["RACEAttention"] = attn
        cls = attn if clsname == "RACEAttention" else load_class(path, clsname, extra)
        res = run_module_case(cls, args, kind=kind, B=B, T=T, d_model=dm, seed=300 + i)
        meta = dict(file=rel, cls=clsname, kind=kind, B=B, T=T, d_model=dm, **args)
        res["meta_json"] = np.array(__import__("json").dumps(meta))
        out = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(out, **res)
        print("wrote", out, os.path.getsize(out))


def main_global(ref_root: str):
    cls = load_class(os.path.join(ref_root, "misc/elsaa_causal_complete.py"), "CausalRACEAttention",
                     {"_HAS_TRITON_RACE": False})
    for i, (name, B, T, H, dk, K, L, C, g, beta, masked) in enumerate(GLOBAL_CASES):
        res = run_global_case(cls, B=B, T=T, H=H, dk=dk, K=K, L=L, chunk=C, group=g, beta=beta,
                              masked=masked, seed=200 + i)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **res)
        print("wrote", path, os.path.getsize(path))


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py REFERENCE_ROOT [all|global|modules]")
    root = sys.argv[1]
    which = sys.argv[2] if len(sys.argv) > 2 else "all"     # all | global | modules
    if which == "all":
        main(root)
    if which in ("all", "global"):
        main_global(root)
    if which in ("all", "modules"):
        main_modules(root)
