"""The drop-in modules against the reference's own RACEAttention / RACEBlock.

Fixtures (tests/golden/mod_*.npz, written by make_golden.py) hold a reference
module's state_dict, an input x, an upstream gradient and the module's float64
output and gradients (x and every parameter).  On the CPU: the state_dict
loads strictly into the drop-in module, and a numpy restatement of the
module's forward -- projections, the oracle, the reference's head merge
``permute(0, 2, 1, 3).reshape(B, T, H * d_k)`` -- reproduces the reference's
output (this pins the head-merge semantics).  On a GPU: the drop-in module
itself, forward and backward, at the path's 1e-4 relative L2.
"""
import numpy as np
import pytest
import torch

from oracle import race_oracle as O
from tests import golden_util as G

FILES = G.module_files()
IDS = [p.split("/")[-1][:-4] for p in FILES]


@pytest.mark.parametrize("path", FILES, ids=IDS)
def test_state_dict_loads_strictly(path):
    meta, sd, _ = G.load_module(path)
    mod = G.build_module(meta)
    mod.load_state_dict(sd, strict=True)


def _np_attention(meta, sd, x, prefix):
    """Forward of the reference attention module in numpy + the oracle."""
    w = lambda n: sd[prefix + n].double().numpy()
    vit = meta["file"] == "misc/vit.py"
    H = meta["num_heads"] if vit else meta["h"]
    K, L = meta["K"], meta["L"]
    M = meta["N_M"] if vit else meta["M"]
    names = ("q_proj", "k_proj", "v_proj", "out") if vit else ("q", "k", "v", "o")
    lin = lambda z, n: z @ w(n + ".weight").T + (w(n + ".bias") if prefix + n + ".bias" in sd
                                                 else 0.0)
    B, T, dm = x.shape
    dk = dm // H
    Q, Kx, V = (lin(x, n).reshape(B, T, H, dk) for n in names[:3])
    flat = lambda z: z.transpose(0, 2, 1, 3).reshape(B * H, T, dk)   # streams (b, h)
    pt = w("ace.planes_T")
    planes = pt.T[None] if pt.ndim == 2 else pt.transpose(0, 2, 1)    # [Mp, L*K, dk]
    if vit:
        scale = float(np.clip(np.exp(sd[prefix + "ace.logit_temp"].double().numpy()), 1e-2, 20.0))
    else:
        scale = float(np.sqrt(dk))
    outs = []
    for m in range(M):
        P = np.broadcast_to(planes[m if planes.shape[0] > 1 else 0], (B * H, K * L, dk))
        o = O.forward(flat(Q), flat(Kx), flat(V), P, K, L, scale, not vit)   # [B*H, T, dk]
        outs.append(o.reshape(B, H, T, dk).transpose(0, 2, 1, 3))          # [B, T, H, dk]
    out = np.mean(outs, axis=0)
    merged = out.transpose(0, 2, 1, 3).reshape(B, T, H * dk)   # the reference's head merge
    return lin(merged, names[3])


def _np_layernorm(z, wgt, b, eps=1e-5):
    mu = z.mean(-1, keepdims=True)
    var = z.var(-1, keepdims=True)
    return (z - mu) / np.sqrt(var + eps) * wgt + b


@pytest.mark.parametrize("path", FILES, ids=IDS)
def test_numpy_restatement_matches_reference_module(path):
    meta, sd, z = G.load_module(path)
    x = z["x"].astype(np.float64)
    if meta["kind"] == "attn":
        out = _np_attention(meta, sd, x, "")
    else:
        from math import erf, sqrt
        vit = meta["file"] == "misc/vit.py"
        am = dict(meta)
        if vit:
            am.update(num_heads=meta["num_heads"], N_M=meta["M"])
        else:
            am.update(h=meta["n_heads"])
        w = lambda n: sd[n].double().numpy()
        h = x
        a = _np_attention(am, sd, _np_layernorm(x, w("norm1.weight"), w("norm1.bias")), "att.")
        x1 = a + h
        y = _np_layernorm(x1, w("norm2.weight"), w("norm2.bias"))
        y = y @ w("ff.0.weight").T + w("ff.0.bias")
        y = 0.5 * y * (1.0 + np.vectorize(lambda t: erf(t / sqrt(2.0)))(y))
        y = y @ w("ff.2.weight").T + w("ff.2.bias")
        out = y + x1
    assert O.rel_l2(out, z["out"].astype(np.float64)) < 1e-6


def test_fused_qkv_matches_three_linears():
    """The one-GEMM q/k/v projection gives the three Linear layers' outputs and
    gradients (CPU, float64)."""
    from race_attention_b200.functional import fused_qkv
    torch.manual_seed(0)
    lins = [torch.nn.Linear(48, 48, bias=True).double() for _ in range(3)]
    x = torch.randn(2, 7, 48, dtype=torch.float64, requires_grad=True)
    q, k, v = fused_qkv(x, *lins, heads=3, head_dim=16)
    ref = [lin(x).view(2, 7, 3, 16) for lin in lins]
    for a, b in zip((q, k, v), ref):
        assert torch.allclose(a, b, rtol=1e-12, atol=1e-12)
    g = [torch.randn_like(a) for a in (q, k, v)]
    gx, *gw = torch.autograd.grad([q, k, v], [x] + [lin.weight for lin in lins], g)
    rx, *rw = torch.autograd.grad(ref, [x] + [lin.weight for lin in lins], g)
    assert torch.allclose(gx, rx, rtol=1e-12, atol=1e-12)
    for a, b in zip(gw, rw):
        assert torch.allclose(a, b, rtol=1e-12, atol=1e-12)


@pytest.mark.gpu
@pytest.mark.parametrize("fuse", [True, False], ids=["fused_qkv", "three_gemms"])
@pytest.mark.parametrize("path", FILES, ids=IDS)
def test_module_forward_backward_on_gpu(path, fuse):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    meta, sd, z = G.load_module(path)
    mod = G.build_module(meta, device="cuda")
    mod.load_state_dict(sd, strict=True)
    mod = mod.cuda().eval()
    (mod.att if meta["kind"] == "block" else mod).fuse_qkv = fuse
    x = torch.tensor(z["x"], device="cuda", requires_grad=True)
    out = mod(x)
    out.backward(torch.tensor(z["dout"], device="cuda"))
    c = lambda t: t.detach().double().cpu().numpy()
    assert O.rel_l2(c(out), z["out"]) < 1e-4
    assert O.rel_l2(c(x.grad), z["dx"]) < 1e-4
    grads = dict(mod.named_parameters())
    for key in z:
        if key.startswith("grad/"):
            name = key[5:]
            assert O.rel_l2(c(grads[name].grad), z[key]) < 1e-4, name
