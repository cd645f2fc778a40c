"""CUDA path vs the oracle and the golden vectors (needs a B200).

Tolerances (relative L2, from the path's specification): 1e-4 for float32
inputs, 2e-2 for bfloat16 inputs (the oracle then sees the same
bf16-rounded inputs).  Where the reference's own float32 op sequence
(oracle/torch_ref.py) is itself further than that from the float64 oracle
-- degenerate cases such as T = 1, where dq and dk are pure cancellation --
the bar is 4x the reference's own float32 error on the same inputs.
"""
import math

import numpy as np
import pytest
import torch

from oracle import race_oracle as O
from tests import golden_util as G
from tests.cuda_util import bf16_round, run_streams

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


def ref_fp32_error(q, k, v, planes, K, L, scale, causal, dout, refs, ref_ds=None):
    """Relative error of the reference's float32 op sequence (CPU) per output:
    relative L2 for out, dq, dk, dv, then (with ref_ds) the relative error of
    the temperature gradient."""
    from oracle import torch_ref
    qt, kt, vt = (torch.tensor(a, dtype=torch.float32, requires_grad=True) for a in (q, k, v))
    st = torch.tensor(float(scale), requires_grad=True)
    out = torch_ref.fwd_bwd(qt, kt, vt, torch.tensor(planes[0]).T, K, L, st,
                            torch_ref.protos_T(K), torch.tensor(dout, dtype=torch.float32),
                            causal)
    got = (out, qt.grad, kt.grad, vt.grad)
    errs = [O.rel_l2(a.detach().double().numpy(), b) for a, b in zip(got, refs)]
    if ref_ds is not None:
        g = 0.0 if st.grad is None else float(st.grad)
        errs.append(abs(g - ref_ds) / max(abs(ref_ds), 1e-30))
    return errs


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from race_attention_b200 import _lib
    _lib.load()   # fails loudly when the extension is missing


@pytest.mark.parametrize("path", G.golden_files(), ids=lambda p: p.split("/")[-1][:-4])
def test_golden(path):
    """Reference modules' own fp64 outputs/gradients on the same inputs."""
    from race_attention_b200 import race_attention
    g = G.load(path)
    M, B, T, H, d, K, L = (g[x] for x in ("M", "B", "T", "H", "d", "K", "L"))
    dev = "cuda"
    q, k, v = (torch.tensor(g[x], device=dev, requires_grad=True) for x in ("q", "k", "v"))
    pack = lambda z: z.unsqueeze(0).expand(M, -1, -1, -1, -1)
    planes = torch.tensor(g["planes"], device=dev)
    if g["causal"]:
        scale = torch.tensor(float(g["scale"]), device=dev)
        out = race_attention(pack(q), pack(k), pack(v), planes, K, L, scale, causal=True,
                             shared_planes=g["share"])
    else:
        lt = torch.tensor(math.log(float(g["scale"])), device=dev, requires_grad=True)
        scale = lt.exp().clamp(1e-2, 20.0)
        out = race_attention(pack(q), pack(k), pack(v), planes, K, L, scale, causal=False,
                             shared_planes=g["share"])
    out.backward(torch.tensor(g["dout"], device=dev))
    c = lambda t: t.detach().double().cpu().numpy()
    assert O.rel_l2(c(out), g["out"]) < 1e-4
    assert O.rel_l2(c(q.grad), g["dq"]) < 1e-4
    assert O.rel_l2(c(k.grad), g["dk"]) < 1e-4
    assert O.rel_l2(c(v.grad), g["dv"]) < 1e-4
    if not g["causal"]:
        assert math.isclose(float(lt.grad), float(g["dlogit_temp"]), rel_tol=1e-4, abs_tol=1e-6)


CASES = [
    # N, T, d, K, L, causal, chunk
    (2, 1, 64, 2, 5, False, 0),
    (3, 7, 64, 2, 5, False, 0),
    (2, 127, 64, 2, 5, True, 0),
    (2, 129, 64, 2, 5, True, 64),
    (1, 785, 64, 4, 2, False, 0),
    (1, 785, 64, 4, 2, True, 128),
    (4, 1000, 32, 1, 8, True, 128),
    (2, 3000, 64, 3, 3, False, 0),
    (2, 3000, 64, 3, 3, True, 0),
    (3, 2049, 32, 5, 1, False, 0),
    (1, 4096, 64, 2, 5, True, 256),
    (4, 4096, 64, 2, 5, False, 0),
    # above 32 buckets (non-causal): S = 64 (K4 L4, the ViT config), 40, 64 at K5
    (2, 785, 64, 4, 4, False, 0),
    (3, 1000, 64, 3, 5, False, 0),
    (1, 3000, 32, 5, 2, False, 0),
    (2, 4096, 64, 4, 4, False, 0),
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("N,T,d,K,L,causal,chunk", CASES)
def test_vs_oracle(N, T, d, K, L, causal, chunk, dtype):
    rng = np.random.default_rng(N * 7919 + T * 31 + d + K * 3 + L)
    q, k, v, dout = (rng.standard_normal((N, T, d)).astype(np.float32) for _ in range(4))
    planes = rng.standard_normal((1, K * L, d)).astype(np.float32)
    scale = 0.8 if causal else 1.3
    if dtype == torch.bfloat16:
        q, k, v, dout = (bf16_round(a) for a in (q, k, v, dout))
    got = run_streams(q, k, v, planes, K, L, scale, causal, dout, dtype=dtype, chunk=chunk)
    P = np.broadcast_to(planes, (N,) + planes.shape[1:])
    ref_out = O.forward(q, k, v, P, K, L, scale, causal)
    (dq, dk, dv, ds), ds_mag = O.dscale_magnitude(O.backward, q, k, v, P, K, L, scale, causal,
                                                  dout)
    tol = TOL[dtype]
    floors = ref_fp32_error(q, k, v, planes, K, L, scale, causal, dout, (ref_out, dq, dk, dv), ds)
    for name, a, b, fl in zip(("out", "dq", "dk", "dv"), got[:4], (ref_out, dq, dk, dv), floors):
        bar = max(tol, 4 * fl)
        assert O.rel_l2(a, b) < bar, (name, O.rel_l2(a, b), bar)
    # the temperature gradient is held to the same bar relative to itself (4x
    # the reference's own float32 error where that is larger), or -- where it
    # is a near-total cancellation, as at T = 1 -- to the bar relative to the
    # sum of the magnitudes of the terms it adds up
    bar = max(tol, 4 * floors[4])
    if T == 1:
        # one token: E = v exactly up to eps, so dpQ and dpK cancel to zero in
        # exact arithmetic and the temperature gradient is an eps-sized
        # remainder of that cancellation; held to 16x the reference's own
        # float32 error on it
        bar = max(tol, 16 * floors[4])
    assert math.isclose(got[4], ds, rel_tol=bar, abs_tol=tol * ds_mag), (got[4], ds, bar, ds_mag)


def test_deterministic():
    rng = np.random.default_rng(5)
    N, T, d, K, L = 2, 5000, 64, 2, 5
    q, k, v, dout = (rng.standard_normal((N, T, d)).astype(np.float32) for _ in range(4))
    planes = rng.standard_normal((1, K * L, d)).astype(np.float32)
    for causal in (False, True):
        a = run_streams(q, k, v, planes, K, L, 1.0, causal, dout)
        b = run_streams(q, k, v, planes, K, L, 1.0, causal, dout)
        for x, y in zip(a[:4], b[:4]):
            assert np.array_equal(x, y)
        assert a[4] == b[4]


def test_chunk_length_independent():
    rng = np.random.default_rng(9)
    N, T, d, K, L = 1, 6000, 64, 2, 5
    q, k, v, dout = (rng.standard_normal((N, T, d)).astype(np.float32) for _ in range(4))
    planes = rng.standard_normal((1, K * L, d)).astype(np.float32)
    a = run_streams(q, k, v, planes, K, L, 1.0, True, dout, chunk=128)
    b = run_streams(q, k, v, planes, K, L, 1.0, True, dout, chunk=1024)
    for x, y in zip(a[:4], b[:4]):
        assert O.rel_l2(x, y) < 1e-5


@pytest.mark.parametrize("causal", [False, True], ids=["noncausal", "causal"])
def test_broadcast_batch_layout(causal):
    """A batch axis broadcast with stride 0 (one sequence shared by two batch
    rows) cannot be walked by the copy engine's tensor maps; the library then
    runs the warp-level kernels (non-causal), or the autograd layer
    materialises the broadcast (per-bucket causal, whose kernels stream every
    input by TMA).  Results must match two explicit copies within the path's
    fp32 bar of 1e-4."""
    from race_attention_b200 import race_attention
    dev = "cuda"
    g = torch.Generator().manual_seed(5)
    T, d, K, L = 700, 64, 2, 5
    base = [torch.randn(1, T, 1, d, generator=g) for _ in range(3)]
    planes = torch.randn(1, K * L, d, generator=g).to(dev)
    dout = torch.randn(2, T, 1, d, generator=g).to(dev)
    scale = torch.tensor(1.1, device=dev)
    outs = []
    for expand in (True, False):
        leaves = [b.to(dev).requires_grad_(True) for b in base]
        ins = [x.expand(2, -1, -1, -1) if expand else x.repeat(2, 1, 1, 1) for x in leaves]
        out = race_attention(*ins, planes, K, L, scale, causal=causal)
        out.backward(dout)
        outs.append([out.detach()] + [x.grad.detach() for x in leaves])
    for a, b in zip(*outs):
        assert O.rel_l2(a.double().cpu().numpy(), b.double().cpu().numpy()) < 1e-4


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_contiguous_layouts_run_tcgen05_kernels(dtype):
    """Ordinary layouts -- contiguous [M, B, T, H, d], the smoke test's
    unsqueezed [1, B, T, 1, d], and the stride-0 ensemble expansion of the
    modules -- must run the tcgen05 + TMA kernels: the autograd layer asks the
    library for strict mode, so a tensor map that fails to encode is an
    error rather than a silent fallback, and the kernel log names the
    tcgen05 kernels."""
    from race_attention_b200 import _lib, race_attention
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(2)
    planes = torch.randn(1, 10, 64, generator=g, device=dev)
    layouts = {
        "unsqueezed": lambda: torch.randn(2, 300, 64, generator=g, device=dev)[None, :, :, None],
        "bthd": lambda: torch.randn(1, 2, 300, 3, 64, generator=g, device=dev),
        "expanded": lambda: torch.randn(2, 300, 3, 64, generator=g, device=dev)[None].expand(
            2, -1, -1, -1, -1),
    }
    for name, make in layouts.items():
        q, k, v = (make().to(dtype).requires_grad_(True) for _ in range(3))
        out = race_attention(q, k, v, planes, 2, 5, 1.0)
        fwd = _lib.last_kernels()
        out.backward(torch.randn_like(out))
        torch.cuda.synchronize()
        bwd = _lib.last_kernels()
        assert "t5_reduce" in fwd and "t5_readout" in fwd, (name, fwd)
        assert "t5_bwd_q" in bwd and "t5_bwd_kv" in bwd, (name, bwd)
        assert not any(x.startswith("tc_") for x in fwd + bwd), (name, fwd, bwd)


def test_broadcast_layout_is_logged_as_fallback():
    from race_attention_b200 import _lib, race_attention
    dev = "cuda"
    x = torch.randn(1, 300, 1, 64, device=dev).expand(2, -1, -1, -1)
    planes = torch.randn(1, 10, 64, device=dev)
    race_attention(x, x, x, planes, 2, 5, 1.0)
    log = _lib.last_kernels()
    assert any("fallback: q: broadcast batch axis" in e or "fallback: k: broadcast batch axis" in e
               for e in log), log


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("causal", [False, True], ids=["noncausal", "causal"])
def test_normalize_qk(causal, dtype):
    """normalize_qk=True hashes q/|q| and k/|k|: the oracle on the normalised
    inputs, its gradients taken back through the normalisation; inputs with
    a wide spread of row norms so that the flag matters."""
    from race_attention_b200 import race_attention
    rng = np.random.default_rng(11 + causal)
    N, T, d, K, L = 2, 1500, 64, 2, 5
    q, k, v, dout = (rng.standard_normal((N, T, d)).astype(np.float32) for _ in range(4))
    q *= rng.uniform(0.1, 20.0, (N, T, 1)).astype(np.float32)
    k *= rng.uniform(0.1, 20.0, (N, T, 1)).astype(np.float32)
    if dtype == torch.bfloat16:
        q, k, v, dout = (bf16_round(a) for a in (q, k, v, dout))
    planes = rng.standard_normal((1, K * L, d)).astype(np.float32)
    dev = "cuda"
    to = lambda a: torch.tensor(a, device=dev).to(dtype)[None, :, :, None]
    qt, kt, vt = (to(a).requires_grad_(True) for a in (q, k, v))
    out = race_attention(qt, kt, vt, torch.tensor(planes, device=dev), K, L, 1.0, causal=causal,
                         normalize_qk=True)
    out.backward(to(dout))
    f = lambda t: t.detach().float()[0, :, :, 0].cpu().numpy().astype(np.float64)
    P = np.broadcast_to(planes, (N, K * L, d))
    qn, kn = O.l2_normalize(q), O.l2_normalize(k)
    ref = O.forward(qn, kn, v, P, K, L, 1.0, causal)
    dqn, dkn, dv, _ = O.backward(qn, kn, v, P, K, L, 1.0, causal, dout)
    dq, dk = O.l2_normalize_backward(q, dqn), O.l2_normalize_backward(k, dkn)
    tol = TOL[dtype]
    for name, a, b in (("out", out, ref), ("dq", qt.grad, dq), ("dk", kt.grad, dk),
                       ("dv", vt.grad, dv)):
        assert O.rel_l2(f(a), b) < tol, (name, O.rel_l2(f(a), b))
    # the flag changes the result (tanh is not scale-invariant)
    plain = O.forward(q, k, v, P, K, L, 1.0, causal)
    assert O.rel_l2(plain, ref) > 10 * tol
