"""CPU oracle (numpy, float64) for RACE attention forward and backward.

TEST INFRASTRUCTURE ONLY: this module is the parity checker.  The product path
(``race_attention_b200``) never imports it.

Parity pin: checked against golden vectors produced by running the reference's
own torch modules under autograd (``tests/golden/make_golden.py``) and against
the reference's compiled OpenMP prefix-mean kernel (``oracle/_ref``, built by
``oracle/Makefile`` from ``kernels/cpu/race_pref.cpp``).

Notation: N streams, T tokens, D head dim, K hyperplanes per table, L tables,
R = 2**K buckets per table, S = L*R.

Reference semantics restated here (paths inside the reference project):
  * corners in ``itertools.product([-1, +1], repeat=K)`` order
    (``misc/vit.py:911-912``, ``misc/race.py:54-58``)
  * soft hash ``softmax(tanh(x @ planes_T) / scale @ protos_T)`` per table
    (``misc/vit.py:943-958``, ``misc/race.py:79-105``)
  * non-causal aggregation ``E = (pK^T V) / (sum_t pK + eps)`` and readout
    ``out = pQ @ E`` summed over all L*R buckets (``misc/vit.py:967-975``)
  * causal per-bucket prefix mean (``misc/race.py:108-138``,
    ``kernels/cpu/race_pref.cpp:36-101``) and its backward
    (``kernels/cpu/race_pref.cpp:104-220``).
  * causal global normalisation, one denominator per token over all buckets
    (``misc/elsaa_causal_complete.py:520-571``, ``misc/race_kernel.py:9-124``),
    pinned by golden vectors of the reference's ``CausalRACEAttention``.
"""
from __future__ import annotations

import itertools

import numpy as np


def corners(K: int) -> np.ndarray:
    """[R, K] bucket prototypes, ``itertools.product`` order (misc/vit.py:911)."""
    return np.array(list(itertools.product([-1.0, 1.0], repeat=K)), dtype=np.float64)


def soft_hash(x, planes, K, L, scale):
    """Soft bucket probabilities.

    x: [N, T, D]; planes: [N, L*K, D] (the hyperplanes each stream uses).
    Returns probs [N, T, L*R] (table-major, as misc/vit.py:962-963 flattens)
    plus the intermediates (h = tanh(proj)) the backward needs.
    """
    x = np.asarray(x, np.float64)
    planes = np.asarray(planes, np.float64)
    N, T, D = x.shape
    proj = np.einsum("ntd,njd->ntj", x, planes, optimize=True)  # misc/vit.py:943-944
    h = np.tanh(proj).reshape(N, T, L, K)
    logits = (h / scale) @ corners(K).T                   # misc/vit.py:955-956
    logits = logits - logits.max(-1, keepdims=True)
    e = np.exp(logits)
    p = e / e.sum(-1, keepdims=True)                      # misc/vit.py:957-958
    return p.reshape(N, T, L * (1 << K)), h


# Sums of |du h| / scale^2 of the soft_hash_backward calls since the last
# dscale_magnitude() -- the size of the terms the (heavily cancelling)
# temperature gradient adds up, i.e. the scale of its rounding error.
_DSCALE_ABS = []


def dscale_magnitude(fn, *args, **kw):
    """Runs a backward function and returns (its result, sum over its
    soft_hash_backward calls of |du h| / scale^2)."""
    _DSCALE_ABS.clear()
    res = fn(*args, **kw)
    return res, float(sum(_DSCALE_ABS))


def soft_hash_backward(dp, p, h, planes, K, L, scale):
    """Back-propagate d(probs) through softmax, the corner matmul, /scale and tanh.

    Returns (dx [N,T,D], dscale scalar).
    """
    N, T, S = dp.shape
    R = 1 << K
    c = corners(K)                                        # [R, K]
    p4 = p.reshape(N, T, L, R)
    dp4 = dp.reshape(N, T, L, R)
    g = p4 * (dp4 - (p4 * dp4).sum(-1, keepdims=True))    # d logits
    du = g @ c                                            # [N,T,L,K]; u = h/scale
    dh = du / scale
    dscale = float(-(du * h).sum() / scale / scale)
    _DSCALE_ABS.append(float(np.abs(du * h).sum() / scale / scale))
    dproj = (dh * (1.0 - h * h)).reshape(N, T, L * K)
    dx = np.einsum("ntj,njd->ntd", dproj, np.asarray(planes, np.float64), optimize=True)
    return dx, dscale


# ----------------------------------------------------------------------------- non-causal
def noncausal_forward(q, k, v, planes, K, L, scale, eps=1e-6):
    """misc/vit.py:918-978 for one ensemble slice: returns (out, A, Bsum)."""
    pK, _ = soft_hash(k, planes, K, L, scale)
    pQ, _ = soft_hash(q, planes, K, L, scale)
    v = np.asarray(v, np.float64)
    Bsum = np.einsum("nts,ntd->nsd", pK, v, optimize=True)  # misc/vit.py:967
    A = pK.sum(1)                                         # misc/vit.py:969
    E = Bsum / (A[..., None] + eps)                       # misc/vit.py:972
    out = np.einsum("nts,nsd->ntd", pQ, E, optimize=True)  # misc/vit.py:975
    return out, A, Bsum


def noncausal_backward(q, k, v, planes, K, L, scale, dout, eps=1e-6):
    """Analytic gradient of ``noncausal_forward``: (dq, dk, dv, dscale)."""
    pK, hK = soft_hash(k, planes, K, L, scale)
    pQ, hQ = soft_hash(q, planes, K, L, scale)
    v = np.asarray(v, np.float64)
    dout = np.asarray(dout, np.float64)
    Bsum = np.einsum("nts,ntd->nsd", pK, v, optimize=True)
    A = pK.sum(1)
    inv = 1.0 / (A + eps)
    E = Bsum * inv[..., None]
    dpQ = np.einsum("ntd,nsd->nts", dout, E, optimize=True)
    dE = np.einsum("nts,ntd->nsd", pQ, dout, optimize=True)
    dB = dE * inv[..., None]
    dA = -(dB * E).sum(-1)
    dv = np.einsum("nts,nsd->ntd", pK, dB, optimize=True)
    dpK = np.einsum("ntd,nsd->nts", v, dB, optimize=True) + dA[:, None, :]
    dq, dsq = soft_hash_backward(dpQ, pQ, hQ, planes, K, L, scale)
    dk, dsk = soft_hash_backward(dpK, pK, hK, planes, K, L, scale)
    return dq, dk, dv, dsq + dsk


# ----------------------------------------------------------------------------- causal
def prefix_mean_flat(w, V, eps=1e-6):
    """kernels/cpu/race_pref.cpp:36-101: w [NS,T], V [NS,T,D] -> E [NS,T,D]."""
    w = np.asarray(w, np.float64)
    V = np.asarray(V, np.float64)
    A = np.cumsum(w, axis=1)
    B = np.cumsum(w[..., None] * V, axis=1)
    return B / (A[..., None] + eps)


def prefix_mean_flat_backward(w, V, gE, eps=1e-6):
    """kernels/cpu/race_pref.cpp:104-220: returns (grad_w [NS,T], grad_V [NS,T,D])."""
    w = np.asarray(w, np.float64)
    V = np.asarray(V, np.float64)
    gE = np.asarray(gE, np.float64)
    A = np.cumsum(w, axis=1)
    B = np.cumsum(w[..., None] * V, axis=1)
    invA = 1.0 / (A + eps)
    alpha = -(invA ** 2) * (gE * B).sum(-1)                       # race_pref.cpp:175-181
    beta = gE * invA[..., None]
    beta_suf = np.cumsum(beta[:, ::-1], axis=1)[:, ::-1]          # race_pref.cpp:194-199
    alpha_suf = np.cumsum(alpha[:, ::-1], axis=1)[:, ::-1]
    gw = alpha_suf + (beta_suf * V).sum(-1)                       # race_pref.cpp:202-208
    gV = w[..., None] * beta_suf                                  # race_pref.cpp:210-215
    return gw, gV


def _causal_states(pK, v, eps):
    A = np.cumsum(pK, axis=1)                                     # [N,T,S]
    B = np.cumsum(pK[..., None] * v[:, :, None, :], axis=1)       # [N,T,S,D]
    return A, B


def causal_forward(q, k, v, planes, K, L, scale, eps=1e-6):
    """misc/race.py:63-142 (per-bucket normalised prefix mean): returns out."""
    pK, _ = soft_hash(k, planes, K, L, scale)
    pQ, _ = soft_hash(q, planes, K, L, scale)
    v = np.asarray(v, np.float64)
    A, B = _causal_states(pK, v, eps)
    E = B / (A[..., None] + eps)                                  # misc/race.py:110
    return np.einsum("nts,ntsd->ntd", pQ, E, optimize=True)  # misc/race.py:135-138


def causal_backward(q, k, v, planes, K, L, scale, dout, eps=1e-6):
    """Gradient of ``causal_forward`` built on the race_pref.cpp backward: (dq, dk, dv, dscale)."""
    pK, hK = soft_hash(k, planes, K, L, scale)
    pQ, hQ = soft_hash(q, planes, K, L, scale)
    v = np.asarray(v, np.float64)
    dout = np.asarray(dout, np.float64)
    N, T, S = pK.shape
    D = v.shape[-1]
    A, B = _causal_states(pK, v, eps)
    E = B / (A[..., None] + eps)
    dpQ = np.einsum("ntd,ntsd->nts", dout, E, optimize=True)
    # per-bucket streams, flat layout [N*S, T(, D)] as race_pref.cpp expects
    w_flat = pK.transpose(0, 2, 1).reshape(N * S, T)
    V_flat = np.broadcast_to(v[:, None], (N, S, T, D)).reshape(N * S, T, D)
    gE = (pQ.transpose(0, 2, 1)[..., None] * dout[:, None]).reshape(N * S, T, D)
    gw, gV = prefix_mean_flat_backward(w_flat, V_flat, gE, eps)
    dpK = gw.reshape(N, S, T).transpose(0, 2, 1)
    dv = gV.reshape(N, S, T, D).sum(1)
    dq, dsq = soft_hash_backward(dpQ, pQ, hQ, planes, K, L, scale)
    dk, dsk = soft_hash_backward(dpK, pK, hK, planes, K, L, scale)
    return dq, dk, dv, dsq + dsk


# ------------------------------------------------------- causal, streamed in chunks
def causal_streamed(q, k, v, planes, K, L, scale, dout=None, eps=1e-6, chunk=2048, threads=None):
    """``causal_forward`` / ``causal_backward`` in bounded memory, for long sequences.

    Same float64 quantities as the dense restatement above (misc/race.py:108-138
    forward, kernels/cpu/race_pref.cpp:104-220 backward), but the [T, S, D]
    prefix states are never materialised.  The token axis is cut into chunks;
    each chunk's entering state is an exclusive scan of the chunk totals
    (sum pK, pK^T v), after which the chunks are independent and run on a
    thread pool.  The backward uses the identities of race_pref.cpp with
    W = pQ / (A + eps): alpha = -W * (dout . E) (race_pref.cpp:175-181) and
    beta = W dout, whose suffix sums (race_pref.cpp:194-199) are carried across
    chunks the same way in reverse.
    Returns ``out`` when ``dout`` is None, else ``(out, dq, dk, dv, dscale)``.
    """
    from concurrent.futures import ThreadPoolExecutor
    import os

    pK, hK = soft_hash(k, planes, K, L, scale)
    pQ, hQ = soft_hash(q, planes, K, L, scale)
    v = np.asarray(v, np.float64)
    N, T, S = pK.shape
    D = v.shape[-1]
    spans = [(c0, min(T, c0 + chunk)) for c0 in range(0, T, chunk)]
    pool = ThreadPoolExecutor(threads or min(32, os.cpu_count() or 1))
    out = np.empty((N, T, D))
    bwd = dout is not None
    if bwd:
        dout = np.asarray(dout, np.float64)
        dpQ = np.empty((N, T, S))
    A = np.cumsum(pK, axis=1)                                           # [N,T,S]
    inv = 1.0 / (A + eps)
    for n in range(N):
        tot = np.stack([pK[n, c0:c1].T @ v[n, c0:c1] for c0, c1 in spans])   # [C,S,D]
        B0 = np.cumsum(tot, axis=0) - tot                                     # entering states

        def fwd_chunk(ci, n=n, B0=B0):
            c0, c1 = spans[ci]
            b = B0[ci] + np.cumsum(pK[n, c0:c1, :, None] * v[n, c0:c1, None, :], axis=0)
            E = b * inv[n, c0:c1, :, None]                                    # misc/race.py:110
            out[n, c0:c1] = np.einsum("ts,tsd->td", pQ[n, c0:c1], E, optimize=True)
            if bwd:
                dpQ[n, c0:c1] = np.einsum("td,tsd->ts", dout[n, c0:c1], E, optimize=True)

        list(pool.map(fwd_chunk, range(len(spans))))
    if not bwd:
        pool.shutdown()
        return out
    W = pQ * inv
    alpha = -W * dpQ                                                    # race_pref.cpp:175-181
    a_suf = np.cumsum(alpha[:, ::-1], axis=1)[:, ::-1]                  # race_pref.cpp:194-199
    dpK = np.empty((N, T, S))
    dv = np.empty((N, T, D))
    for n in range(N):
        tot = np.stack([W[n, c0:c1].T @ dout[n, c0:c1] for c0, c1 in spans])  # [C,S,D]
        after = tot[::-1].cumsum(axis=0)[::-1] - tot                          # later chunks

        def bwd_chunk(ci, n=n, after=after):
            c0, c1 = spans[ci]
            beta = W[n, c0:c1, :, None] * dout[n, c0:c1, None, :]
            b_suf = np.cumsum(beta[::-1], axis=0)[::-1] + after[ci]
            dpK[n, c0:c1] = a_suf[n, c0:c1] + np.einsum("tsd,td->ts", b_suf, v[n, c0:c1],
                                                        optimize=True)      # race_pref.cpp:202-208
            dv[n, c0:c1] = np.einsum("ts,tsd->td", pK[n, c0:c1], b_suf, optimize=True)  # :210-215

        list(pool.map(bwd_chunk, range(len(spans))))
    pool.shutdown()
    dq, dsq = soft_hash_backward(dpQ, pQ, hQ, planes, K, L, scale)
    dk, dsk = soft_hash_backward(dpK, pK, hK, planes, K, L, scale)
    return out, dq, dk, dv, dsq + dsk


# ------------------------------------------------------- causal, global normalisation
def causal_global(q, k, v, planes, K, L, scale, dout=None, dden=None, eps=1e-6):
    """Global-normalised causal RACE (the chunked ELSAA form).

    misc/elsaa_causal_complete.py:520-571 (CausalRACEAttention.forward, the
    torch path) and misc/race_kernel.py:9-124 (the Triton chunk kernel): with
    inclusive prefixes A_s(t) = sum_{u<=t} pK_s(u), B_s(t) = sum_{u<=t} pK_s(u) v(u),
    num(t) = sum_s pQ_s(t) B_s(t), den(t) = sum_s pQ_s(t) A_s(t) (summed over
    tables, like den_sumL) and out = num / max(den, eps).  The chunking of the
    reference only reorganises these sums.  Here ``scale`` is 1 / beta
    (beta = exp(log_beta).clamp(1e-2, 20), misc/elsaa_causal_complete.py:502-506).

    Returns (out, den) when ``dout`` is None, else
    (out, den, dq, dk, dv, dscale); ``dden`` is an optional incoming gradient
    of den.  Backward (derived from the forward above):
      gnum = dout / dd, gden = -(dout . out) / dd (0 where the clamp holds) + dden
      dpQ_s(t) = B_s(t) . gnum(t) + A_s(t) gden(t)
      dA_s(t) = pQ_s gden, dB_s(t) = pQ_s gnum, pushed to every key u <= t.
    """
    pK, hK = soft_hash(k, planes, K, L, scale)
    pQ, hQ = soft_hash(q, planes, K, L, scale)
    v = np.asarray(v, np.float64)
    A, B = _causal_states(pK, v, eps)
    num = np.einsum("nts,ntsd->ntd", pQ, B, optimize=True)
    den = np.einsum("nts,nts->nt", pQ, A)
    dd = np.maximum(den, eps)
    out = num / dd[..., None]
    if dout is None:
        return out, den
    dout = np.asarray(dout, np.float64)
    gnum = dout / dd[..., None]
    gden = np.where(den >= eps, -(dout * out).sum(-1) / dd, 0.0)
    if dden is not None:
        gden = gden + np.asarray(dden, np.float64)
    dpQ = np.einsum("ntsd,ntd->nts", B, gnum, optimize=True) + A * gden[..., None]
    alpha = pQ * gden[..., None]                                  # d A_s(t)
    beta = pQ[..., None] * gnum[:, :, None, :]                    # d B_s(t)
    a_suf = np.cumsum(alpha[:, ::-1], axis=1)[:, ::-1]
    b_suf = np.cumsum(beta[:, ::-1], axis=1)[:, ::-1]
    dpK = a_suf + np.einsum("ntsd,ntd->nts", b_suf, v, optimize=True)
    dv = np.einsum("nts,ntsd->ntd", pK, b_suf, optimize=True)
    dq, dsq = soft_hash_backward(dpQ, pQ, hQ, planes, K, L, scale)
    dk, dsk = soft_hash_backward(dpK, pK, hK, planes, K, L, scale)
    return out, den, dq, dk, dv, dsq + dsk


def l2_normalize(x, floor=1e-12):
    """x / max(|x|, floor) over the head dimension: torch.nn.functional.normalize
    (dim=-1), as the reference's angular baselines apply it to q and k
    (misc/vit.py:2559-2560, misc/classification.py:370-371).  The RACE path's
    optional normalize_qk flag hashes these instead of q and k."""
    x = np.asarray(x, np.float64)
    n = np.linalg.norm(x, axis=-1, keepdims=True)
    return x / np.maximum(n, floor)


def l2_normalize_backward(x, g, floor=1e-12):
    """Gradient through l2_normalize: (g - xn (xn . g)) / |x| (g / floor where
    |x| < floor, where the clamp has zero derivative)."""
    x = np.asarray(x, np.float64)
    g = np.asarray(g, np.float64)
    n = np.linalg.norm(x, axis=-1, keepdims=True)
    clamp = n < floor
    nn_ = np.where(clamp, floor, n)
    xn = x / nn_
    c = np.where(clamp, 0.0, (xn * g).sum(-1, keepdims=True))
    return (g - xn * c) / nn_


def forward(q, k, v, planes, K, L, scale, causal, eps=1e-6):
    if causal:
        return causal_forward(q, k, v, planes, K, L, scale, eps)
    return noncausal_forward(q, k, v, planes, K, L, scale, eps)[0]


def backward(q, k, v, planes, K, L, scale, causal, dout, eps=1e-6):
    fn = causal_backward if causal else noncausal_backward
    return fn(q, k, v, planes, K, L, scale, dout, eps)


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b.ravel())
    return float(np.linalg.norm((a - b).ravel()) / (den if den > 0 else 1.0))
