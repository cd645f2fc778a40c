"""Sequence sharding host logic on 2 CPU ranks (gloo).

The exchange steps of race_attention_b200.sequence_parallel (all-reduce of
the non-causal bucket sums, exclusive scans of the causal rank totals in
both directions) run for real over torch.distributed; the per-rank compute
is a numpy stand-in built from the oracle's soft hash (test-only).  The
concatenated shard results must equal the oracle on the whole sequence.
"""
import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import race_oracle as O
from race_attention_b200.sequence_parallel import exchange_backward_state, exchange_forward_state

N, T, D, K, L, SCALE, EPS = 2, 60, 8, 2, 2, 0.9, 1e-6
MODES = ("nc", "bucket", "global")   # non-causal; causal per-bucket; causal global


def data():
    rng = np.random.default_rng(3)
    q, k, v, do = (rng.standard_normal((N, T, D)) for _ in range(4))
    P = rng.standard_normal((N, K * L, D))
    return q, k, v, do, P


def shard_fwd_bwd(rank, world, mode):
    causal = mode != "nc"
    glob = mode == "global"
    q, k, v, do, P = data()
    lo, hi = T * rank // world, T * (rank + 1) // world
    q, k, v, do = (x[:, lo:hi] for x in (q, k, v, do))
    pK, hK = O.soft_hash(k, P, K, L, SCALE)
    pQ, hQ = O.soft_hash(q, P, K, L, SCALE)
    S = pK.shape[-1]
    # ---- forward: local state, exchange, readout
    Bl = np.einsum("nts,ntd->nsd", pK, v)
    Al = pK.sum(1)
    local_total = torch.tensor(np.concatenate([Bl, Al[..., None]], -1))     # [N,S,D+1]
    if not causal:
        state = local_total.clone()
        exchange_forward_state(state, None, False, None, None)
        B, A = state[..., :D].numpy(), state[..., D].numpy()
        E = B / (A[..., None] + EPS)
        out = np.einsum("nts,nsd->ntd", pQ, E)
    else:
        state = torch.zeros_like(local_total)                                   # rank-local prefix
        def add(off):
            state.add_(off)
        exchange_forward_state(state, local_total.clone(), True, None, add)
        B0, A0 = state[..., :D].numpy(), state[..., D].numpy()
        Acum = A0[:, None] + np.cumsum(pK, 1)
        Bcum = B0[:, None] + np.cumsum(pK[..., None] * v[:, :, None], 1)
        if glob:   # one denominator per token (the ELSAA form)
            den = (pQ * Acum).sum(-1)
            out = np.einsum("nts,ntsd->ntd", pQ, Bcum) / np.maximum(den, EPS)[..., None]
        else:
            out = np.einsum("nts,ntsd->ntd", pQ, Bcum / (Acum[..., None] + EPS))
    # ---- backward
    if not causal:
        gstate = torch.tensor(np.einsum("nts,ntd->nsd", pQ, do))
        exchange_backward_state(gstate, None, False, None, None)
        dE = gstate.numpy()
        inv = 1.0 / (A + EPS)
        dpQ = np.einsum("ntd,nsd->nts", do, E)
        dB = dE * inv[..., None]
        dA = -(dB * E).sum(-1)
        dv = np.einsum("nts,nsd->ntd", pK, dB)
        dpK = np.einsum("ntd,nsd->nts", v, dB) + dA[:, None]
    elif glob:
        dd = np.maximum(den, EPS)
        W = pQ / dd[..., None]
        R = np.einsum("ntd,ntsd->nts", do, Bcum)
        gden = -(W * R).sum(-1) / dd
        dpQ = R / dd[..., None] + Acum * gden[..., None]
        alpha = pQ * gden[..., None]
    else:
        invA = 1.0 / (Acum + EPS)
        W = pQ * invA
        dpQ = np.einsum("ntd,ntsd->nts", do, Bcum) * invA
        alpha = -W * dpQ
    if causal:
        GB = np.einsum("nts,ntd->nsd", W, do)
        GA = alpha.sum(1)
        gtotal = torch.tensor(np.concatenate([GB, GA[..., None]], -1))
        gstate = torch.zeros_like(gtotal)
        def gadd(off):
            gstate.add_(off)
        exchange_backward_state(gstate, gtotal.clone(), True, None, gadd)
        GB0, GA0 = gstate[..., :D].numpy(), gstate[..., D].numpy()
        beta = GB0[:, None] + np.cumsum((W[..., None] * do[:, :, None])[:, ::-1], 1)[:, ::-1]
        asuf = GA0[:, None] + np.cumsum(alpha[:, ::-1], 1)[:, ::-1]
        dv = np.einsum("nts,ntsd->ntd", pK, beta)
        dpK = asuf + np.einsum("ntsd,ntd->nts", beta, v)
    dq, dsq = O.soft_hash_backward(dpQ, pQ, hQ, P, K, L, SCALE)
    dk, dsk = O.soft_hash_backward(dpK, pK, hK, P, K, L, SCALE)
    ds = torch.tensor([dsq + dsk], dtype=torch.float64)
    dist.all_reduce(ds)
    return out, dq, dk, dv, float(ds)


def worker(rank, world, port, outdir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        for mode in MODES:
            res = shard_fwd_bwd(rank, world, mode)
            np.savez(os.path.join(outdir, f"r{rank}_{mode}.npz"), out=res[0], dq=res[1],
                     dk=res[2], dv=res[3], ds=res[4])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_equals_full_sequence(world):
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    with tempfile.TemporaryDirectory() as td:
        mp.spawn(worker, args=(world, port, td), nprocs=world, join=True)
        q, k, v, do, P = data()
        for mode in MODES:
            parts = [np.load(os.path.join(td, f"r{r}_{mode}.npz")) for r in range(world)]
            cat = lambda key: np.concatenate([p[key] for p in parts], axis=1)
            if mode == "global":
                ref, _, dq, dk, dv, ds = O.causal_global(q, k, v, P, K, L, SCALE, dout=do, eps=EPS)
            else:
                ref = O.forward(q, k, v, P, K, L, SCALE, mode != "nc")
                dq, dk, dv, ds = O.backward(q, k, v, P, K, L, SCALE, mode != "nc", do)
            np.testing.assert_allclose(cat("out"), ref, rtol=1e-9, atol=1e-11)
            np.testing.assert_allclose(cat("dq"), dq, rtol=1e-9, atol=1e-11)
            np.testing.assert_allclose(cat("dk"), dk, rtol=1e-9, atol=1e-11)
            np.testing.assert_allclose(cat("dv"), dv, rtol=1e-9, atol=1e-11)
            for p in parts:
                assert abs(float(p["ds"]) - ds) < 1e-9 * max(1.0, abs(ds))
