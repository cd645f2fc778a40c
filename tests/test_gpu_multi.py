"""Sequence sharding over NCCL on 2 GPUs (skipped with fewer than 2).

Each rank runs the library on its contiguous token range through the public
``race_attention(..., group=pg)`` call (and, non-causal, the host-buffer
``streaming.fwd_bwd_host(..., group=pg)``); the exchange between the split entry
points is one NCCL collective per direction.  The concatenated shards must
match the float64 oracle on the whole sequence (1e-4 relative L2), and the
temperature gradient must agree on every rank.
"""
import math
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import race_oracle as O

pytestmark = pytest.mark.gpu

N, T, D, K, L = 2, 20000, 64, 2, 5


def _data():
    rng = np.random.default_rng(21)
    q, k, v, dout = (rng.standard_normal((N, T, D), dtype=np.float32) for _ in range(4))
    planes = rng.standard_normal((1, K * L, D), dtype=np.float32)
    return q, k, v, dout, planes


def _log(rank, *a):
    import sys
    print(f"[rank {rank}]", *a, file=sys.stderr, flush=True)


def _worker(rank, world, port, outdir):
    import datetime

    import torch.distributed as dist
    from race_attention_b200 import race_attention
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=120))
    _log(rank, "process group up")
    try:
        q, k, v, dout, planes = _data()
        lo, hi = T * rank // world, T * (rank + 1) // world
        dev = torch.device("cuda", rank)
        for causal in (False, True):
            scale = 8.0 if causal else 1.3
            t = lambda a: torch.tensor(a[:, lo:hi], device=dev).unsqueeze(0).unsqueeze(3)
            qt, kt, vt = (t(a).requires_grad_(True) for a in (q, k, v))
            sc = torch.tensor(scale, device=dev, requires_grad=True)
            out = race_attention(qt, kt, vt, torch.tensor(planes, device=dev), K, L, sc,
                                 causal=causal, group=dist.group.WORLD)
            out.backward(t(dout))
            f = lambda x: x.detach().squeeze(3).squeeze(0).double().cpu().numpy()
            np.savez(os.path.join(outdir, f"r{rank}_c{int(causal)}.npz"), out=f(out),
                     dq=f(qt.grad), dk=f(kt.grad), dv=f(vt.grad), ds=float(sc.grad))
            _log(rank, "race_attention done, causal =", causal)
        # the host-buffer pipeline, sharded the same way (non-causal)
        from race_attention_b200.streaming import fwd_bwd_host
        h = lambda a: torch.tensor(a[:, lo:hi]).unsqueeze(0).unsqueeze(3).contiguous().pin_memory()
        out, dq, dk, dv, ds = fwd_bwd_host(h(q), h(k), h(v), h(dout), torch.tensor(planes), K, L,
                                           1.3, device=dev, chunks=3, group=dist.group.WORLD)
        torch.cuda.current_stream(dev).synchronize()
        g = lambda x: x.squeeze(3).squeeze(0).double().numpy()
        np.savez(os.path.join(outdir, f"r{rank}_host.npz"), out=g(out), dq=g(dq), dk=g(dk),
                 dv=g(dv), ds=float(ds))
        torch.cuda.synchronize()
        _log(rank, "host pipeline done")
    except BaseException:
        import traceback
        _log(rank, traceback.format_exc())
        raise
    finally:
        dist.destroy_process_group()


def test_two_gpu_sharded_matches_oracle():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    q, k, v, dout, planes = _data()
    with tempfile.TemporaryDirectory() as td:
        mp.spawn(_worker, args=(2, port, td), nprocs=2, join=True)
        for causal, tag in ((False, "c0"), (True, "c1"), (False, "host")):
            scale = 8.0 if causal else 1.3
            parts = [np.load(os.path.join(td, f"r{r}_{tag}.npz")) for r in range(2)]
            cat = lambda key: np.concatenate([p[key] for p in parts], axis=1)
            P = np.broadcast_to(planes, (N,) + planes.shape[1:])
            if causal:
                ref = O.causal_streamed(q, k, v, P, K, L, scale, dout)
            else:
                ref = (O.forward(q, k, v, P, K, L, scale, False),) + \
                    O.backward(q, k, v, P, K, L, scale, False, dout)
            for name, b in zip(("out", "dq", "dk", "dv"), ref[:4]):
                err = O.rel_l2(cat(name), b)
                assert err < 1e-4, (causal, name, err)
            for p in parts:
                assert math.isclose(float(p["ds"]), ref[4], rel_tol=1e-3), (float(p["ds"]), ref[4])


def _worker_capi(rank, world, port, outdir):
    """The library's own hook: race_set_comm with an NCCL communicator made by
    race_comm_init, then plain race_forward / race_backward calls through the
    C ABI on this rank's shard; the library runs the exchange itself."""
    import ctypes
    import torch.distributed as dist
    from race_attention_b200 import _lib
    from race_attention_b200.functional import Buffers, _ptr, _rt, _stream, make_desc, query
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    lib = _lib.load()
    comm = ctypes.c_void_p()
    try:
        dev = torch.device("cuda", rank)
        uid = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            host = torch.zeros(128, dtype=torch.uint8)
            _lib.check(lib.race_comm_unique_id(_ptr(host)))
            uid.copy_(host)
        dist.broadcast(uid, 0)
        uid_h = uid.cpu().contiguous()
        _lib.check(lib.race_comm_init(ctypes.byref(comm), world, _ptr(uid_h), rank))
        _lib.check(lib.race_set_comm(comm))
        q, k, v, dout, planes = _data()
        lo, hi = T * rank // world, T * (rank + 1) // world
        Pd = torch.tensor(planes, device=dev)
        for causal in (False, True):
            scale = torch.tensor(8.0 if causal else 1.3, device=dev)
            t = lambda a: torch.tensor(a[:, lo:hi], device=dev).unsqueeze(0).unsqueeze(3).contiguous()
            qt, kt, vt, dot = (t(a) for a in (q, k, v, dout))
            shape = tuple(qt.shape)
            desc = make_desc(shape, torch.float32, K, L, causal, 1e-6, 0, True, 0,
                             _lib.RACE_FLAG_STRICT_TMA)
            sizes = query(desc)
            buf = Buffers(sizes, dev)
            state, gstate, ws = (buf.floats(sizes.state_bytes), buf.floats(sizes.gstate_bytes),
                                 buf.workspace())
            out, dq, dk, dv = (torch.empty(shape, device=dev) for _ in range(4))
            ds = torch.zeros((), device=dev)
            _lib.check(lib.race_forward(desc, _rt(qt), _rt(kt), _rt(vt), _ptr(Pd), _ptr(scale),
                                        _rt(out), _ptr(state), _ptr(ws), ws.numel(), _stream()))
            _lib.check(lib.race_backward(desc, _rt(qt), _rt(kt), _rt(vt), _ptr(Pd), _ptr(scale),
                                         _ptr(state), _rt(dot), _rt(dq), _rt(dk), _rt(dv),
                                         _ptr(ds), _ptr(gstate), _ptr(ws), ws.numel(),
                                         _stream()))
            dist.all_reduce(ds)   # rank-local through the C ABI: sum as a parameter gradient
            torch.cuda.synchronize()
            f = lambda x: x.detach().squeeze(3).squeeze(0).double().cpu().numpy()
            np.savez(os.path.join(outdir, f"r{rank}_capi{int(causal)}.npz"), out=f(out),
                     dq=f(dq), dk=f(dk), dv=f(dv), ds=float(ds))
    finally:
        lib.race_set_comm(None)
        if comm.value:
            lib.race_comm_destroy(comm)
        dist.destroy_process_group()


def test_two_gpu_library_hook_matches_oracle():
    """race_set_comm: the sharded exchange run by the library itself (C ABI)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    q, k, v, dout, planes = _data()
    with tempfile.TemporaryDirectory() as td:
        mp.spawn(_worker_capi, args=(2, port, td), nprocs=2, join=True)
        for causal in (False, True):
            scale = 8.0 if causal else 1.3
            parts = [np.load(os.path.join(td, f"r{r}_capi{int(causal)}.npz")) for r in range(2)]
            cat = lambda key: np.concatenate([p[key] for p in parts], axis=1)
            P = np.broadcast_to(planes, (N,) + planes.shape[1:])
            if causal:
                ref = O.causal_streamed(q, k, v, P, K, L, scale, dout)
            else:
                ref = (O.forward(q, k, v, P, K, L, scale, False),) + \
                    O.backward(q, k, v, P, K, L, scale, False, dout)
            for name, b in zip(("out", "dq", "dk", "dv"), ref[:4]):
                err = O.rel_l2(cat(name), b)
                assert err < 1e-4, (causal, name, err)
            for p in parts:
                assert math.isclose(float(p["ds"]), ref[4], rel_tol=1e-3), (float(p["ds"]), ref[4])
