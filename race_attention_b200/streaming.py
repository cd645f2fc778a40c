"""One RACE attention forward + backward on HOST-resident tensors, with the
host<->device copies overlapped with the kernels.

For callers whose activations live in host memory (offloaded long-context
layers, data too large to keep on the device between steps): the token axis
is cut into chunks that the split entry points of the C ABI treat exactly
like the sequence shards of the multi-GPU path (non-causal: summed bucket
states; causal: exclusive scans of chunk totals added with race_add_offset).
Copies go on two side streams, H2D in the order the phases consume inputs
(k and v, then q, then dO) and D2H as soon as each output chunk is final
(out after the readout, dq after the query backward, dk and dv at the end),
so both PCIe directions run at once and under the compute.

No counterpart exists in the reference (its modules take device tensors);
the result is that of ``race_attention`` forward + ``backward(dout)`` on the
same values.  Host tensors must be pinned (``pin_memory()``) for the copies
to be asynchronous.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from ._lib import check
from .functional import (_SUPPORTED, Buffers, _ptr, _rt, _scale_tensor, make_desc, query)


def _chunks(T: int, n: int):
    step = max(1, -(-T // max(1, n)))
    step = -(-step // 128) * 128          # chunk starts on 128-token boundaries
    return [(t0, min(T, t0 + step)) for t0 in range(0, T, step)]


def fwd_bwd_host(q, k, v, dout, planes, num_bits: int, num_tables: int, scale=1.0,
                 causal: bool = False, eps: float = 1e-6, shared_planes: Optional[bool] = None,
                 chunks: int = 8, device=None, outputs=None, group=None):
    """Forward + backward of RACE attention on host tensors [M, B, T, H, d]
    (4-D [B, T, H, d] taken as M = 1; all four the same shape and dtype,
    float32 or bfloat16, contiguous).

    Returns ``(out, dq, dk, dv, dscale)``: four host tensors of the inputs'
    shape (pinned; pass ``outputs=(out, dq, dk, dv)`` to reuse buffers) and the
    temperature gradient as a device scalar.  All work is enqueued on the
    current CUDA stream of ``device`` and two side streams that it waits for
    before returning, so the host tensors are final once that stream is
    synchronised (``torch.cuda.current_stream().synchronize()``).

    ``group``: a torch.distributed process group over which the token axis is
    sharded (this rank's tensors hold its contiguous range, ranks in order);
    non-causal only here -- the summed bucket states and dE are all-reduced
    across it like in ``race_attention(..., group=...)``, and ``dscale`` is the
    whole sequence's.
    """
    device = torch.device(device if device is not None else "cuda")
    squeeze = q.dim() == 4
    if squeeze:
        q, k, v, dout = (t.unsqueeze(0) for t in (q, k, v, dout))
    if q.dtype not in _SUPPORTED or any(t.dtype != q.dtype for t in (k, v, dout)):
        raise ValueError("q, k, v, dout must share one dtype, float32 or bfloat16")
    if any(t.shape != q.shape or not t.is_contiguous() for t in (k, v, dout)) or \
            not q.is_contiguous():
        raise ValueError("q, k, v, dout must be contiguous and share one [M, B, T, H, d] shape")
    if group is not None and causal:
        raise NotImplementedError("fwd_bwd_host shards only the non-causal form across ranks; "
                                  "use race_attention(..., group=...) for causal")
    if group is not None and q.shape[2] == 0:
        raise ValueError("every rank needs at least one token when sharding across a group")
    if q.is_cuda:
        raise ValueError("fwd_bwd_host takes host tensors; use race_attention for device tensors")
    M, B, T, H, d = q.shape
    dtype = q.dtype
    if planes.dim() == 2:
        planes = planes.unsqueeze(0)
    if shared_planes is None:
        shared_planes = planes.shape[0] == 1
    planes = planes.detach().to(device=device, dtype=torch.float32).contiguous()
    scale_d = _scale_tensor(scale, device).detach().to(torch.float32).reshape(()).contiguous()
    lib = _lib.load()
    if outputs is None:
        outputs = tuple(torch.empty(q.shape, dtype=dtype).pin_memory() for _ in range(4))
    else:
        outputs = tuple(o if o.dim() == 5 else o.unsqueeze(0) for o in outputs)
    h_out, h_dq, h_dk, h_dv = outputs

    comp = torch.cuda.current_stream(device)
    s_in = torch.cuda.Stream(device)
    s_out = torch.cuda.Stream(device)
    s_in.wait_stream(comp)
    s_out.wait_stream(comp)
    with torch.cuda.device(device):
        out_, dq_d, dk_, dv_ = (torch.empty(q.shape, dtype=dtype, device=device)
                                for _ in range(4))
        q_d, k_d, v_d, do_d = (torch.empty(q.shape, dtype=dtype, device=device) for _ in range(4))
    spans = _chunks(T, chunks)
    sl = lambda x, a, b: x[:, :, a:b]
    descs, sizes = [], []
    for a, b in spans:
        desc = make_desc((M, B, b - a, H, d), dtype, num_bits, num_tables, causal, eps, 0,
                         shared_planes)
        descs.append(desc)
        sizes.append(query(desc))
    n = len(spans)
    buf = [Buffers(sz, device) for sz in sizes]
    state = [bf.floats(sz.state_bytes) for bf, sz in zip(buf, sizes)]
    gstate = [bf.floats(sz.gstate_bytes) for bf, sz in zip(buf, sizes)]
    total = [bf.floats(sz.total_bytes) for bf, sz in zip(buf, sizes)]
    ws = max((bf.workspace() for bf in buf), key=lambda w: w.numel()) if n else None
    dscale_q = torch.zeros(max(n, 1), dtype=torch.float32, device=device)
    dscale_kv = torch.zeros(max(n, 1), dtype=torch.float32, device=device)
    st_ptr = comp.cuda_stream

    # ---- H2D, in the order the phases consume the inputs
    ev_kv, ev_q, ev_do = [], [], []
    with torch.cuda.stream(s_in):
        for (a, b) in spans:
            sl(k_d, a, b).copy_(sl(k, a, b), non_blocking=True)
            sl(v_d, a, b).copy_(sl(v, a, b), non_blocking=True)
            ev_kv.append(s_in.record_event())
        for (a, b) in spans:
            sl(q_d, a, b).copy_(sl(q, a, b), non_blocking=True)
            ev_q.append(s_in.record_event())
        for (a, b) in spans:
            sl(do_d, a, b).copy_(sl(dout, a, b), non_blocking=True)
            ev_do.append(s_in.record_event())

    def d2h(dst, src, a, b):
        ev = comp.record_event()
        s_out.wait_event(ev)
        with torch.cuda.stream(s_out):
            sl(dst, a, b).copy_(sl(src, a, b), non_blocking=True)

    P, sc, W, nw = _ptr(planes), _ptr(scale_d), _ptr(ws), (ws.numel() if n else 0)
    # ---- forward: chunk states, then the cross-chunk sum / exclusive scan
    for j, (a, b) in enumerate(spans):
        comp.wait_event(ev_kv[j])
        check(lib.race_forward_reduce(descs[j], _rt(sl(k_d, a, b)), _rt(sl(v_d, a, b)), P, sc,
                                      _ptr(state[j]), _ptr(total[j]), W, nw, st_ptr))
    if not causal:
        for j in range(1, n):
            state[0].add_(state[j])
        if group is not None:
            torch.distributed.all_reduce(state[0], group=group)
    else:
        run = torch.zeros_like(total[0]) if n else None
        for j in range(1, n):
            run.add_(total[j - 1])
            check(lib.race_add_offset(descs[j], _ptr(state[j]), _ptr(run), 0, st_ptr))
    for j, (a, b) in enumerate(spans):
        comp.wait_event(ev_q[j])
        stj = state[0] if not causal else state[j]
        check(lib.race_forward_readout(descs[j], _rt(sl(q_d, a, b)), _rt(sl(k_d, a, b)),
                                       _rt(sl(v_d, a, b)), P, sc, _ptr(stj),
                                       _rt(sl(out_, a, b)), W, nw, st_ptr))
        d2h(h_out, out_, a, b)
    # ---- backward: query side per chunk, then the gradient-state exchange
    for j, (a, b) in enumerate(spans):
        comp.wait_event(ev_do[j])
        stj = state[0] if not causal else state[j]
        check(lib.race_backward_q(descs[j], _rt(sl(q_d, a, b)), _rt(sl(k_d, a, b)),
                                  _rt(sl(v_d, a, b)), P, sc, _ptr(stj), _rt(sl(do_d, a, b)),
                                  _rt(sl(dq_d, a, b)), _ptr(dscale_q[j:j + 1]), _ptr(gstate[j]),
                                  _ptr(total[j]), W, nw, st_ptr))
        d2h(h_dq, dq_d, a, b)
    if not causal:
        for j in range(1, n):
            gstate[0].add_(gstate[j])
        if group is not None:
            torch.distributed.all_reduce(gstate[0], group=group)
    else:
        run = torch.zeros_like(total[0]) if n else None
        for j in range(n - 2, -1, -1):
            run.add_(total[j + 1])
            check(lib.race_add_offset(descs[j], _ptr(gstate[j]), _ptr(run), 1, st_ptr))
    for j, (a, b) in enumerate(spans):
        stj = state[0] if not causal else state[j]
        gsj = gstate[0] if not causal else gstate[j]
        check(lib.race_backward_kv(descs[j], _rt(sl(q_d, a, b)), _rt(sl(k_d, a, b)),
                                   _rt(sl(v_d, a, b)), P, sc, _ptr(stj), _ptr(gsj),
                                   _rt(sl(do_d, a, b)), _rt(sl(dk_, a, b)), _rt(sl(dv_, a, b)),
                                   _ptr(dscale_kv[j:j + 1]), W, nw, st_ptr))
        d2h(h_dk, dk_, a, b)
        d2h(h_dv, dv_, a, b)
    dscale = (dscale_q + dscale_kv).sum()
    if group is not None:
        torch.distributed.all_reduce(dscale, group=group)
    comp.wait_stream(s_out)
    comp.wait_stream(s_in)
    res = [h_out, h_dq, h_dk, h_dv]
    if squeeze:
        res = [r.squeeze(0) for r in res]
    return (*res, dscale)
