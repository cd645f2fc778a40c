"""Sequence sharding of RACE attention across ranks (one process per GPU).

Every rank holds a contiguous token range of every stream, in rank order.
The only data exchanged are the bucket states, S x (d+1) floats per stream:

  non-causal  forward: all-reduce (sum) of the [V | 1] bucket sums
              backward: all-reduce of dE = sum_t pQ(t) dO(t)
  causal      forward: exclusive scan across ranks of the rank totals
              (all-gather of the totals, then the sum over LOWER ranks is
              added to every chunk prefix of this rank)
              backward: the reverse exclusive scan of the gradient totals
              (sum over HIGHER ranks)

The temperature gradient is summed over the group, so every rank holds the
gradient of the whole sequence.  Collectives run through torch.distributed
(NCCL over NVLink on B200; gloo on CPU for tests) on the current stream.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from ._lib import check


def _ordered_sum(parts, like):
    out = torch.zeros_like(like)
    for p in parts:
        out += p
    return out


def exchange_forward_state(state: torch.Tensor, total: Optional[torch.Tensor], causal: bool,
                           group, add_offset: Callable[[torch.Tensor], None]) -> None:
    """Makes the rank-local forward state global (see module docstring)."""
    if not causal:
        dist.all_reduce(state, op=dist.ReduceOp.SUM, group=group)
        return
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    gathered = [torch.empty_like(total) for _ in range(world)]
    dist.all_gather(gathered, total, group=group)
    if rank > 0:
        add_offset(_ordered_sum(gathered[:rank], total))


def exchange_backward_state(gstate: torch.Tensor, total: Optional[torch.Tensor], causal: bool,
                            group, add_offset: Callable[[torch.Tensor], None]) -> None:
    """Makes the rank-local gradient state global (see module docstring)."""
    if not causal:
        dist.all_reduce(gstate, op=dist.ReduceOp.SUM, group=group)
        return
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    gathered = [torch.empty_like(total) for _ in range(world)]
    dist.all_gather(gathered, total, group=group)
    if rank < world - 1:
        add_offset(_ordered_sum(gathered[rank + 1:], total))


def sharded_forward(lib, desc, sizes, buf, q, k, v, planes, scale, out, state, ws, group,
                    den=None):
    from .functional import _ptr, _rt, _stream
    total = buf.floats(sizes.total_bytes) if desc.causal else None
    check(lib.race_forward_reduce(desc, _rt(k), _rt(v), _ptr(planes), _ptr(scale), _ptr(state),
                                  _ptr(total), _ptr(ws), ws.numel(), _stream()))
    add = lambda off: check(lib.race_add_offset(desc, _ptr(state), _ptr(off), 0, _stream()))
    exchange_forward_state(state, total, bool(desc.causal), group, add)
    check(lib.race_forward_readout_ex(desc, _rt(q), _rt(k), _rt(v), _ptr(planes), _ptr(scale),
                                      _ptr(state), _rt(out), _ptr(den), _ptr(ws), ws.numel(),
                                      _stream()))


def sharded_backward(lib, desc, sizes, buf, q, k, v, planes, scale, state, dout, dq, dk, dv,
                     dscale, gstate, ws, group, dden=None):
    from .functional import _ptr, _rt, _stream
    total = buf.floats(sizes.total_bytes) if desc.causal else None
    check(lib.race_backward_q_ex(desc, _rt(q), _rt(k), _rt(v), _ptr(planes), _ptr(scale),
                                 _ptr(state), _rt(dout), _ptr(dden), _rt(dq), _ptr(dscale),
                                 _ptr(gstate), _ptr(total), _ptr(ws), ws.numel(), _stream()))
    slots = gstate if not desc.causal else gstate[: (sizes.num_chunks * sizes.slot_floats
                                                     * desc.ensembles * desc.batch * desc.heads)]
    add = lambda off: check(lib.race_add_offset(desc, _ptr(gstate), _ptr(off), 1, _stream()))
    exchange_backward_state(slots, total, bool(desc.causal), group, add)
    check(lib.race_backward_kv(desc, _rt(q), _rt(k), _rt(v), _ptr(planes), _ptr(scale),
                               _ptr(state), _ptr(gstate), _rt(dout), _rt(dk), _rt(dv),
                               _ptr(dscale), _ptr(ws), ws.numel(), _stream()))
    dist.all_reduce(dscale, op=dist.ReduceOp.SUM, group=group)
