"""Autograd entry point of RACE attention on B200.

``race_attention`` takes q, k, v in the reference's [M, B, T, H, d] layout
(``BatchedACE.forward`` inputs, misc/vit.py:918 and misc/race.py:63) -- any
strided view whose head dimension is contiguous, including the stride-0
ensemble expansion the reference's ``RACEAttention`` builds -- and returns the
[M, B, T, H, d] output.  Gradients flow to q, k, v and to the temperature
divisor ``scale``; the hyperplanes are a buffer (misc/vit.py:906-908) and get
none.  The bucket probabilities are recomputed in the backward pass, never
stored.

The role of the reference's ``RACEPrefixMeanFlatFn`` (misc/race.py:9-24:
save the inputs and eps, call the kernel forward / backward) is played by
``_RaceFunction`` here, one level higher so the hash is fused in.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib
from ._lib import RaceDesc, RaceSizes, RaceTensor, check

_SUPPORTED = (torch.float32, torch.bfloat16)


def _aligned(x: torch.Tensor) -> bool:
    """Rows must start on 16-byte boundaries (vector loads and bulk copies)."""
    if x.stride(-1) != 1 or x.data_ptr() % 16 != 0:
        return False
    q = 16 // x.element_size()
    return all(s % q == 0 for s in x.stride()[:-1])


def _prep(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    if x.dtype != dtype:
        x = x.to(dtype)
    if not _aligned(x):
        x = x.contiguous()
        if not _aligned(x):
            raise ValueError("RACE attention needs 16-byte aligned rows (head_dim * element size % 16 == 0)")
    return x


def _rt(x: Optional[torch.Tensor]) -> RaceTensor:
    """[M,B,T,H,d] view -> race_tensor_t (strides in (m, b, h, t) order)."""
    if x is None:
        return RaceTensor(None, 0, 0, 0, 0)
    s = x.stride()
    return RaceTensor(x.data_ptr(), s[0], s[1], s[3], s[2])


def _ptr(x: Optional[torch.Tensor]):
    return None if x is None else x.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _mappable(*xs) -> bool:
    """True when the copy engine can walk every tensor (no broadcast batch or
    head axis): the library is then told to fail rather than fall back."""
    for x in xs:
        if x is None:
            continue
        M, B, T, H, _ = x.shape
        s = x.stride()
        if (s[1] == 0 and B > 1) or (s[2] == 0 and T > 1) or (s[3] == 0 and H > 1) or min(s) < 0:
            return False
    return True


class DeviceStatus:
    """Stream-ordered check of the library's device status word.

    After a forward or backward the word is copied into pinned host memory
    on the launching stream and an event is recorded; completed copies are
    inspected at the next call (no forced synchronisation), and
    ``check(wait=True)`` waits for all of them.  A nonzero word means a kernel
    gave up on a bounded wait and that call's outputs are partial."""

    def __init__(self):
        self.pending = []

    def push(self, lib, ws: torch.Tensor) -> None:
        host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        check(lib.race_device_status(ws.data_ptr(), ws.numel(), host.data_ptr(), _stream()))
        ev = torch.cuda.Event()
        ev.record()
        self.pending.append((host, ev))
        self.check(wait=False)

    def check(self, wait: bool = True) -> None:
        while self.pending:
            host, ev = self.pending[0]
            if not wait and not ev.query():
                return
            ev.synchronize()
            self.pending.pop(0)
            word = int(host.item())
            if word:
                self.pending.clear()
                raise _lib.RaceError(
                    f"race_b200 device status 0x{word:x}: a kernel gave up on a bounded wait "
                    "(timeout); the outputs of that call are incomplete")


device_status = DeviceStatus()


def check_device_status() -> None:
    """Waits for the outstanding status reads and raises RaceError if any
    forward or backward since the last check ended a kernel early."""
    device_status.check(wait=True)


_NORMS = {"bucket": _lib.RACE_NORM_BUCKET, "global": _lib.RACE_NORM_GLOBAL}


def make_desc(shape, dtype, K, L, causal, eps, chunk, shared_planes, normalize=0,
              flags=0) -> RaceDesc:
    M, B, T, H, d = shape
    return RaceDesc(flags=int(flags),
        dtype=_lib.RACE_F32 if dtype == torch.float32 else _lib.RACE_BF16,
        causal=int(bool(causal)), head_dim=d, num_bits=K, num_tables=L, ensembles=M,
        batch=B, heads=H, tokens=T, chunk=int(chunk), shared_planes=int(bool(shared_planes)),
        eps=float(eps), normalize=int(normalize))


def query(desc: RaceDesc) -> RaceSizes:
    lib = _lib.load()
    sz = RaceSizes()
    check(lib.race_query(desc, sz))
    return sz


class Buffers:
    """Device buffers one call needs, sized by race_query()."""

    def __init__(self, sizes: RaceSizes, device):
        self.sizes = sizes
        self.device = device

    def floats(self, nbytes: int) -> torch.Tensor:
        return torch.empty(max(1, nbytes // 4), dtype=torch.float32, device=self.device)

    def workspace(self) -> torch.Tensor:
        return torch.empty(max(16, self.sizes.workspace_bytes), dtype=torch.uint8,
                           device=self.device)


def _scale_tensor(scale, device) -> torch.Tensor:
    if isinstance(scale, torch.Tensor):
        return scale
    return torch.tensor(float(scale), dtype=torch.float32, device=device)


class _RaceFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, planes, scale, K, L, causal, eps, chunk, shared_planes, group,
                normalize, head_major_out, normalize_qk):
        ctx.set_materialize_grads(False)
        if not q.is_cuda:
            raise RuntimeError("race_attention runs on CUDA devices only (no CPU fallback)")
        ctx.in_dtypes = (q.dtype, k.dtype, v.dtype)
        dtype = q.dtype if q.dtype in _SUPPORTED else torch.float32
        q, k, v = (_prep(t, dtype) for t in (q, k, v))
        if causal and not _mappable(q, k, v):
            # the causal kernels stream every input through the copy engine,
            # which cannot walk a broadcast axis: materialise it
            q, k, v = (t if _mappable(t) else t.contiguous() for t in (q, k, v))
        planes = planes.detach().to(torch.float32).contiguous()
        scale_d = scale.detach().to(torch.float32).reshape(()).contiguous()
        flags = _lib.RACE_FLAG_STRICT_TMA if _mappable(q, k, v) else 0
        if normalize_qk:
            flags |= _lib.RACE_FLAG_NORMALIZE_QK
        desc = make_desc(tuple(q.shape), dtype, K, L, causal, eps, chunk, shared_planes, normalize,
                         flags)
        sizes = query(desc)
        buf = Buffers(sizes, q.device)
        lib = _lib.load()
        M, B, T, H, dh = q.shape
        if head_major_out:   # [M, B, H, T, d] memory seen as [M, B, T, H, d]
            out = torch.empty((M, B, H, T, dh), dtype=dtype, device=q.device).permute(0, 1, 3, 2, 4)
        else:
            out = torch.empty(q.shape, dtype=dtype, device=q.device)
        # the per-token denominator of the global mode, [M, B, H, T] float32
        den = (torch.empty((M, B, H, T), dtype=torch.float32, device=q.device) if normalize
               else torch.empty(0, dtype=torch.float32, device=q.device))
        state = buf.floats(sizes.state_bytes)
        ws = buf.workspace()
        if group is None:
            check(lib.race_forward_ex(desc, _rt(q), _rt(k), _rt(v), _ptr(planes), _ptr(scale_d),
                                      _rt(out), _ptr(den) if normalize else None, _ptr(state),
                                      _ptr(ws), ws.numel(), _stream()))
            device_status.push(lib, ws)
        else:
            from .sequence_parallel import sharded_forward
            sharded_forward(lib, desc, sizes, buf, q, k, v, planes, scale_d, out, state, ws, group,
                            den if normalize else None)
        ctx.save_for_backward(q, k, v, planes, scale_d, state)
        ctx.desc = desc
        ctx.group = group
        ctx.scale_shape = scale.shape
        if not normalize:
            ctx.mark_non_differentiable(den)
        return out, den

    @staticmethod
    def backward(ctx, dout, dden):
        q, k, v, planes, scale_d, state = ctx.saved_tensors
        desc = ctx.desc
        dtype = q.dtype
        if dout is None:
            dout = torch.zeros(q.shape, dtype=dtype, device=q.device)
        dout = _prep(dout, dtype)
        if not _mappable(dout):
            dout = dout.contiguous()
        if dden is not None and desc.normalize:
            dden = dden.to(torch.float32).contiguous()
        else:
            dden = None
        sizes = query(desc)
        buf = Buffers(sizes, q.device)
        lib = _lib.load()
        shape = tuple(q.shape)
        dq = torch.empty(shape, dtype=dtype, device=q.device)
        dk = torch.empty(shape, dtype=dtype, device=q.device)
        dv = torch.empty(shape, dtype=dtype, device=q.device)
        dscale = torch.empty((), dtype=torch.float32, device=q.device)
        gstate = buf.floats(sizes.gstate_bytes)
        ws = buf.workspace()
        if ctx.group is None:
            check(lib.race_backward_ex(desc, _rt(q), _rt(k), _rt(v), _ptr(planes), _ptr(scale_d),
                                       _ptr(state), _rt(dout), _ptr(dden), _rt(dq), _rt(dk),
                                       _rt(dv), _ptr(dscale), _ptr(gstate), _ptr(ws), ws.numel(),
                                       _stream()))
            device_status.push(lib, ws)
        else:
            from .sequence_parallel import sharded_backward
            sharded_backward(lib, desc, sizes, buf, q, k, v, planes, scale_d, state, dout,
                             dq, dk, dv, dscale, gstate, ws, ctx.group, dden)
        dq, dk, dv = (g.to(t) for g, t in zip((dq, dk, dv), ctx.in_dtypes))
        return (dq, dk, dv, None, dscale.reshape(ctx.scale_shape), None, None, None, None, None,
                None, None, None, None, None)


def race_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, planes: torch.Tensor,
                   num_bits: int, num_tables: int, scale=1.0, causal: bool = False,
                   eps: float = 1e-6, chunk: int = 0, shared_planes: Optional[bool] = None,
                   group=None, normalize: str = "bucket", return_den: bool = False,
                   head_major_out: bool = False, normalize_qk: bool = False):
    """RACE attention forward (autograd-aware) on [M, B, T, H, d] inputs.

    Args:
      q, k, v: [M, B, T, H, d] (4-D [B, T, H, d] is taken as M = 1), float32
        or bfloat16 (other float types compute in float32).
      planes: hyperplanes [Mp, L*K, d] (Mp = 1 shared, or M), float32.
      num_bits: K hyperplanes per table; num_tables: L tables.
      scale: temperature divisor -- a tensor (learnable: gets a gradient) or a
        float.  The reference uses exp(logit_temp).clamp(1e-2, 20) for the
        non-causal module (misc/vit.py:923) and sqrt(d) for the causal one
        (misc/race.py:67).
      causal: per-bucket prefix mean (misc/race.py:108-138) instead of the
        full-sequence bucket mean (misc/vit.py:967-975).
      eps: added to the bucket mass.
      chunk: accepted for the reference's signature and ignored (the causal
        kernels work on 128-token tiles; results do not depend on a chunk).
      group: torch.distributed process group across which the token axis is
        sharded (contiguous ranges in rank order), or None.
      normalize: causal only.  "bucket" (default): every bucket normalised by
        its own prefix mass (misc/race.py).  "global": one denominator per
        token summed over all L*2^K buckets, out = num / max(den, eps) (the
        ELSAA chunked form, misc/elsaa_causal_complete.py:520-571 and
        misc/race_kernel.py); ``eps`` is then the clamp floor of den.
      return_den: global mode only: also return den, the unclamped per-token
        denominator [M, B, H, T] float32 (differentiable; 4-D inputs give
        [B, H, T]).
      normalize_qk: hash q / |q| and k / |k| instead of q and k (the values and
        the output are unchanged; gradients flow through the normalisation).
        Off by default: the reference's RACE path never normalises, and tanh
        is not scale-invariant, so turning it on changes the model.
      head_major_out: lay the output out in memory as [M, B, H, T, d] (the
        returned tensor is still indexed [M, B, T, H, d]), so that the
        reference modules' head merge ``permute(0, 2, 1, 3).reshape(B, T,
        H*d)`` is a view rather than a copy.
    """
    squeeze = False
    if q.dim() == 4:
        q, k, v = q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0)
        squeeze = True
    if q.dim() != 5 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k, v must share one [M, B, T, H, d] shape")
    M = q.shape[0]
    if planes.dim() == 2:
        planes = planes.unsqueeze(0)
    if shared_planes is None:
        shared_planes = planes.shape[0] == 1
    LK = num_bits * num_tables
    if planes.shape[-2:] != (LK, q.shape[-1]):
        raise ValueError(f"planes must be [Mp, {LK}, {q.shape[-1]}], got {tuple(planes.shape)}")
    if not shared_planes and planes.shape[0] != M:
        raise ValueError("per-ensemble planes need one set per ensemble")
    if normalize not in _NORMS:
        raise ValueError(f"normalize must be 'bucket' or 'global', got {normalize!r}")
    norm = _NORMS[normalize]
    if norm and not causal:
        raise ValueError("normalize='global' is defined for the causal form only")
    if return_den and not norm:
        raise ValueError("return_den needs normalize='global'")
    scale_t = _scale_tensor(scale, q.device)
    out, den = _RaceFunction.apply(q, k, v, planes, scale_t, int(num_bits), int(num_tables),
                                   bool(causal), float(eps), int(chunk), bool(shared_planes),
                                   group, norm, bool(head_major_out), bool(normalize_qk))
    if squeeze:
        out, den = out.squeeze(0), (den.squeeze(0) if norm else den)
    return (out, den) if return_den else out


def fused_qkv(x: torch.Tensor, q_lin, k_lin, v_lin, heads: int, head_dim: int):
    """q, k, v projections of x [B, T, d_in] as ONE GEMM over the three Linear
    layers' concatenated weights (the reference runs three, misc/vit.py:1012-1014,
    misc/race.py:160-162), returned as [B, T, H, d_k] strided views of the
    [B, T, 3, H, d_k] result: the kernels read them in place (token stride
    3 H d_k), so no copy or permute follows.  Gradients flow back to the three
    layers' weights and biases through the concatenation."""
    B, T, _ = x.shape
    w = torch.cat([q_lin.weight, k_lin.weight, v_lin.weight], dim=0)
    if q_lin.bias is not None:
        b = torch.cat([q_lin.bias, k_lin.bias, v_lin.bias], dim=0)
        y = torch.nn.functional.linear(x, w, b)
    else:
        y = torch.nn.functional.linear(x, w)
    y = y.view(B, T, 3, heads, head_dim)
    return y[:, :, 0], y[:, :, 1], y[:, :, 2]


def default_causal_scale(head_dim: int) -> float:
    """Fixed divisor of the causal module (misc/race.py:67)."""
    return math.sqrt(head_dim)


class _ProbsFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, planes, scale, K, L, shared_planes):
        if not x.is_cuda:
            raise RuntimeError("bucket_probs runs on CUDA devices only (no CPU fallback)")
        ctx.in_dtype = x.dtype
        dtype = x.dtype if x.dtype in _SUPPORTED else torch.float32
        x = _prep(x, dtype)
        planes = planes.detach().to(torch.float32).contiguous()
        scale_d = scale.detach().to(torch.float32).reshape(()).contiguous()
        M, B, T, H, d = x.shape
        desc = make_desc(tuple(x.shape), dtype, K, L, False, 0.0, 0, shared_planes)
        S = L << K
        probs = torch.empty((M, B, H, T, L, 1 << K), dtype=torch.float32, device=x.device)
        check(_lib.load().race_probs(desc, _rt(x), _ptr(planes), _ptr(scale_d), _ptr(probs),
                                     _stream()))
        ctx.save_for_backward(x, planes, scale_d)
        ctx.desc = desc
        ctx.scale_shape = scale.shape
        assert probs.numel() == M * B * H * T * S
        return probs

    @staticmethod
    def backward(ctx, dprobs):
        x, planes, scale_d = ctx.saved_tensors
        lib = _lib.load()
        dprobs = dprobs.to(torch.float32).contiguous()
        dx = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        dscale = torch.empty((), dtype=torch.float32, device=x.device)
        ws = torch.empty(max(16, lib.race_probs_workspace(ctx.desc)), dtype=torch.uint8,
                         device=x.device)
        check(lib.race_probs_backward(ctx.desc, _rt(x), _ptr(planes), _ptr(scale_d),
                                      _ptr(dprobs), _rt(dx), _ptr(dscale), 0, _ptr(ws),
                                      ws.numel(), _stream()))
        return dx.to(ctx.in_dtype), None, dscale.reshape(ctx.scale_shape), None, None, None


def bucket_probs(x: torch.Tensor, planes: torch.Tensor, num_bits: int, num_tables: int,
                 scale=1.0, shared_planes: Optional[bool] = None) -> torch.Tensor:
    """Soft-hash bucket probabilities of x [M, B, T, H, d] (4-D [B, T, H, d]
    is taken as M = 1): [M, B, H, T, L, 2^K] float32, the tensor the
    reference's race_bucket_probs_from_qk returns (misc/arxiv_64K.py:1580-1642).
    Differentiable in x and in ``scale`` (a tensor or a float)."""
    if x.dim() == 4:
        x = x.unsqueeze(0)
    if planes.dim() == 2:
        planes = planes.unsqueeze(0)
    if shared_planes is None:
        shared_planes = planes.shape[0] == 1
    scale_t = _scale_tensor(scale, x.device)
    return _ProbsFunction.apply(x, planes, scale_t, num_bits, num_tables, bool(shared_planes))
