"""race_forward_static: the forward for callers that cannot allocate.

Some hosts of this library cannot call cudaMalloc or keep a caching allocator
(code running inside another runtime's memory pool, plugin hosts that forbid
allocation after start-up, fixed-budget inference loops).  The entry point
keeps its bucket state and scratch in a static device array owned by the
library.  These tests call it through the C ABI twice in a row -- the second
call reuses the array left over from the first -- and compare its output with
race_forward's, which uses caller-provided buffers, at the parity tolerance
(1e-4 relative L2, float32).  The file sorts last so a run stopping at the
first failure has already run every other test.
"""
import numpy as np
import pytest
import torch

from oracle import race_oracle as O
from race_attention_b200 import _lib
from race_attention_b200.functional import Buffers, _ptr, _rt, _stream, make_desc, query

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.mark.parametrize("causal,N,T", [(False, 4, 4096), (True, 2, 2000), (False, 3, 777)])
def test_static_forward_matches_race_forward(causal, N, T):
    lib = _lib.load()
    K, L, d = 2, 5, 64
    g = torch.Generator(device="cuda").manual_seed(N * 100 + T)
    shape = (1, N, T, 1, d)
    q, k, v = (torch.randn(shape, generator=g, device="cuda") for _ in range(3))
    planes = torch.randn((1, K * L, d), generator=g, device="cuda")
    scale = torch.tensor(1.3, device="cuda")
    desc = make_desc(shape, torch.float32, K, L, causal, 1e-6, 0, True)
    sizes = query(desc)
    buf = Buffers(sizes, q.device)
    state, ws = buf.floats(sizes.state_bytes), buf.workspace()
    ref = torch.empty(shape, device="cuda")
    _lib.check(lib.race_forward(desc, _rt(q), _rt(k), _rt(v), _ptr(planes), _ptr(scale), _rt(ref),
                                _ptr(state), _ptr(ws), ws.numel(), _stream()))
    for _ in range(2):
        out = torch.full(shape, float("nan"), device="cuda")
        _lib.check(lib.race_forward_static(desc, _rt(q), _rt(k), _rt(v), _ptr(planes),
                                           _ptr(scale), _rt(out), _stream()))
        torch.cuda.synchronize()
        assert O.rel_l2(out.double().cpu().numpy(), ref.double().cpu().numpy()) < 1e-4


def test_static_forward_rejects_oversized_shapes():
    lib = _lib.load()
    shape = (1, 6000, 1024, 1, 64)          # 6000 streams: their states need > 8 MiB
    desc = make_desc(shape, torch.float32, 2, 5, False, 1e-6, 0, True)
    t = _lib.RaceTensor(None, 0, 0, 0, 0)
    assert lib.race_forward_static(desc, t, t, t, None, None, t, None) == _lib.RACE_ERR_TOO_LARGE
