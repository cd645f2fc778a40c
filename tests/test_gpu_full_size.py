"""CUDA path vs the oracle at the benchmark's full sequence length (needs a B200).

One stream of 2**20 tokens, d = 64, K = 2, L = 5 -- the bench's per-GPU
workload.  The non-causal oracle runs densely; the causal one streams the
prefix states in chunks (``O.causal_streamed``), so both finish in tens of
seconds on the host.  Tolerances are the path's: 1e-4 relative L2 for
float32, 2e-2 for bfloat16.  Float32 prefix sums over a million tokens are
where a single-precision scan would drift; the library carries them in
float64, which these cases check.
"""
import math

import numpy as np
import pytest
import torch

from oracle import race_oracle as O
from tests.cuda_util import bf16_round, run_streams

pytestmark = pytest.mark.gpu

T, D, K, L = 1 << 20, 64, 2, 5


@pytest.fixture(autouse=True, scope="module")
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from race_attention_b200 import _lib
    _lib.load()


def _inputs(seed, bf16):
    rng = np.random.default_rng(seed)
    q, k, v, dout = (rng.standard_normal((1, T, D), dtype=np.float32) for _ in range(4))
    planes = rng.standard_normal((1, K * L, D), dtype=np.float32)
    if bf16:
        q, k, v, dout = (bf16_round(a) for a in (q, k, v, dout))
    return q, k, v, dout, planes


@pytest.mark.parametrize("causal", [False, True], ids=["noncausal", "causal"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_full_length(causal, dtype):
    bf16 = dtype == torch.bfloat16
    q, k, v, dout, planes = _inputs(11 + causal, bf16)
    scale = 8.0 if causal else 1.3        # sqrt(d) (misc/race.py:67); a learnt temperature
    got = run_streams(q, k, v, planes, K, L, scale, causal, dout, dtype=dtype)
    if causal:
        ref, ds_mag = O.dscale_magnitude(O.causal_streamed, q, k, v, planes, K, L, scale, dout)
    else:
        bwd, ds_mag = O.dscale_magnitude(O.backward, q, k, v, planes, K, L, scale, False, dout)
        ref = (O.forward(q, k, v, planes, K, L, scale, False),) + bwd
    tol = 2e-2 if bf16 else 1e-4
    for name, a, b in zip(("out", "dq", "dk", "dv"), got[:4], ref[:4]):
        err = O.rel_l2(a, b)
        assert err < tol, (name, err)
    # The temperature gradient is a sum of 2^20 signed terms that cancel to a
    # few parts in 10^5 of their magnitudes.  fp32: the path's bar relative to
    # itself.  bf16 (one-part bf16 operands): the bar on the root-sum-square
    # scale of the terms, sum|term| / sqrt(T) -- the size of independent
    # per-token rounding errors -- since relative to the cancelled total it
    # would ask for more than bf16 operands carry.
    abs_tol = 0.0 if not bf16 else tol * ds_mag / math.sqrt(T)
    assert math.isclose(got[4], ref[4], rel_tol=tol, abs_tol=abs_tol), (got[4], ref[4], ds_mag)
