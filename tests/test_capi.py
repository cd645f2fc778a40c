"""CPU checks of the C-ABI library: it loads, exports every declared entry
point, and validates descriptors (no GPU compute is called here)."""
import ctypes
import os
import re

import pytest

from race_attention_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "race_b200.h")


def declared_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:int|size_t|const char\*)\s+(race_[a-z_]+)\(", txt, re.M)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        from race_attention_b200.build import build
        build()
    return _lib.load()


def test_exports_every_declared_symbol(lib):
    syms = declared_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.SYMBOLS)


def test_version_and_errors(lib):
    assert b"sm_100a" in lib.race_version()
    for rc in range(7):
        assert lib.race_strerror(rc)


def desc(**kw):
    d = dict(dtype=0, causal=0, head_dim=64, num_bits=2, num_tables=5, ensembles=1, batch=1,
             heads=4, tokens=4096, chunk=0, shared_planes=0, eps=1e-6)
    d.update(kw)
    return _lib.RaceDesc(**d)


def test_query_sizes(lib):
    sz = _lib.RaceSizes()
    assert lib.race_query(desc(), sz) == 0
    S, D, N = 20, 64, 4
    assert sz.slot_floats == (S * D + S + 3) // 4 * 4
    assert sz.state_bytes == N * sz.slot_floats * 4
    assert sz.workspace_bytes > 0
    assert lib.race_query(desc(causal=1, tokens=1000, chunk=128, normalize=1), sz) == 0
    assert lib.race_query(desc(causal=1, tokens=1000, chunk=128), sz) == 0
    # causal (per-bucket): one prefix slot per token range of whole 128-token
    # tiles, then the fp32 projections of q and k ([N][T][16] each); behind the
    # gradient slots alpha [N][T][S rounded to 4] and the float64 key mass at
    # every tile start [N][tiles][SP]
    assert 1 <= sz.num_chunks <= 8
    slots = N * sz.num_chunks * sz.slot_floats
    up = lambda x: (x + 63) // 64 * 64
    assert sz.state_bytes == (up(slots) + 2 * N * 1000 * 16) * 4
    tiles = (1000 + 127) // 128
    alpha_off = up(slots)
    mass_off = up(alpha_off + N * 1000 * 20)
    assert sz.gstate_bytes == (mass_off + 2 * N * tiles * 32 + 2) * 4


@pytest.mark.parametrize("bad,code", [
    (dict(head_dim=48), 2), (dict(num_bits=5, num_tables=3), 2),
    (dict(num_bits=3, num_tables=5, causal=1), 2), (dict(num_tables=0), 1),
    (dict(dtype=7), 1), (dict(tokens=-1), 1), (dict(num_bits=6, num_tables=1), 2),
    (dict(batch=70000), 2), (dict(normalize=1), 2), (dict(causal=1, normalize=3), 1),
])
def test_query_rejects(lib, bad, code):
    sz = _lib.RaceSizes()
    assert lib.race_query(desc(**bad), sz) == code


def test_null_args(lib):
    assert lib.race_query(None, _lib.RaceSizes()) == 1
    t = _lib.RaceTensor(None, 0, 0, 0, 0)
    rc = lib.race_forward(desc(), t, t, t, None, None, t, None, None, 0, None)
    assert rc in (1, 4)
