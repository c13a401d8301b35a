"""The 64-bit argmax key of the vocabulary-sharded greedy argmax (hv_argmax_key), restated
on the host: the maximum key over all shards must name np.argmax's token
(engine/reference.py:219: the first maximal id; np compares -0 and +0 equal and returns
the first NaN). The device kernels are checked against np.argmax in
test_gpu_head_argmax.py."""
import numpy as np
import pytest

import hvdrv

F32 = np.float32


def keys_of(v: np.ndarray, base: int = 0) -> np.ndarray:
    """hv_argmax_key's key for every element: high word the f32 bits in unsigned total
    order (-0 -> +0, NaN -> above +inf), low word ~(global id)."""
    v = np.ascontiguousarray(v, F32)
    u = v.view(np.uint32).astype(np.uint64)
    u[np.isnan(v)] = 0x7FC00000
    u[v == 0] = 0
    neg = (u & 0x80000000) != 0
    order = np.where(neg, ~u & 0xFFFFFFFF, u | 0x80000000)
    ids = np.arange(base, base + v.size, dtype=np.uint64)
    return (order << np.uint64(32)) | (~ids & np.uint64(0xFFFFFFFF))


def sharded_token(v: np.ndarray, shards: int) -> int:
    rows = v.size // shards
    best = max(int(keys_of(v[s * rows:(s + 1) * rows], s * rows).max()) for s in range(shards))
    return hvdrv.token_of_key(best)


def cases():
    g = np.random.default_rng(3)
    n = 151936
    out = [g.standard_normal(n).astype(F32) for _ in range(20)]
    v = g.standard_normal(n).astype(F32)
    v[[100000, 37984, 151935]] = 9.0
    out.append(v)
    v = -np.abs(g.standard_normal(n).astype(F32)) - 1
    v[5000], v[3000] = -0.0, 0.0
    out.append(v)
    v = v.copy()
    v[5000], v[3000] = 0.0, -0.0
    out.append(v)
    v = g.standard_normal(n).astype(F32)
    v[[140000, 70000]] = np.nan
    v[10] = np.inf
    out.append(v)
    v = np.full(n, -np.inf, F32)
    v[n - 1] = -3.0e38
    out.append(v)
    out.append(np.round(g.standard_normal(n).astype(F32) * 2) / 2)   # many exact ties
    return out


@pytest.mark.parametrize("shards", [1, 2, 4, 8])
def test_max_key_is_np_argmax(shards):
    for v in cases():
        assert sharded_token(v, shards) == int(np.argmax(v))


def test_keys_are_never_zero_and_decode():
    v = np.array([-np.inf, -3e38, -1.0, -0.0, 0.0, 1e-45, 1.0, np.inf, np.nan], F32)
    k = keys_of(v, base=151930)
    assert (k > 0).all()
    assert [hvdrv.token_of_key(int(x)) for x in k] == list(range(151930, 151939))
    assert hvdrv.token_of_key(0) == -1
    # strictly increasing order of value (the two zeros tie and rank the lower id first)
    assert list(np.argsort(k[[0, 1, 2, 5, 6, 7, 8]])) == list(range(7))
    assert k[3] > k[4]
