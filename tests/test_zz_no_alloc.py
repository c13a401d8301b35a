"""hv_attn_decode_noalloc against hv_attn_decode and the oracle, through the C ABI.

The no-allocation entry point keeps its scratch in a fixed static device array shared by
every call, so the test makes two calls in a row (the second runs over the first one's
leftover scores) and compares each bit for bit with the allocating entry point and with
the oracle's restatement of the reference's attention (computed on the CPU, so a fault
the two entry points share would still show). The file is named to be collected last; it
also passes on its own in a fresh process, where its first call does the per-device
set-up.
"""
import numpy as np
import pytest

import hv_oracle as O
from gpu_util import Dev, bits

F32 = np.float32


def _case(seed, nq, nkv, cap, pos):
    g = np.random.default_rng(seed)
    q = g.standard_normal((nq, 128)).astype(F32)
    kc = g.standard_normal((nkv, cap, 128)).astype(F32)
    vc = g.standard_normal((nkv, cap, 128)).astype(F32)
    return q, kc, vc


@pytest.mark.gpu
def test_noalloc_attention_matches_allocating_entry_two_calls(hv):
    scale = Dev(np.array([1.0 / np.sqrt(128)], F32))
    # Qwen3-8B attention at a 4k context (the reference host's split BLAS runs), then a
    # smaller group-2 case: the second call runs over the first call's leftover scratch.
    cases = [(3, 32, 8, 4352, 4224), (4, 16, 8, 1024, 700)]
    for seed, nq, nkv, cap, pos in cases:
        q, kc, vc = _case(seed, nq, nkv, cap, pos)
        dq, dk, dv, p = Dev(q), Dev(kc), Dev(vc), Dev(np.array([pos], np.int32))
        want = Dev(nbytes=nq * 128 * 4)
        got = Dev(nbytes=nq * 128 * 4)
        hv.attn_decode(dq, dk, dv, want, scale, p, nq, 128, nq // nkv, cap * 128)
        hv.attn_decode_noalloc(dq, dk, dv, got, scale, p, nq, 128, nq // nkv, cap * 128)
        o = got.get(F32, (nq, 128))
        assert np.array_equal(bits(o), bits(want.get(F32, (nq, 128))))
        ref = O.attention(q, kc, vc, pos, nq // nkv, 1.0 / np.sqrt(128))
        assert np.array_equal(bits(o), bits(ref))


@pytest.mark.gpu
def test_noalloc_position_outside_cache_gives_nan(hv):
    # *pos lives on the device, so only the kernels can check it: pos == cap reads no
    # cache row and leaves NaN in every output element
    nq, nkv, cap = 8, 2, 64
    q, kc, vc = _case(5, nq, nkv, cap, 0)
    out = Dev(np.zeros((nq, 128), F32))
    hv.attn_decode_noalloc(Dev(q), Dev(kc), Dev(vc), out, Dev(np.array([1.0], F32)),
                           Dev(np.array([cap], np.int32)), nq, 128, nq // nkv, cap * 128)
    assert np.isnan(out.get(F32)).all()


@pytest.mark.gpu
def test_noalloc_rejects_oversized_problem(hv):
    # 64 heads at a 16k-position cache need 4 MiB of scores: refused on the host before
    # any launch (the pointers are never dereferenced)
    scale = Dev(np.array([1.0], F32))
    pos = Dev(np.array([0], np.int32))
    q = Dev(nbytes=64 * 128 * 4)
    with pytest.raises(hv.CudaError, match="exceed the fixed scratch"):
        hv.attn_decode_noalloc(q, q, q, q, scale, pos, 64, 128, 8, 16384 * 128)
