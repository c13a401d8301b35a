"""hv_attn_decode_noalloc against hv_attn_decode, through the C ABI.

The no-allocation entry point keeps its scratch in a fixed static device array shared by
every call, so the test makes two calls in a row (the second sees the first one's
leftover partials and tickets) and compares each with the allocating entry point at the
attention tests' tolerance. The file is named to be collected last; it also passes on
its own in a fresh process, where its first call does the per-device set-up.
"""
import numpy as np
import pytest

from gpu_util import Dev

F32 = np.float32
RTOL, ATOL = 1e-4, 2e-6          # the attention tests' tolerance (test_gpu_ops.py)


def _case(seed, nq, nkv, cap, pos):
    g = np.random.default_rng(seed)
    q = g.standard_normal((nq, 128)).astype(F32)
    kc = g.standard_normal((nkv, cap, 128)).astype(F32)
    vc = g.standard_normal((nkv, cap, 128)).astype(F32)
    return Dev(q), Dev(kc), Dev(vc), Dev(np.array([pos], np.int32))


@pytest.mark.gpu
def test_noalloc_attention_matches_allocating_entry_two_calls(hv):
    scale = Dev(np.array([1.0 / np.sqrt(128)], F32))
    # Qwen3-8B attention at a 4k context, then a smaller group-2 case: the second call
    # runs over the first call's leftover scratch.
    cases = [(3, 32, 8, 4352, 4224), (4, 16, 8, 1024, 700)]
    for seed, nq, nkv, cap, pos in cases:
        q, kc, vc, p = _case(seed, nq, nkv, cap, pos)
        want = Dev(nbytes=nq * 128 * 4)
        got = Dev(nbytes=nq * 128 * 4)
        hv.attn_decode(q, kc, vc, want, scale, p, nq, 128, nq // nkv, cap * 128)
        hv.attn_decode_noalloc(q, kc, vc, got, scale, p, nq, 128, nq // nkv, cap * 128)
        w, o = want.get(F32, (nq, 128)), got.get(F32, (nq, 128))
        assert np.isfinite(o).all()
        np.testing.assert_allclose(o, w, rtol=RTOL, atol=ATOL)


@pytest.mark.gpu
def test_noalloc_rejects_oversized_problem(hv):
    # 8 kv heads x group 8 at a 1M-position cache needs ~35 MB of partials: refused on
    # the host before any launch (the pointers are never dereferenced).
    scale = Dev(np.array([1.0], F32))
    pos = Dev(np.array([0], np.int32))
    q = Dev(nbytes=64 * 128 * 4)
    with pytest.raises(hv.CudaError, match="exceed the fixed scratch"):
        hv.attn_decode_noalloc(q, q, q, q, scale, pos, 64, 128, 8, (1 << 20) * 128)
    with pytest.raises(hv.CudaError, match="kv heads exceed"):
        hv.attn_decode_noalloc(q, q, q, q, scale, pos, 65, 128, 1, 128 * 128)
