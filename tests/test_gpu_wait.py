"""Failure detection without a GPU fault: the bounded wait that every cross-CTA and
cross-rank wait of the fused step uses, run on a device word that nothing sets. The wait
gives up after its limit with HV_E_TIMEOUT in the status word, ends at once when another
failure is already reported there, and leaves the context usable."""
import time

import numpy as np
import pytest

from gpu_util import Dev

pytestmark = pytest.mark.gpu
HV_E_TIMEOUT = 1004


def test_bounded_wait_times_out_and_the_context_stays_usable(hv):
    word = Dev(np.zeros(1, np.uint32))
    status = Dev(np.zeros(1, np.int32))
    t0 = time.perf_counter()
    hv.wait_probe(word, 1, 1, 200_000_000, status)          # 0.2 s on a word nothing sets
    hv.synchronize()
    dt = time.perf_counter() - t0
    assert status.get(np.int32)[0] == HV_E_TIMEOUT
    assert 0.15 < dt < 5.0, dt
    # a word already set: no wait, the status is left alone
    status.put(np.zeros(1, np.int32))
    word.put(np.ones(1, np.uint32))
    hv.wait_probe(word, 1, 1, 200_000_000, status)
    assert status.get(np.int32)[0] == 0
    # a failure already reported ends a long wait early and is not overwritten
    status.put(np.array([7], np.int32))
    word.put(np.zeros(1, np.uint32))
    t0 = time.perf_counter()
    hv.wait_probe(word, 1, 1, 5_000_000_000, status)
    hv.synchronize()
    assert time.perf_counter() - t0 < 2.0
    assert status.get(np.int32)[0] == 7
    # the context still runs kernels
    a = Dev(np.arange(64, dtype=np.float32))
    out = Dev(nbytes=256)
    hv.vadd(a, a, out, 64)
    assert np.array_equal(out.get(np.float32), 2 * np.arange(64, dtype=np.float32))


def test_wait_probe_rejects_unbounded_limits(hv):
    word, status = Dev(np.zeros(1, np.uint32)), Dev(np.zeros(1, np.int32))
    for limit in (0, -1, 20_000_000_000):
        with pytest.raises(hv.CudaError):
            hv.wait_probe(word, 1, 1, limit, status)
