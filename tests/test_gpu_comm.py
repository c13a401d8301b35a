"""hv_comm_* / hv_allgather through the C ABI on a B200: the all-gather gives every rank
every rank's slice, rank after rank, exactly the bytes a host all-gather gives (one GPU
always; two GPUs of one process when the box has them)."""
import numpy as np
import pytest

from gpu_util import Dev

pytestmark = pytest.mark.gpu


def test_allgather_one_device(hv):
    comm = hv.Comm(devs=[0])
    try:
        assert comm.size() == (1, 1)
        x = np.random.default_rng(1).integers(0, 256, 4096, dtype=np.uint8)
        send, recv = Dev(x), Dev(nbytes=x.nbytes)
        comm.allgather([send], [recv], x.nbytes)
        assert np.array_equal(recv.get(np.uint8), x)
    finally:
        comm.destroy()


def test_allgather_two_devices_matches_host_gather(hv):
    if hv.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    g = np.random.default_rng(2)
    parts = [g.standard_normal(3000).astype(np.float32) for _ in range(2)]
    want = np.concatenate(parts)
    bufs = []
    for d in range(2):
        hv.set_current(d)
        bufs.append((Dev(parts[d]), Dev(nbytes=want.nbytes)))
    hv.set_current(0)
    comm = hv.Comm(devs=[0, 1])
    try:
        comm.allgather([b[0] for b in bufs], [b[1] for b in bufs], parts[0].nbytes)
        for d in range(2):
            hv.set_current(d)
            hv.synchronize()
            got = bufs[d][1].get(np.float32)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), d
    finally:
        hv.set_current(0)
        comm.destroy()
