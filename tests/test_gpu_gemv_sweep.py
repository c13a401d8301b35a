"""The isolated W4A8 GEMV sweep (N x K): 2048x2048, 6144x2048, 2048x6144, 12288x4096,
4096x12288, 151936x4096; weights N(0,0.02) from seed 1, activations N(0,1).

Bit-exact against the reference: the device quantiser reproduces the reference's packed
weights and scales (sha256), quant_a8s its int8 activations, scales and block sums, the
GEMV its int32 block dots (sampled rows) and its full fp32 output vector (sha256)."""
import hashlib

import numpy as np
import pytest

import synth
from gpu_util import Dev, bits, quantize_on_device

pytestmark = pytest.mark.gpu
F32 = np.float32


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("j", range(len(synth.GEMV_SHAPES)))
def test_sweep_shape_bit_exact(hv, golden, j):
    g = golden("gemv_sweep.npz")
    n, k = synth.GEMV_SHAPES[j]
    assert g[f"s{j}_shape"].tolist() == [n, k]
    w, a = synth.gemv_case(j, n, k)
    b4, sw = Dev(nbytes=n * k // 2), Dev(nbytes=n * k // 32 * 4)
    wd = Dev(w)
    hv.quantize_w4(wd, b4, sw, n, k)
    wd.free()
    del w
    assert sha(b4.get(np.uint32)) == str(g[f"s{j}_packed_sha"])
    assert sha(sw.get(F32)) == str(g[f"s{j}_scale_sha"])
    a8, sa = quantize_on_device(a)
    nb = k // 32
    s = sa.get(F32)
    assert np.array_equal(a8.get(np.int8), g[f"s{j}_qa"].reshape(-1))
    assert np.array_equal(bits(s[:nb]), bits(g[f"s{j}_sa"]))
    assert np.array_equal(s[nb:].view(np.int32), g[f"s{j}_bsum"])
    y, idot = Dev(nbytes=n * 4), Dev(nbytes=n * nb * 4)
    hv.a4gv_idot(a8, sa, b4, sw, y, idot, k // 8, n)
    yv = y.get(F32)
    assert np.array_equal(bits(yv[:2048]), bits(g[f"s{j}_y_head"]))
    assert sha(yv) == str(g[f"s{j}_y_sha"])
    rows = g[f"s{j}_rows"]
    assert np.array_equal(idot.get(np.int32, (n, nb))[rows], g[f"s{j}_idot"])
    y2 = Dev(nbytes=n * 4)
    hv.a4gv(a8, sa, b4, sw, y2, k // 8, n)
    assert sha(y2.get(F32)) == str(g[f"s{j}_y_sha"])
    # the engine's tile-interleaved layout gives the same bits
    nib, scb = hv.w4_prepacked_size(n, k, 0)
    pb4, psw = Dev(nbytes=nib), Dev(nbytes=scb)
    hv.w4_prepack(b4, sw, n, k, 0, pb4, psw)
    y3 = Dev(nbytes=n * 4)
    hv.a4gv_pp(a8, sa, pb4, psw, y3, k // 8, n, 0)
    assert sha(y3.get(F32)) == str(g[f"s{j}_y_sha"])
