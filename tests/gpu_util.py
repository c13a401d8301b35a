"""Device-buffer helpers for the GPU tests (through the library's own C ABI)."""
import numpy as np

import hvdrv


class Dev:
    """A device allocation filled from (or sized for) a numpy array."""

    def __init__(self, arr=None, nbytes=None):
        if arr is not None:
            arr = np.ascontiguousarray(arr)
            nbytes = arr.nbytes
        self.nbytes = int(nbytes)
        self.ptr = hvdrv.alloc(self.nbytes)
        if arr is not None:
            hvdrv.upload(self.ptr, arr.ctypes.data, arr.nbytes)
        else:
            hvdrv.memset8(self.ptr, 0, self.nbytes)

    def get(self, dtype, shape=None):
        dtype = np.dtype(dtype)
        n = self.nbytes // dtype.itemsize
        out = np.empty(n, dtype)
        hvdrv.synchronize()
        hvdrv.download(out.ctypes.data, self.ptr, out.nbytes)
        return out if shape is None else out.reshape(shape)

    def put(self, arr):
        arr = np.ascontiguousarray(arr)
        hvdrv.upload(self.ptr, arr.ctypes.data, arr.nbytes)

    def free(self):
        if self.ptr:
            hvdrv.free(self.ptr)
            self.ptr = 0

    def __int__(self):
        return self.ptr

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a


def ulp_diff(a, b):
    """Max distance in float32 ulps (same-sign values)."""
    ia = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    ib = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    return int(np.abs(ia - ib).max()) if ia.size else 0


def quantize_on_device(a):
    """quant_a8s on the GPU: returns device buffers (a8, sa) and host copies."""
    a = np.ascontiguousarray(a, np.float32)
    nb = a.size // 32
    src = Dev(a)
    a8 = Dev(nbytes=a.size)
    sa = Dev(nbytes=nb * 8)
    hvdrv.qa8s(src, a8, sa, nb)
    return a8, sa


def unprepack(pb4, psw, rows, k, pair_ffn=0):
    """The tile-interleaved layout (hv_w4_prepack) back to the reference layout:
    (packed u32 [rows, k/8], scales f32 [rows, k/32])."""
    nb = k // 32
    niter = (nb + 7) // 8
    ntile = (pair_ffn + 3) // 4 if pair_ffn else (rows + 7) // 8
    # nibbles: [tile][iter][half][g][t][jj] = word t of block 8 iter + 4 half + jj of row(g)
    w = np.asarray(pb4, np.uint32).reshape(ntile, niter, 2, 8, 4, 4)
    w = w.transpose(0, 3, 1, 2, 5, 4).reshape(ntile * 8, niter * 8, 4)
    # scales: [tile][iter][g][t][e] = scale of block 8 iter + 2t + e of row(g)
    sc = np.asarray(psw, np.float32).reshape(ntile, niter, 8, 4, 2)
    sc = sc.transpose(0, 2, 1, 3, 4).reshape(ntile * 8, niter * 8)
    if pair_ffn:
        tiles = np.arange(ntile * 8) // 8
        g = np.arange(ntile * 8) % 8
        p = tiles * 4 + (g % 4)
        row = np.where(g < 4, p, pair_ffn + p)
        keep = p < pair_ffn
        packed = np.zeros((rows, nb * 4), np.uint32)
        scale = np.zeros((rows, nb), np.float32)
        packed[row[keep]] = w[keep, :nb].reshape(-1, nb * 4)
        scale[row[keep]] = sc[keep, :nb]
        return packed.reshape(rows, k // 8), scale
    return (np.ascontiguousarray(w[:rows, :nb].reshape(rows, k // 8)),
            np.ascontiguousarray(sc[:rows, :nb]))
