"""Engine construction that fails part way (here: the third weight prepack raises) frees
every device buffer it had allocated, since the caller never gets an engine to free().
Run on the CPU against a fake driver that records allocations."""
import types

import pytest

import limited
import synth


class Boom(RuntimeError):
    pass


class FakeDriver(types.ModuleType):
    def __init__(self, fail_at):
        super().__init__("hvdrv")
        self.live, self.next, self.prepacks, self.fail_at = set(), 1 << 20, 0, fail_at

    def alloc(self, n):
        self.next += (int(n) + 255) // 256 * 256
        self.live.add(self.next)
        return self.next

    def free(self, p):
        self.live.remove(p)                  # a double free would raise here

    def compute_capability(self, dev):
        return 10, 0

    def w4_prepacked_size(self, n, k, pair=0):
        return n * k // 2, n * k // 32 * 4

    def w4_prepack(self, *a):
        self.prepacks += 1
        if self.prepacks == self.fail_at:
            raise Boom("prepack failed")

    def __getattr__(self, name):        # every other call: accepted, no effect
        if name.startswith("__"):
            raise AttributeError(name)
        return lambda *a, **k: 0


@pytest.mark.parametrize("fail_at", [1, 3, 10**9])
def test_failed_construction_frees_everything(monkeypatch, fail_at):
    drv = FakeDriver(fail_at)
    monkeypatch.setattr(limited, "hvdrv", drv)
    cfg = synth.tiny_arch()
    if fail_at < 10**9:
        with pytest.raises(Boom):
            limited.Engine(config=cfg, tensors=synth.iter_tensors(limited.Config(cfg), 7),
                           quiet=True, max_context=32)
        assert not drv.live, f"{len(drv.live)} buffers left allocated"
    else:                                    # a construction that succeeds, then free()
        eng = limited.Engine(config=cfg, tensors=synth.iter_tensors(limited.Config(cfg), 7),
                             quiet=True, max_context=32)
        assert drv.live
        eng.free()
        assert not drv.live
