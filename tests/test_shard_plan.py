"""Column-parallel shard plan (host logic, no GPU): every projection's rows are split
into whole, disjoint, ordered ranges that cover the full matrix."""
import pytest

import limited
import synth
from w4format import Config


@pytest.mark.parametrize("arch", ["qwen3-1.7b", "qwen3-8b", "qwen3-32b"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_cover_every_row_once(arch, world):
    cfg = Config(synth.ARCH[arch])
    plans = [limited.shard_plan(cfg, world, r) for r in range(world)]
    full = {"q": cfg.n_head * cfg.head_dim, "kv": cfg.n_kv * cfg.head_dim,
            "hid": cfg.hidden, "ffn": cfg.ffn, "vocab": cfg.vocab}
    for key, n in full.items():
        ranges = [p[key] for p in plans]
        assert ranges[0][0] == 0 and ranges[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        assert len({r1 - r0 for r0, r1 in ranges}) == 1          # equal shards
    for p in plans:
        assert p["n_head"] * world == cfg.n_head and p["n_kv"] * world == cfg.n_kv
        assert p["ffn_n"] % 32 == 0 and (p["hid"][1] - p["hid"][0]) % 8 == 0
        # q heads of a rank use exactly its kv heads (grouped-query attention stays local)
        assert p["n_head"] // p["n_kv"] == cfg.n_head // cfg.n_kv


def test_indivisible_shapes_are_refused():
    cfg = Config(synth.tiny_arch(n_head=4, n_kv=2))
    with pytest.raises(ValueError):
        limited.shard_plan(cfg, 4, 0)                 # 2 kv heads over 4 ranks
    with pytest.raises(ValueError):
        limited.shard_plan(cfg, 2, 2)                 # rank outside the world
    with pytest.raises(ValueError):
        limited.shard_plan(cfg, 16, 0)                # more ranks than the step supports


def test_sharded_engine_arguments_are_checked_before_any_device_work():
    cfg = Config(synth.tiny_arch())
    with pytest.raises(ValueError):       # the sharded step exists only in the fused form
        limited.Engine(config=cfg, tensors={}, world=2, rank=0, fused=False,
                       exchange=lambda b: [b, b])
    with pytest.raises(ValueError):       # the IPC handle swap needs a transport
        limited.Engine(config=cfg, tensors={}, world=2, rank=1)


def test_prefill_mode_is_checked_before_any_device_work():
    cfg = Config(synth.tiny_arch())
    with pytest.raises(ValueError, match="prefill"):
        limited.Engine(config=cfg, tensors={}, prefill="bulk")
    with pytest.raises(ValueError, match="one GPU"):
        limited.Engine(config=cfg, tensors={}, world=2, rank=0, exchange=lambda b: [b, b],
                       prefill="batched")
