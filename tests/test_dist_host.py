"""The multi-rank host path on CPU: two ranks (spawned processes) over bench.Dist's TCP
plumbing, as bench.py --gpus 2 runs them (barrier, max over ranks, sum, the all-gather of
bytes that carries the sharded engine's one swap of CUDA IPC handles), and the
cross-rank half of the vocabulary-sharded greedy argmax: each rank folds its shard of
the logits into a 64-bit key, the keys are all-gathered, and every rank picks the same
token, np.argmax's over the whole vocabulary. A rank that dies before a collective makes
the other rank's collective fail instead of hanging."""
import multiprocessing as mp
import os
import socket
import sys

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TESTS = os.path.dirname(os.path.abspath(__file__))
V = 151936


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _paths():
    for p in (os.path.join(REPO, "hive-limited_b200"), os.path.join(REPO, "oracle"), REPO,
              TESTS):
        if p not in sys.path:
            sys.path.insert(0, p)


def _env(rank, world, port):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), HV_BENCH_PORT=str(port))


def _rank_main(rank, world, port, result):
    try:
        _paths()
        _env(rank, world, port)
        import bench
        import hvdrv
        assert "torch" not in sys.modules          # the bench's plumbing is stdlib only
        from test_argmax_key import keys_of
        d = bench.Dist(timeout_s=60)
        out = {}
        d.barrier()
        out["max"] = d.max(rank + 0.5)
        out["sum"] = d.sum(1.0)
        out["gather"] = d.allgather_bytes(f"handles of rank {rank}".encode())
        # the sharded argmax: the same seeded logits on every rank, rank r holds a slice
        for seed in range(6):
            v = np.random.default_rng(seed).standard_normal(V).astype(np.float32)
            if seed == 1:
                v[[7, V // world + 7]] = 10.0          # equal maxima on different ranks
            if seed == 2:
                v[V - 1] = np.nan
            rows = V // world
            key = int(keys_of(v[rank * rows:(rank + 1) * rows], rank * rows).max())
            keys = [int.from_bytes(b, "little")
                    for b in d.allgather_bytes(key.to_bytes(8, "little"))]
            out[f"tok{seed}"] = (hvdrv.token_of_key(max(keys)), int(np.argmax(v)))
        d.barrier()
        d.close()
        result.put((rank, out))
    except BaseException as e:                      # reported to the parent
        result.put((rank, repr(e)))


def _dies_early(rank, world, port, result):
    try:
        _paths()
        _env(rank, world, port)
        import bench
        d = bench.Dist(timeout_s=20)
        if rank == 1:
            result.put((rank, "left"))
            result.close()
            result.join_thread()                    # the message is out of the process
            os._exit(0)                             # gone without a word
        import time
        t0 = time.monotonic()
        try:
            d.barrier()
            d.allgather_bytes(b"x")
            result.put((rank, "no error"))
        except Exception as e:                      # the expected outcome
            result.put((rank, f"error after {time.monotonic() - t0:.0f} s: "
                              f"{type(e).__name__}"))
    except BaseException as e:
        result.put((rank, f"setup: {e!r}"))


def _spawn(target, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, result)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        return dict(result.get(timeout=timeout) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()


def test_two_ranks_plumbing_and_sharded_argmax():
    out = _spawn(_rank_main)
    for rank in (0, 1):
        o = out[rank]
        assert isinstance(o, dict), o
        assert o["max"] == 1.5 and o["sum"] == 2.0
        assert o["gather"] == [b"handles of rank 0", b"handles of rank 1"]
        for seed in range(6):
            got, want = o[f"tok{seed}"]
            assert got == want, (rank, seed, got, want)
    assert out[0]["tok1"][0] == 7                   # the tie goes to the lower id


def test_a_rank_that_leaves_makes_the_collective_fail_not_hang():
    out = _spawn(_dies_early, timeout=90)
    assert out[1] == "left"
    assert out[0].startswith("error"), out[0]
