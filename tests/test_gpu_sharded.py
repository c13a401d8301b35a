"""The column-sharded fused step on 2 GPUs (one process per GPU, CUDA IPC peer buffers)
against the same model on one GPU: identical greedy tokens and, rank by rank, logits
shards bit-identical to the slices of the one-GPU logits. Needs 2 GPUs (skipped
otherwise). Workers are spawned (no fork after CUDA use) and joined with a timeout; every
device-side wait of the sharded step is bounded, so a failure surfaces as an error."""
import multiprocessing as mp
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ARCH = dict(n_layer=2, hidden=512, ffn=1024, n_head=8, n_kv=2, vocab=4096)
SEED, PROMPT, NEW, CAP = 11, [3, 1, 4, 1, 5, 9, 2, 6], 6, 64


def _paths():
    for p in (os.path.join(REPO, "hive-limited_b200"), REPO):
        if p not in sys.path:
            sys.path.insert(0, p)


def _run(world, rank, inbox, outbox, result, kw):
    """One rank: build the (sharded) engine, decode, report tokens and the logits shard
    of the prompt's last position."""
    try:
        _paths()
        import hvdrv
        import limited
        import synth
        from w4format import Config

        def exchange(blob):
            outbox.put((rank, blob))
            return inbox.get(timeout=120)

        hvdrv.init()
        cfg = Config(synth.tiny_arch(**ARCH))
        eng = limited.Engine(config=cfg, tensors=synth.iter_tensors(cfg, SEED), quiet=True,
                             max_context=CAP, device=rank, world=world, rank=rank,
                             exchange=exchange if world > 1 else None, **kw)
        toks, _, _ = eng.generate(PROMPT, NEW, stop_on_eos=False)
        lg = eng.logits(PROMPT)
        result.put((rank, toks, lg.tobytes()))
        eng.free()
    except BaseException as e:            # reported to the parent, never swallowed
        result.put((rank, "error", repr(e)))


def _launch(world, kw=None):
    ctx = mp.get_context("spawn")
    inboxes = [ctx.Queue() for _ in range(world)]
    outbox, result = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_run, args=(world, r, inboxes[r], outbox, result, kw or {}))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        if world > 1:                     # relay the one all-gather of IPC handles
            blobs = dict(outbox.get(timeout=300) for _ in range(world))
            for q in inboxes:
                q.put([blobs[r] for r in range(world)])
        out = {}
        for _ in range(world):
            rank, toks, lg = result.get(timeout=300)
            assert toks != "error", lg
            out[rank] = (toks, np.frombuffer(lg, np.float32))
        return out
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()


@pytest.mark.gpu
def test_two_gpu_sharded_step_matches_one_gpu(hv):
    if hv.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    one = _launch(1)[0]
    two = _launch(2)
    assert two[0][0] == one[0] and two[1][0] == one[0], (two[0][0], two[1][0], one[0])
    full = one[1]
    n = full.size // 2
    assert np.array_equal(two[0][1].view(np.uint32), full[:n].view(np.uint32))
    assert np.array_equal(two[1][1].view(np.uint32), full[n:].view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("kw", [{"kv_dtype": "f16"}, {"gemv_layout": "dq"},
                                {"kv_dtype": "f16", "gemv_layout": "dq"}])
def test_two_gpu_sharded_variants_match_one_gpu(hv, kw):
    """The binary16 cache and the dq weight tiles sharded over 2 GPUs: the same tokens
    and logits shards, bit for bit, as the same variant on one GPU."""
    if hv.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    one = _launch(1, kw)[0]
    two = _launch(2, kw)
    assert two[0][0] == one[0] and two[1][0] == one[0], (two[0][0], two[1][0], one[0])
    full = one[1]
    n = full.size // 2
    assert np.array_equal(two[0][1].view(np.uint32), full[:n].view(np.uint32))
    assert np.array_equal(two[1][1].view(np.uint32), full[n:].view(np.uint32))
