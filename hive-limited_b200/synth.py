"""Seeded synthetic Qwen3-shaped models and GEMV inputs.

There is no network here for checkpoints, so every workload is random-init with the
geometry of a real Qwen3 size. The draw is fixed down to the RNG stream so that the GPU
engine, the oracle and the golden-vector script all see the same numbers:

* tensor i of a model (in the order of `tensor_plan`) is drawn from
  ``np.random.default_rng(np.random.SeedSequence(seed, spawn_key=(i,)))``; a tensor of
  more than BIG_DRAW elements (the 8B and 32B embeddings and LM heads) is drawn as
  BIG_BLOCKS row blocks, block b from spawn key (i, b), in parallel -- a single stream
  of 600M+ values would take ~20 s on one core;
* projection matrices and the embedding: ``standard_normal(float32) * 0.02``;
* RMSNorm gains: ``1 + standard_normal(float32) * 0.01``;
* a tied model's embedding is stored as float16 (the reference gathers from an f16
  copy and quantises its LM head from that same f16 copy, engine/reference.py:138,158).

Every tensor has its own stream, so tensors can be drawn on several threads at once and
the result does not depend on the thread count.
"""
from __future__ import annotations

import concurrent.futures as cf
import os

import numpy as np

from w4format import Config

F32 = np.float32

ARCH = {
    # hidden 2048, ffn 6144, 28 layers, 16 q heads / 8 kv heads of 128, tied embeddings
    "qwen3-1.7b": dict(num_hidden_layers=28, hidden_size=2048, intermediate_size=6144,
                       num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                       vocab_size=151936, rope_theta=1000000.0, rms_norm_eps=1e-6,
                       tie_word_embeddings=True, eos_token_id=None),
    # hidden 4096, ffn 12288, 36 layers, 32 q heads / 8 kv heads, untied LM head
    "qwen3-8b": dict(num_hidden_layers=36, hidden_size=4096, intermediate_size=12288,
                     num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                     vocab_size=151936, rope_theta=1000000.0, rms_norm_eps=1e-6,
                     tie_word_embeddings=False, eos_token_id=None),
    # hidden 5120, ffn 25600, 64 layers, 64 q heads / 8 kv heads, untied LM head
    "qwen3-32b": dict(num_hidden_layers=64, hidden_size=5120, intermediate_size=25600,
                      num_attention_heads=64, num_key_value_heads=8, head_dim=128,
                      vocab_size=151936, rope_theta=1000000.0, rms_norm_eps=1e-6,
                      tie_word_embeddings=False, eos_token_id=None),
    # the 8B layer shapes with 2 layers: a small case of the same kernels for profiler
    # captures (every launch holds well under the device's memory)
    # the 32B layer shapes (64 q heads over 8 kv heads, ffn 25600) with 2 layers: the
    # fused step's group-8 path at full width, for parity runs of seconds
    "qwen3-32b-2l": dict(num_hidden_layers=2, hidden_size=5120, intermediate_size=25600,
                         num_attention_heads=64, num_key_value_heads=8, head_dim=128,
                         vocab_size=151936, rope_theta=1000000.0, rms_norm_eps=1e-6,
                         tie_word_embeddings=False, eos_token_id=None),
    "qwen3-8b-2l": dict(num_hidden_layers=2, hidden_size=4096, intermediate_size=12288,
                        num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                        vocab_size=151936, rope_theta=1000000.0, rms_norm_eps=1e-6,
                        tie_word_embeddings=False, eos_token_id=None),
}

# Named workloads: architecture, weight seed, prompt length, tokens generated.
WORKLOADS = {
    "qwen3-1.7b-p32-g64": ("qwen3-1.7b", 0, 32, 64),
    "qwen3-8b-p4096-g256": ("qwen3-8b", 2, 4096, 256),
    "qwen3-32b-p2048-g256": ("qwen3-32b", 3, 2048, 256),
    "qwen3-8b-2l-p4096-g16": ("qwen3-8b-2l", 2, 4096, 16),
}

# The isolated GEMV sweep (N x K), weights from seed 1.
GEMV_SHAPES = [(2048, 2048), (6144, 2048), (2048, 6144),
               (12288, 4096), (4096, 12288), (151936, 4096)]
GEMV_SEED = 1
HEAD_SEED = 4            # LM head + argmax workload: 151936 x 5120
HEAD_SHAPE = (151936, 5120)


def tiny_arch(n_layer=2, hidden=256, ffn=512, n_head=4, n_kv=2, vocab=1000,
              tied=False) -> dict:
    """A small Qwen3-shaped geometry for quick parity runs."""
    return dict(num_hidden_layers=n_layer, hidden_size=hidden, intermediate_size=ffn,
                num_attention_heads=n_head, num_key_value_heads=n_kv, head_dim=128,
                vocab_size=vocab, rope_theta=1000000.0, rms_norm_eps=1e-6,
                tie_word_embeddings=tied, eos_token_id=None)


def tensor_plan(cfg: Config) -> list[tuple[str, tuple, str]]:
    """(HF name, shape, kind) in draw order: embedding, then per layer q,k,v,o,gate,up,
    down and its four norms, then the final norm and (untied) the LM head."""
    c = cfg
    qd = c.head_dim
    plan = [("model.embed_tokens.weight", (c.vocab, c.hidden), "w")]
    for l in range(c.n_layer):
        p = f"model.layers.{l}."
        plan += [
            (p + "self_attn.q_proj.weight", (c.n_head * qd, c.hidden), "w"),
            (p + "self_attn.k_proj.weight", (c.n_kv * qd, c.hidden), "w"),
            (p + "self_attn.v_proj.weight", (c.n_kv * qd, c.hidden), "w"),
            (p + "self_attn.o_proj.weight", (c.hidden, c.n_head * qd), "w"),
            (p + "mlp.gate_proj.weight", (c.ffn, c.hidden), "w"),
            (p + "mlp.up_proj.weight", (c.ffn, c.hidden), "w"),
            (p + "mlp.down_proj.weight", (c.hidden, c.ffn), "w"),
            (p + "input_layernorm.weight", (c.hidden,), "norm"),
            (p + "post_attention_layernorm.weight", (c.hidden,), "norm"),
            (p + "self_attn.q_norm.weight", (qd,), "norm"),
            (p + "self_attn.k_norm.weight", (qd,), "norm"),
        ]
    plan.append(("model.norm.weight", (c.hidden,), "norm"))
    if not c.tied:
        plan.append(("lm_head.weight", (c.vocab, c.hidden), "w"))
    return plan


def rng_for(seed: int, *key: int) -> np.random.Generator:
    return np.random.default_rng(np.random.SeedSequence(seed, spawn_key=tuple(key)))


BIG_DRAW = 1 << 29      # elements above which a tensor is drawn in row blocks
BIG_BLOCKS = 16


def draw(seed: int, index: int, shape, kind: str) -> np.ndarray:
    if int(np.prod(shape)) > BIG_DRAW:
        x = np.empty(shape, F32)
        edges = [shape[0] * b // BIG_BLOCKS for b in range(BIG_BLOCKS + 1)]

        def fill(b):
            part = x[edges[b]:edges[b + 1]]
            rng_for(seed, index, b).standard_normal(part.shape, dtype=F32, out=part)

        with cf.ThreadPoolExecutor(min(BIG_BLOCKS, os.cpu_count() or 1)) as ex:
            list(ex.map(fill, range(BIG_BLOCKS)))
    else:
        x = rng_for(seed, index).standard_normal(shape, dtype=F32)
    if kind == "w":
        x *= F32(0.02)
    else:
        x *= F32(0.01)
        x += F32(1.0)
    return x


def iter_tensors(cfg: Config, seed: int, threads: int | None = None, names=None):
    """Yield (name, array) in plan order, drawing a few tensors ahead on a thread pool.

    The tied embedding is yielded as float16. `names`, if given, restricts the draw.
    """
    plan = [(i, n, s, k) for i, (n, s, k) in enumerate(tensor_plan(cfg))
            if names is None or n in names]
    threads = threads or min(16, os.cpu_count() or 1)

    def make(item):
        i, n, s, k = item
        x = draw(seed, i, s, k)
        if n == "model.embed_tokens.weight" and cfg.tied:
            x = x.astype(np.float16)
        return n, x

    with cf.ThreadPoolExecutor(threads) as ex:
        futs = []
        it = iter(plan)
        for item in it:
            futs.append(ex.submit(make, item))
            if len(futs) >= threads + 1:
                break
        for item in it:
            yield futs.pop(0).result()
            futs.append(ex.submit(make, item))
        for f in futs:
            yield f.result()


def model_tensors(cfg: Config, seed: int) -> dict[str, np.ndarray]:
    """The whole synthetic model as a name -> array dict (small models only)."""
    return dict(iter_tensors(cfg, seed))


def prompt_ids(cfg: Config, seed: int, n: int) -> list[int]:
    """Uniform random prompt ids in [0, vocab), drawn from the workload seed."""
    g = rng_for(seed, 1_000_000)
    return [int(t) for t in g.integers(0, cfg.vocab, size=n)]


def gemv_case(index: int, n: int, k: int, seed: int = GEMV_SEED):
    """Weights N(0,0.02) [n, k] and an activation N(0,1) [k] for one sweep shape."""
    w = rng_for(seed, index, 0).standard_normal((n, k), dtype=F32) * F32(0.02)
    a = rng_for(seed, index, 1).standard_normal(k, dtype=F32)
    return w, a


def head_case(n_states: int, seed: int = HEAD_SEED, shape=HEAD_SHAPE, threads: int | None = None):
    """LM-head workload: weights [151936, 5120] N(0,0.02) and `n_states` N(0,1) hidden
    states (stream (seed, 1)). The weight rows are drawn in 8 row blocks, block b from
    stream (seed, 0, b), on a thread pool; the draw does not depend on the thread count."""
    n, k = shape
    w = np.empty(shape, F32)
    nblk = 8
    edges = [n * b // nblk for b in range(nblk + 1)]

    def fill(b):
        part = w[edges[b]:edges[b + 1]]
        rng_for(seed, 0, b).standard_normal(part.shape, dtype=F32, out=part)
        part *= F32(0.02)

    with cf.ThreadPoolExecutor(threads or min(nblk, os.cpu_count() or 1)) as ex:
        list(ex.map(fill, range(nblk)))
    h = rng_for(seed, 1).standard_normal((n_states, k), dtype=F32)
    return w, h
