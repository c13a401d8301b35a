"""The calls the reference's demo server makes on the engine and on the driver module
(serve.py:176, 223-246, 419-437, 846-866), checked against this package's signatures
without a GPU: a server written for the reference runs on this engine by changing its
import path only.

Engine: Engine(model_dir, kernels_dir=...), verify_graph(ids, n=24), _graph_ok,
device_name, bind_thread(), stream(ids, max_new=..., stop_evt=...) yielding
("prefill", seconds) then ("tok", id, seconds), bits_per_weight(), weight_bytes(),
cfg.max_context, free(). Driver: mem_info(), device(0), device_name(dev),
compute_capability(dev), device_attribute(dev, 16 | 36 | 37), driver_version()."""
import inspect
import threading

import numpy as np

import hvdrv
import limited
import synth
from w4format import Config


def binds(fn, *args, **kwargs):
    inspect.signature(fn).bind(*args, **kwargs)
    return True


def test_engine_calls_of_the_server_bind():
    E = limited.Engine
    assert binds(E.__init__, object(), "/models/qwen3", kernels_dir="/opt/kernels")
    assert binds(E.verify_graph, object(), [1, 2, 3], n=24)
    assert binds(E.stream, object(), [1, 2, 3], max_new=8, stop_evt=threading.Event())
    for name in ("bind_thread", "bits_per_weight", "weight_bytes", "free"):
        assert binds(getattr(E, name), object())
    assert inspect.isgeneratorfunction(E.stream)


def test_driver_calls_of_the_server_bind():
    assert binds(hvdrv.mem_info)
    assert binds(hvdrv.device, 0)
    assert binds(hvdrv.device_name, 0)
    assert binds(hvdrv.compute_capability, 0)
    for attr in (16, 36, 37):                 # SM count, memory clock, bus width
        assert binds(hvdrv.device_attribute, 0, attr)
    assert binds(hvdrv.driver_version)
    assert hvdrv.device(0) == 0


def test_weight_figures_the_server_reports():
    """bits_per_weight and weight_bytes from the uploaded matrices (no GPU call)."""
    cfg = Config(synth.tiny_arch())
    eng = object.__new__(limited.Engine)
    eng.cfg = cfg
    c = cfg
    qd = c.head_dim
    mats = {"qkv": ((c.n_head + 2 * c.n_kv) * qd, c.hidden), "o": (c.hidden, c.n_head * qd),
            "gu": (2 * c.ffn, c.hidden), "down": (c.hidden, c.ffn)}
    eng.layers = [{k: (0, 0, kk, n, 0) for k, (n, kk) in mats.items()}
                  for _ in range(c.n_layer)]
    eng.head = (0, 0, c.hidden, c.vocab, 0)
    assert eng.bits_per_weight() == 5.0
    weights = sum(n * k for n, k in mats.values()) * c.n_layer + c.vocab * c.hidden
    assert eng.weight_bytes() == weights * 5 // 8
    assert np.isclose(eng.weight_bytes() * 8 / weights, 5.0)
