"""The weight cache on a B200: an engine built from a cache entry uploads the bytes the
first engine quantised and prepacked, so logits and greedy tokens are bit-identical to
an engine that quantised from the tensors; the first cached engine wrote the entry (a
miss) and the second read it (a hit). An untied and a tied (LM head from the f16
embedding) model."""
import numpy as np
import pytest

import limited
import synth
from gpu_util import bits
from w4format import Config

pytestmark = pytest.mark.gpu
ARCHS = [dict(n_layer=2, hidden=512, ffn=1024, n_head=8, n_kv=2, vocab=4096),
         dict(n_layer=2, hidden=512, ffn=1024, n_head=8, n_kv=2, vocab=2048, tied=True)]


@pytest.mark.parametrize("arch", ARCHS)
def test_cache_miss_then_hit_gives_identical_decode(hv, tmp_path, arch):
    cfg = Config(synth.tiny_arch(**arch))
    prompt = synth.prompt_ids(cfg, 11, 6)
    out = []
    for cache in (None, tmp_path, tmp_path):
        eng = limited.Engine(config=cfg, tensors=synth.iter_tensors(cfg, 11), quiet=True,
                             max_context=32, weight_cache=cache,
                             cache_tag=None if cache is None else "synthetic:tiny:11")
        try:
            toks, _, _ = eng.generate(prompt, max_new=4)
            out.append((eng.cache_hit, toks, eng.logits(prompt)))
        finally:
            eng.free()
    assert [o[0] for o in out] == [None, False, True]
    for hit, toks, lg in out[1:]:
        assert toks == out[0][1]
        assert np.array_equal(bits(lg), bits(out[0][2]))
