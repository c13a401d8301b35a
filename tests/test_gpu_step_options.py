"""Fused-step options that change how the step runs but not what it computes: with the
attention merge split into its own phase (HV_STEP_OPT_SPLIT_MERGE) the logits and greedy
tokens are bit-identical to the default step, for every query-group size the tiny models
cover."""
import os

import numpy as np
import pytest

from gpu_util import bits

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(
    not os.environ.get("HV_NEW_GPU_TESTS"),
    reason="kernels not yet run on a B200: set HV_NEW_GPU_TESTS=1")]

ARCHS = [dict(n_layer=2, hidden=512, ffn=1024, n_head=8, n_kv=2, vocab=4096),     # group 4
         dict(n_layer=2, hidden=512, ffn=1024, n_head=8, n_kv=8, vocab=4096),     # group 1
         dict(n_layer=2, hidden=1024, ffn=1024, n_head=16, n_kv=2, vocab=4096)]   # group 8


@pytest.mark.parametrize("arch", ARCHS)
def test_split_merge_is_bit_identical(hv, arch):
    import limited
    import synth
    from w4format import Config
    cfg = Config(synth.tiny_arch(**arch))
    prompt = synth.prompt_ids(cfg, 13, 40)
    out = []
    try:
        for split in (0, 1):
            hv.step_set_option(hv.STEP_OPT_SPLIT_MERGE, split)
            eng = limited.Engine(config=cfg, tensors=synth.iter_tensors(cfg, 13), quiet=True,
                                 max_context=128, fused=True)
            try:
                lg = eng.logits(prompt)
                toks, _, _ = eng.generate(prompt, max_new=12)
                out.append((lg, toks))
            finally:
                eng.free()
    finally:
        hv.step_set_option(hv.STEP_OPT_SPLIT_MERGE, 0)
    assert np.array_equal(bits(out[0][0]), bits(out[1][0]))
    assert out[0][1] == out[1][1]
