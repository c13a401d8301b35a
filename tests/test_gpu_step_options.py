"""Fused-step tuning options change how the step runs, not what it computes: with fewer
bulk copies in flight, without the L2 evict-first hint, the logits and greedy tokens are
bit-identical to the default step, for every query-group size the tiny models cover.
The reference-host BLAS run count (HV_STEP_OPT_REF_BLAS_RUNS) only changes the row dots of
gemvs of at least 3600 rows, so at these contexts it changes nothing either."""
import numpy as np
import pytest

from gpu_util import bits

pytestmark = pytest.mark.gpu

ARCHS = [dict(n_layer=2, hidden=512, ffn=1024, n_head=8, n_kv=2, vocab=4096),     # group 4
         dict(n_layer=2, hidden=512, ffn=1024, n_head=8, n_kv=8, vocab=4096),     # group 1
         dict(n_layer=2, hidden=1024, ffn=1024, n_head=16, n_kv=2, vocab=4096)]   # group 8

SETS = [{}, {1: 2}, {2: 0}, {5: 1}]
DEFAULTS = {1: 6, 2: 1, 5: 8}


@pytest.mark.parametrize("arch", ARCHS)
def test_tuning_options_are_bit_identical(hv, arch):
    import limited
    import synth
    from w4format import Config
    cfg = Config(synth.tiny_arch(**arch))
    prompt = synth.prompt_ids(cfg, 13, 40)
    out = []
    try:
        for opts in SETS:
            for k, v in DEFAULTS.items():
                hv.step_set_option(k, opts.get(k, v))
            eng = limited.Engine(config=cfg, tensors=synth.iter_tensors(cfg, 13), quiet=True,
                                 max_context=128, fused=True)
            try:
                lg = eng.logits(prompt)
                toks, _, _ = eng.generate(prompt, max_new=12)
                out.append((lg, toks))
            finally:
                eng.free()
    finally:
        for k, v in DEFAULTS.items():
            hv.step_set_option(k, v)
    for lg, toks in out[1:]:
        assert np.array_equal(bits(out[0][0]), bits(lg))
        assert out[0][1] == toks
