"""Generate golden vectors by running HIVE Limited's own numpy reference.

Runs ONLY where the reference checkout exists; the resulting
.npz files are committed and the tests read those, never the reference itself.

    python tests/golden/make_golden.py ops         # op-level vectors (seconds)
    python tests/golden/make_golden.py gemv        # GEMV sweep digests (a minute)
    python tests/golden/make_golden.py tiny        # tiny-model greedy decode (seconds)
    python tests/golden/make_golden.py long        # tiny model, 300- and 2000-token prompts
    python tests/golden/make_golden.py c1          # 1.7B-shape 32+64 decode (~1 hour)
    python tests/golden/make_golden.py c3          # 8B-shape 4+2 decode (~40 GB RAM)
    python tests/golden/make_golden.py numerics    # np.exp and `keys @ q` samples (seconds)

The reference's engine/limited.py dlopens libcuda at import; a stub `cudrv` module is
placed in sys.modules first so that its pure-numpy parts (quantize_w4, Config) and all of
engine/reference.py import without a GPU. Model weights are handed to the reference by
replacing limited.Config.load / limited.load_model_tensors with the synthetic model.
"""
from __future__ import annotations

import hashlib
import os
import sys
import time
import types
from pathlib import Path

import numpy as np

REF_ENGINE = Path(os.environ.get("HIVE_REFERENCE", "/root/reference")) / "engine"
HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "hive-limited_b200"))

F32 = np.float32


def load_reference():
    if not REF_ENGINE.exists():
        raise SystemExit(f"reference not found at {REF_ENGINE}")
    sys.modules.setdefault("cudrv", types.ModuleType("cudrv"))
    sys.path.insert(0, str(REF_ENGINE))
    import limited as ref_limited      # noqa: E402  (the reference's module)
    import reference as ref            # noqa: E402
    return ref_limited, ref


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ---------------------------------------------------------------------------

def make_ops(out: Path):
    L, R = load_reference()
    g = np.random.default_rng(12345)
    d = {}
    # quantize_act: random, a zero block, exact .5 ties, huge/tiny magnitudes, negatives
    acts = []
    a = g.standard_normal(32 * 64).astype(F32)
    acts.append(a)
    z = g.standard_normal(32 * 8).astype(F32)
    z[32:64] = 0.0
    z[64:96] = -0.0
    z[96:128] = np.linspace(-127, 127, 32).astype(F32)          # s == 1, exact .5 cases
    z[128:160] = (np.arange(32) - 15.5).astype(F32) * F32(127.0 / 16.0)
    z[160:192] = g.standard_normal(32).astype(F32) * F32(1e-30)
    z[192:224] = g.standard_normal(32).astype(F32) * F32(1e30)
    z[224:256] = -np.abs(g.standard_normal(32)).astype(F32)
    acts.append(z)
    for i, a in enumerate(acts):
        q, s, bs = R.quantize_act(a)
        d[f"qa{i}_in"], d[f"qa{i}_q"], d[f"qa{i}_s"], d[f"qa{i}_bsum"] = a, q, s, bs
    # quantize_w4: random + crafted blocks (all-zero, exact halves, extremes)
    w = (g.standard_normal((16, 256)) * 0.02).astype(F32)
    w[0, :32] = 0.0
    w[1, :32] = (np.arange(32) - 16).astype(F32) * F32(0.5)     # w/s hits .5 ties
    w[2, :32] = np.where(np.arange(32) % 2, 1.0, -1.0).astype(F32)
    w[3] = g.standard_normal(256).astype(F32) * F32(1e3)
    p, sc = L.quantize_w4(w)
    d["qw_in"], d["qw_packed"], d["qw_scale"] = w, p, sc
    # gemv on a small matrix with every intermediate
    for i, (n, k) in enumerate([(64, 256), (12, 5120), (6, 25600), (8, 32 * 13), (5, 32 * 5)]):
        w = (g.standard_normal((n, k)) * 0.02).astype(F32)
        a = g.standard_normal(k).astype(F32)
        p, sc = L.quantize_w4(w)
        qa, sa, _ = R.quantize_act(a)
        qw = R._weight_ints(p, k)
        idot = np.einsum("nbk,bk->nb", qw.reshape(n, k // 32, 32), qa,
                         optimize=True).astype(np.int32)
        y = R.gemv_w4(a, p, sc, k)
        d[f"gv{i}_a"], d[f"gv{i}_packed"], d[f"gv{i}_scale"] = a, p, sc
        d[f"gv{i}_idot"], d[f"gv{i}_y"] = idot, y
    # rmsnorm: per-head [rows,128] and full vectors
    for i, shape in enumerate([(16, 128), (2048,), (4096,), (5120,), (6144,), (12288,),
                               (25600,), (3, 200)]):
        x = (g.standard_normal(shape) * g.uniform(0.1, 10)).astype(F32)
        wgt = (1.0 + 0.01 * g.standard_normal(shape[-1])).astype(F32)
        d[f"rn{i}_x"], d[f"rn{i}_w"], d[f"rn{i}_y"] = x, wgt, R.rmsnorm(x, wgt)
    # rope
    half = 64
    pos = np.arange(4400, dtype=np.float64)[:, None]
    inv = 1.0 / (1e6 ** (np.arange(half, dtype=np.float64) * 2.0 / 128))
    cos_t, sin_t = np.cos(pos * inv).astype(F32), np.sin(pos * inv).astype(F32)
    for i, p_ in enumerate([0, 1, 77, 4351]):
        v = g.standard_normal((8, 128)).astype(F32)
        d[f"rp{i}_v"], d[f"rp{i}_pos"] = v, np.int32(p_)
        d[f"rp{i}_cos"], d[f"rp{i}_sin"] = cos_t[p_], sin_t[p_]
        d[f"rp{i}_y"] = R.rope(v, p_, cos_t, sin_t)
    # silu
    gt = (g.standard_normal(4096) * 4).astype(F32)
    gt[:4] = [0.0, -0.0, 80.0, -80.0]
    up = g.standard_normal(4096).astype(F32)
    d["silu_g"], d["silu_u"], d["silu_y"] = gt, up, R.silu_mul(gt, up)
    # attention (small)
    for i, (nq, nkv, P) in enumerate([(4, 2, 1), (8, 2, 37), (8, 2, 150)]):
        kc = g.standard_normal((nkv, P + 3, 128)).astype(F32)
        vc = g.standard_normal((nkv, P + 3, 128)).astype(F32)
        q = g.standard_normal((nq, 128)).astype(F32)
        y = R.attention(q, kc, vc, P - 1, nq // nkv, 1.0 / np.sqrt(128))
        d[f"at{i}_q"], d[f"at{i}_kc"], d[f"at{i}_vc"] = q, kc, vc
        d[f"at{i}_pos"], d[f"at{i}_y"] = np.int32(P - 1), y
    np.savez_compressed(out, **d)


def make_gemv(out: Path):
    """Sweep shapes: digests of the reference's quantised weights and full outputs."""
    L, R = load_reference()
    import synth
    d = {}
    for j, (n, k) in enumerate(synth.GEMV_SHAPES):
        t0 = time.time()
        w, a = synth.gemv_case(j, n, k)
        p, sc = L.quantize_w4(w)
        del w
        qa, sa, bs = R.quantize_act(a)
        y = R.gemv_w4(a, p, sc, k)
        rows = np.unique(np.linspace(0, n - 1, 8).astype(np.int64))
        qw = R._weight_ints(p[rows], k)
        idot = np.einsum("nbk,bk->nb", qw.reshape(len(rows), k // 32, 32), qa,
                         optimize=True).astype(np.int32)
        d[f"s{j}_shape"] = np.array([n, k], np.int64)
        d[f"s{j}_packed_sha"] = np.array(sha(p))
        d[f"s{j}_scale_sha"] = np.array(sha(sc))
        d[f"s{j}_qa"], d[f"s{j}_sa"], d[f"s{j}_bsum"] = qa.astype(np.int8), sa, bs
        d[f"s{j}_y_sha"] = np.array(sha(y))
        d[f"s{j}_y_head"] = y[:2048]
        d[f"s{j}_rows"], d[f"s{j}_idot"] = rows, idot
        print(f"  gemv {n}x{k}: {time.time() - t0:.1f} s", flush=True)
    np.savez_compressed(out, **d)


def _patch_model(L, arch: dict, tensors: dict):
    cfg = L.Config(arch)
    L.Config.load = classmethod(lambda cls, _d: cfg)
    L.load_model_tensors = lambda _d: tensors
    return cfg


def make_decode(out: Path, arch: dict, seed: int, n_prompt: int, n_new: int,
                full_logits: bool):
    L, R = load_reference()
    import synth
    from w4format import Config
    cfg = Config(arch)
    t0 = time.time()
    tensors = synth.model_tensors(cfg, seed)
    ids = synth.prompt_ids(cfg, seed, n_prompt)
    _patch_model(L, arch, tensors)
    model = R.ReferenceModel("<synthetic>", max_context=n_prompt + n_new + 2)
    del tensors
    print(f"  reference model built in {time.time() - t0:.1f} s", flush=True)
    # greedy decode exactly as ReferenceModel.generate, keeping every logits vector
    model.reset()
    logits = None
    for i, tok in enumerate(ids):
        logits = model.step(int(tok), i)
    all_logits, toks, pos = [logits], [], len(ids)
    for s in range(n_new):
        nxt = int(np.argmax(logits))
        toks.append(nxt)
        logits = model.step(nxt, pos)
        all_logits.append(logits)
        pos += 1
        print(f"  step {s}: tok {nxt}  ({time.time() - t0:.0f} s)", flush=True)
    L_ = np.stack(all_logits).astype(F32)
    d = {"prompt": np.array(ids, np.int32), "tokens": np.array(toks, np.int32),
         "seed": np.int64(seed), "n_new": np.int64(n_new)}
    if full_logits:
        d["logits"] = L_
    else:
        top = np.argsort(-L_, axis=1, kind="stable")[:, :16]
        d["top_ids"] = top.astype(np.int32)
        d["top_vals"] = np.take_along_axis(L_, top, 1)
        d["sample_stride"] = np.int64(149)
        d["sample"] = L_[:, ::149]
        d["absmax"] = np.abs(L_).max(1)
        d["logits_sha"] = np.array([sha(x) for x in L_])
        d["logits0"] = L_[0]
    np.savez_compressed(out, **d)
    print(f"  done in {time.time() - t0:.0f} s", flush=True)


# Row counts of the `keys @ q` samples: every remainder mod 4 of short and long runs,
# the single-run limit of the host's OpenBLAS (128 rows x T < 460800) and the split runs
# above it (up to the 8B workload's 4352 positions).
NUMERICS_T = list(range(2, 70)) + [127, 128, 129, 130, 255, 256, 257, 299, 300, 301, 302,
                                   1999, 2000, 2001, 2002, 3598, 3599, 3600, 3601, 3602,
                                   4095, 4096, 4097, 4098, 4349, 4350, 4351, 4352, 4353]


def numerics_inputs():
    """The inputs of numerics.npz, regenerated by the tests from these seeds."""
    # float32 bit patterns spread over [-104, 0] and [0, 89] (exp's finite range)
    xneg = np.linspace(0x80000000, 0xC2D00000, 262144).astype(np.uint32).view(F32)
    xpos = np.linspace(0x00000000, 0x42B20000, 65536).astype(np.uint32).view(F32)
    rng = np.random.default_rng(12)
    q = rng.standard_normal(128, dtype=F32)
    keys = (rng.standard_normal((max(NUMERICS_T), 128), dtype=F32) * F32(0.5)).astype(F32)
    return np.concatenate([xneg, xpos]), q, keys


def make_numerics(out: Path):
    """np.exp over float32 samples and `keys @ q` (OpenBLAS gemv through numpy) for the
    row counts NUMERICS_T: the two library calls of the reference's attention and SiLU
    (engine/reference.py:99, 112-114) whose results depend on the host."""
    x, q, keys = numerics_inputs()
    arrs = {"exp_x": x, "exp_y": np.exp(x).astype(F32), "dot_T": np.array(NUMERICS_T)}
    for T in NUMERICS_T:
        arrs[f"dot_{T}"] = (np.ascontiguousarray(keys[:T]) @ q).astype(F32)
    arrs["host_cpus"] = np.array(os.cpu_count())
    np.savez_compressed(out, **arrs)
    print(f"wrote {out}", flush=True)


def main(argv):
    what = argv[1] if len(argv) > 1 else "ops"
    import synth
    if what == "ops":
        make_ops(HERE / "ops.npz")
    elif what == "gemv":
        make_gemv(HERE / "gemv_sweep.npz")
    elif what == "tiny":
        make_decode(HERE / "decode_tiny.npz", synth.tiny_arch(), 7, 5, 12, True)
        make_decode(HERE / "decode_tiny_tied.npz",
                    synth.tiny_arch(n_layer=3, hidden=512, ffn=1024, n_head=8, n_kv=2,
                                    vocab=2048, tied=True), 8, 9, 10, True)
    elif what == "long":
        # a prompt long enough that decode attention runs over several sequence chunks
        make_decode(HERE / "decode_tiny_long.npz", synth.tiny_arch(), 9, 300, 8, True)
        # over 20 positions per chunk on a 148-SM part: several position blocks per chunk
        make_decode(HERE / "decode_tiny_2k.npz", synth.tiny_arch(), 10, 2000, 4, True)
    elif what == "c3":
        # the 8B geometry (weights of the 8B workload's seed), the 4-token prompt the GPU
        # test of the large shapes uses, 2 greedy tokens
        arch, seed = synth.WORKLOADS["qwen3-8b-p4096-g256"][:2]
        make_decode(HERE / "decode_qwen3_8b_p4.npz", synth.ARCH[arch], seed, 4, 2, False)
    elif what == "c1":
        arch, seed, n_prompt, n_new = synth.WORKLOADS["qwen3-1.7b-p32-g64"]
        make_decode(HERE / "decode_qwen3_1p7b.npz", synth.ARCH[arch], seed, n_prompt,
                    n_new, False)
    elif what == "numerics":
        make_numerics(HERE / "numerics.npz")
    else:
        raise SystemExit(f"unknown target {what}")


if __name__ == "__main__":
    main(sys.argv)
