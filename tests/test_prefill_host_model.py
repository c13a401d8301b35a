"""The batched prefill's host orchestration (Engine._prefill_batched), run on the CPU.

limited.Engine._prefill_batched issues its kernels through the `hvdrv` module. Here that
module is replaced, for this test only, by a fake device: one numpy byte array behind
pointer-sized integers, and every kernel the prefill launches implemented with the
oracle's own ops (gather, RMSNorm, quant_a8s, gemv_w4, q/k norm + RoPE, attention, SiLU,
residual add). The Engine code itself is unchanged. A 300-token prompt (two runs of the
256-token batch) must then leave the oracle model's KV cache and last-token logits bit for
bit, and the device state the token-by-token prefill leaves: the buffers, offsets,
positions, gate/up layout and batching of the host code are checked without a GPU. The
kernels themselves are checked on the GPU (test_gpu_prefill.py) and, for the GEMM's
indexing, by a lane-level model (test_prefill_gemm_model.py)."""
import ctypes

import numpy as np
import pytest

import hv_oracle as O
import limited
import synth
from test_prefill_gemm_model import prepack
from w4format import Config

F32 = np.float32


class FakeDevice:
    """A flat byte array addressed by integers (base + offset), and the hvdrv calls the
    batched prefill makes, computed with the oracle's ops."""

    BASE = 1 << 40

    def __init__(self, nbytes=96 << 20):
        self.mem = np.zeros(nbytes, np.uint8)
        self.top = 0
        self.w4 = {}                    # prepacked nibble pointer -> (packed, scale, qw)
        self.calls = []

    # -- memory
    def alloc(self, n):
        n = (int(n) + 255) // 256 * 256
        p = self.BASE + self.top
        self.top += n
        assert self.top <= self.mem.size, "fake device full"
        return p

    def view(self, ptr, dtype, count):
        off = int(ptr) - self.BASE
        dt = np.dtype(dtype)
        assert 0 <= off and off + count * dt.itemsize <= self.top, (ptr, count)
        return self.mem[off:off + count * dt.itemsize].view(dt)

    def put(self, arr):
        arr = np.ascontiguousarray(arr)
        p = self.alloc(arr.nbytes)
        self.view(p, np.uint8, arr.nbytes)[:] = arr.view(np.uint8).reshape(-1)
        return p

    def upload(self, dst, host_ptr, n):
        ctypes.memmove(self.mem.ctypes.data + (dst - self.BASE), host_ptr, n)

    def download(self, host_ptr, src, n):
        ctypes.memmove(host_ptr, self.mem.ctypes.data + (src - self.BASE), n)

    def memset8(self, ptr, value, n):
        self.view(ptr, np.uint8, n)[:] = value

    def copy_async(self, dst, src, n, stream=0):
        self.view(dst, np.uint8, n)[:] = self.view(src, np.uint8, n).copy()

    def synchronize(self):
        pass

    def attn_rows_scratch(self, nq, group, cap, ntok):
        return 256, 4 * ntok * (nq // group)

    # -- kernels
    def gather_rows(self, emb16, tok, h, hid, ntok, stream=0):
        self.calls.append("gather_rows")
        toks = self.view(tok, np.int32, ntok)
        vocab = (self.emb_rows, hid)
        emb = self.view(emb16, np.float16, vocab[0] * hid).reshape(vocab)
        self.view(h, F32, ntok * hid).reshape(ntok, hid)[:] = emb[toks].astype(F32)

    def rmsnorm(self, src, dst, w, rows, cols, eps=1e-5, stream=0):
        x = self.view(src, F32, rows * cols).reshape(rows, cols).copy()
        g = self.view(w, F32, cols)
        out = self.view(dst, F32, rows * cols).reshape(rows, cols)
        for r in range(rows):
            out[r] = O.rmsnorm(x[r], g, F32(eps))

    def _quant(self, src, a8, sa, nb, ntok):
        x = self.view(src, F32, ntok * nb * 32).reshape(ntok, nb * 32)
        q8 = self.view(a8, np.int8, ntok * nb * 32).reshape(ntok, nb * 32)
        s = self.view(sa, F32, ntok * 2 * nb).reshape(ntok, 2 * nb)
        for t in range(ntok):
            q, sc, b = O.quantize_act(x[t])
            q8[t], s[t, :nb], s[t, nb:] = q, sc, b.view(F32)

    def qa8s_rows(self, src, a8, sa, nb, ntok, stream=0):
        self.calls.append("qa8s_rows")
        self._quant(src, a8, sa, nb, ntok)

    def qa8s(self, src, a8, sa, nb, stream=0):
        self._quant(src, a8, sa, nb, 1)

    def _gemm(self, a8, sa, pb4, psw, dst, k8, rows, pair, ntok):
        packed, scale, qw = self.w4[pb4]
        k, nb = k8 * 8, k8 // 4
        assert packed.shape == (rows, k // 8)
        q8 = self.view(a8, np.int8, ntok * k).reshape(ntok, k)
        s = self.view(sa, F32, ntok * 2 * nb).reshape(ntok, 2 * nb)
        y = self.view(dst, F32, ntok * rows).reshape(ntok, rows)
        for t in range(ntok):
            y[t] = O.gemv_q(q8[t], s[t, :nb], packed, scale, k, qw)[1]

    def a4gemm_pp(self, a8, sa, pb4, psw, dst, k8, rows, pair, ntok, stream=0):
        self.calls.append("a4gemm_pp")
        self._gemm(a8, sa, pb4, psw, dst, k8, rows, pair, ntok)

    def a4gemm_dq(self, a8, sa, pb4, psw, dst, k8, rows, pair, ntok, stream=0):
        self.calls.append("a4gemm_dq")
        self._gemm(a8, sa, pb4, psw, dst, k8, rows, pair, ntok)

    def a4gv_pp(self, a8, sa, pb4, psw, dst, k8, rows, pair=0, stream=0):
        self._gemm(a8, sa, pb4, psw, dst, k8, rows, pair, 1)

    def a4gv_dq(self, a8, sa, pb4, psw, dst, k8, rows, pair=0, stream=0):
        self.calls.append("a4gv_dq")
        self._gemm(a8, sa, pb4, psw, dst, k8, rows, pair, 1)

    def qk_rows(self, qkv, qn, kn, cos_t, sin_t, pos0, q_out, kc, vc, nq, nkv, hd, cap, eps,
                ntok, stream=0, f16=False):
        self.calls.append("qk_rows_f16" if f16 else "qk_rows")
        kt = np.float16 if f16 else F32
        rows = self.view(qkv, F32, ntok * (nq + 2 * nkv) * hd).reshape(ntok, -1)
        cs = self.view(cos_t, F32, cap * hd // 2).reshape(cap, hd // 2)
        sn = self.view(sin_t, F32, cap * hd // 2).reshape(cap, hd // 2)
        qo = self.view(q_out, F32, ntok * nq * hd).reshape(ntok, nq, hd)
        K = self.view(kc, kt, nkv * cap * hd).reshape(nkv, cap, hd)
        V = self.view(vc, kt, nkv * cap * hd).reshape(nkv, cap, hd)
        gq, gk = self.view(qn, F32, hd), self.view(kn, F32, hd)
        for t in range(ntok):
            pos = pos0 + t
            r = rows[t]
            qo[t] = O.rope(O.rmsnorm(r[:nq * hd].reshape(nq, hd), gq, F32(eps)), pos, cs, sn)
            K[:, pos] = O.rope(O.rmsnorm(r[nq * hd:(nq + nkv) * hd].reshape(nkv, hd), gk,
                                         F32(eps)), pos, cs, sn).astype(kt)
            V[:, pos] = r[(nq + nkv) * hd:].reshape(nkv, hd).astype(kt)

    def attn_rows(self, q, kc, vc, ctx, scale, pos0, nq, hd, group, kvstride, ntok, part,
                  ticket, stream=0, f16=False):
        self.calls.append("attn_rows_f16" if f16 else "attn_rows")
        kt = np.float16 if f16 else F32
        cap = kvstride // hd
        nkv = nq // group
        Q = self.view(q, F32, ntok * nq * hd).reshape(ntok, nq, hd)
        K = self.view(kc, kt, nkv * cap * hd).reshape(nkv, cap, hd).astype(F32)
        V = self.view(vc, kt, nkv * cap * hd).reshape(nkv, cap, hd).astype(F32)
        C = self.view(ctx, F32, ntok * nq * hd).reshape(ntok, nq, hd)
        sc = float(self.view(scale, F32, 1)[0])
        for t in range(ntok):
            C[t] = O.attention(Q[t], K, V, pos0 + t, group, sc)

    def vadd(self, a, b, out, n, stream=0):
        x, y = self.view(a, F32, n).copy(), self.view(b, F32, n).copy()
        self.view(out, F32, n)[:] = (x + y).astype(F32)

    def silu_rows(self, gu, act, ffn, ntok, stream=0):
        self.calls.append("silu_rows")
        g = self.view(gu, F32, ntok * 2 * ffn).reshape(ntok, 2 * ffn)
        a = self.view(act, F32, ntok * ffn).reshape(ntok, ffn)
        for t in range(ntok):
            a[t] = O.silu_mul(g[t, :ffn], g[t, ffn:])

    def argmax_partial(self, logits, pv, pi, n, parts, stream=0):
        self._argmax = O.argmax(self.view(logits, F32, n))

    def argmax_final(self, pv, pi, tok, gen, step, pos, parts, stream=0):
        s = int(self.view(step, np.int32, 1)[0])
        self.view(tok, np.int32, 1)[0] = self._argmax
        self.view(gen, np.int32, s + 1)[s] = self._argmax
        self.view(step, np.int32, 1)[0] = s + 1
        self.view(pos, np.int32, 1)[0] += 1


def fake_engine(dev, cfg, w, cap, fused, kv_dtype="f32", gemv_layout="pp"):
    """An Engine whose device state lives on the fake device (constructor bypassed)."""
    c = cfg
    eng = object.__new__(limited.Engine)
    eng.cfg, eng.fused, eng.prefill_mode = c, fused, "batched"
    eng.kv_dtype, eng.kv_f16 = kv_dtype, kv_dtype == "f16"
    eng.gemv_layout = gemv_layout
    eng.world, eng.rank, eng._pf, eng._buffers, eng._stream_cur = 1, 0, None, [], 0
    eng.quiet = True

    def w4(name, pair=0):
        packed, scale, k = w[name]
        n = packed.shape[0]
        pb4, psw = prepack(packed, scale, n, k, pair)
        p_nib, p_sc = dev.put(pb4), dev.put(psw)
        dev.w4[p_nib] = (packed, scale, O.unpack_w4(packed, k))
        return p_nib, p_sc, k, n, pair

    dev.emb_rows = c.vocab
    eng.d_emb16 = dev.put(w["emb16"])
    eng.layers = []
    for l in range(c.n_layer):
        eng.layers.append({"an": dev.put(w[f"{l}.an"]), "fn": dev.put(w[f"{l}.fn"]),
                           "qn": dev.put(w[f"{l}.qn"]), "kn": dev.put(w[f"{l}.kn"]),
                           "qkv": w4(f"{l}.qkv"), "o": w4(f"{l}.o"),
                           "gu": w4(f"{l}.gu", pair=c.ffn), "down": w4(f"{l}.down")})
    eng.d_onorm = dev.put(w["onorm"])
    eng.head = w4("head")
    eng.n_head_rows = eng.head[3]
    cos_t, sin_t = O.rope_tables(cap, c.head_dim, c.rope_theta)
    eng.d_cos, eng.d_sin = dev.put(cos_t.astype(F32)), dev.put(sin_t.astype(F32))
    eng.d_scale = dev.put(np.array([1.0 / np.sqrt(c.head_dim)], F32))
    hid, qd = c.hidden, c.head_dim
    wide = max(hid, c.ffn, c.n_head * qd)
    eng.d_h, eng.d_hn = dev.alloc(hid * 4), dev.alloc(hid * 4)
    eng.d_logits = dev.alloc(eng.n_head_rows * 4)
    eng.d_a8, eng.d_sa = dev.alloc(wide), dev.alloc(2 * (wide // 32) * 4)
    eng.d_tok, eng.d_pos, eng.d_step = dev.alloc(4), dev.alloc(4), dev.alloc(4)
    eng.d_gen = dev.alloc((cap + 1) * 4)
    eng.d_pv, eng.d_pi = dev.alloc(512), dev.alloc(512)
    per = c.n_kv * cap * qd * (2 if eng.kv_f16 else 4)
    eng.kv_bytes = 2 * c.n_layer * per
    eng.d_kv = dev.alloc(eng.kv_bytes)
    eng.KC = [eng.d_kv + 2 * l * per for l in range(c.n_layer)]
    eng.VC = [eng.d_kv + (2 * l + 1) * per for l in range(c.n_layer)]
    return eng


@pytest.mark.parametrize("fused,kv_dtype,layout", [(False, "f32", "pp"), (True, "f32", "pp"),
                                                   (True, "f16", "pp"), (False, "f32", "dq")])
def test_batched_prefill_host_code_matches_oracle(monkeypatch, fused, kv_dtype, layout):
    """kv_dtype "f16": the compressed-KV lane's prefill against the oracle run with the
    same binary16 cache rounding. layout "dq": the GEMMs and the head GEMV go to the dq
    entry points (the fake device computes them from the same weights)."""
    arch = synth.tiny_arch(n_layer=2, hidden=256, ffn=512, n_head=4, n_kv=2, vocab=1000)
    cfg = Config(arch)
    cap = 320
    cfg.max_context = cap
    w = O.quantize_model(cfg, synth.model_tensors(cfg, 5))
    prompt = synth.prompt_ids(cfg, 5, 300)
    dev = FakeDevice()
    monkeypatch.setattr(limited, "hvdrv", dev)
    eng = fake_engine(dev, cfg, w, cap, fused, kv_dtype, layout)
    eng._prefill_batched(prompt, argmax=True)
    gemm = "a4gemm_dq" if layout == "dq" else "a4gemm_pp"
    assert dev.calls.count(gemm) == 2 * cfg.n_layer * 4      # 2 batches x 4 matrices
    assert ("a4gv_dq" in dev.calls) == (layout == "dq")      # the LM head GEMV
    assert dev.calls.count("gather_rows") == 2               # 256 + 44 tokens
    sfx = "_f16" if kv_dtype == "f16" else ""
    assert dev.calls.count("qk_rows" + sfx) == dev.calls.count("attn_rows" + sfx) == 4

    m = O.OracleModel(cfg, w, cap, kv_dtype=kv_dtype)
    logits = None
    for i, tok in enumerate(prompt):
        logits = m.step(tok, i, head=(i == len(prompt) - 1))
    got = dev.view(eng.d_logits, F32, cfg.vocab)
    assert np.array_equal(got.view(np.uint32), logits.view(np.uint32))
    per = cfg.n_kv * cap * cfg.head_dim
    kt = np.float16 if kv_dtype == "f16" else F32
    for l in range(cfg.n_layer):
        K = dev.view(eng.KC[l], kt, per).reshape(cfg.n_kv, cap, cfg.head_dim).astype(F32)
        V = dev.view(eng.VC[l], kt, per).reshape(cfg.n_kv, cap, cfg.head_dim).astype(F32)
        assert np.array_equal(K.view(np.uint32), m.KC[l].view(np.uint32)), l
        assert np.array_equal(V.view(np.uint32), m.VC[l].view(np.uint32)), l
    tok, pos, step = (int(dev.view(p, np.int32, 1)[0]) for p in (eng.d_tok, eng.d_pos,
                                                                   eng.d_step))
    if fused:      # the fused step's state: first greedy token taken, position advanced
        assert (tok, pos, step) == (O.argmax(logits), len(prompt), 1)
        assert int(dev.view(eng.d_gen, np.int32, 1)[0]) == O.argmax(logits)
    else:          # the eager step's state: logits of the last prompt token, step 0
        assert (tok, pos, step) == (prompt[-1], len(prompt) - 1, 0)
