"""Parity at the shapes the benchmark times.

* TinyLlama width (hidden 2048, 32 q / 4 kv heads = GQA group 8, FFN 5632, vocab 32000,
  Q4_K for Q/K/O/gate/up and Q6_K for V/down/head), two layers so the oracle stays fast:
  a 2048-token prompt, then greedy decode steps, once through the one-launch decode
  kernel and once through the per-op path (SMALLMIND_MEGA=0).  Every step's logits are
  compared with the oracle's KV-cached forward on the same token history
  (TransformerModel.cs:272-344, MultiHeadAttention.cs:206-317): cosine >= 0.9999 and the
  same greedy top-1.
* Causal prefill attention at T = S = 2048 with 32 / 4 heads (MultiHeadAttention.cs:676-744,
  810-844): |y - y_ref| <= 1e-4 * max(max|y_ref|, rms(y_ref)).
* The largest op-sweep shape, K x N = 4096 x 11008, at M = 512 and 2048 through the
  tensor-core GEMM, against the fp64 product of the bit-exact dequantized weights
  (FusedQ4KMatMul.cs:90-134 M-blocked path), same tolerance.
"""
import os

import numpy as np
import pytest

from conftest import cosine, rel_err

pytestmark = pytest.mark.gpu

THREADS = max(1, min(32, os.cpu_count() or 8))
TL2 = dict(vocab_size=32000, hidden=2048, n_layers=2, n_heads=32, n_kv_heads=4, head_dim=64, ffn_hidden=5632,
           max_context=2048 + 512, norm_eps=1e-5, rope_theta=10000.0)
PROMPT = 2048
STEPS = 5


def _schemes(O):
    return dict(wq=O.Q4_K, wk=O.Q4_K, wv=O.Q6_K, wo=O.Q4_K, w_gate=O.Q4_K, w_up=O.Q4_K, w_down=O.Q6_K,
                output=O.Q6_K)


@pytest.fixture(scope="module")
def tl2(O):
    """Host model, prompt and the oracle's logits for the prompt's last row."""
    host = O.make_model(TL2, _schemes(O), seed=2024, threads=THREADS)
    prompt = np.random.RandomState(77).randint(0, TL2["vocab_size"], PROMPT).astype(np.int32)
    dec = O.KVDecoder(host, threads=THREADS)
    first = dec.step(prompt)
    return host, prompt, dec.kv.copy(), first


@pytest.mark.parametrize("mega", ["1", "0"])
def test_tinyllama_width_prefill_2048_then_decode(ctx, O, tl2, monkeypatch, mega):
    import smallmind_b200 as sm
    host, prompt, kv_after_prompt, first = tl2
    monkeypatch.setenv("SMALLMIND_MEGA", mega)
    model = sm.CudaModel.from_host(ctx, host)
    kv = sm.KVCache(model, 1, PROMPT + STEPS + 8)
    tok, lg = kv.prefill(0, prompt)
    assert cosine(lg, first) >= 0.9999
    assert tok == int(np.argmax(first))
    # both modes continue from the oracle's cache as it stood after the prompt
    dec = O.KVDecoder(host, threads=THREADS)
    dec.kv[:] = kv_after_prompt
    dec.pos = PROMPT
    launches = []
    for _ in range(STEPS):
        n0 = ctx.launch_count()
        toks, lgs = kv.decode([0], [tok])
        launches.append(ctx.launch_count() - n0)
        ref = dec.step([tok])
        assert cosine(lgs[0], ref) >= 0.9999
        assert int(toks[0]) == int(np.argmax(ref))
        tok = int(toks[0])
    assert kv.length(0) == PROMPT + STEPS
    if mega == "1":
        # one-launch decode: the whole step (22 layers or 2) is a single kernel plus the argmax tail
        assert max(launches) <= 2, launches
    else:
        assert min(launches) > 2, launches


@pytest.mark.parametrize("T", [2048])
def test_attention_prefill_2048_gqa8(ctx, O, T):
    import smallmind_b200 as sm
    nH, nKv, hd = 32, 4, 64
    rs = np.random.RandomState(2048)
    q = rs.randn(T, nH * hd).astype(np.float32)
    k = rs.randn(T, nKv * hd).astype(np.float32)
    v = rs.randn(T, nKv * hd).astype(np.float32)
    ref = O.attention(q, k, v, T, T, nH, nKv, hd, threads=THREADS)
    out = sm.attention(ctx, q, k, v, T, T, nH, nKv, hd)
    assert rel_err(out, ref) < 1e-4


@pytest.mark.parametrize("scheme", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("m", [512, 2048])
def test_op_sweep_4096x11008_prefill_m(ctx, O, scheme, m):
    import smallmind_b200 as sm
    k, n = 4096, 11008
    t = O.quantize(O.fill_normal(n * k, 4242, 0.02, THREADS), getattr(O, scheme), n, k)
    cw = sm.CudaWeightTensor.from_qtensor(ctx, t)
    w = cw.ToFloat32().reshape(n, k)
    assert np.array_equal(w.view(np.uint32), O.dequantize(t).reshape(n, k).view(np.uint32))
    a = np.random.RandomState(m).randn(m, k).astype(np.float32)
    out = np.empty((m, n), np.float32)
    cw.MatMul(a, out, m, k, n)
    ref = a.astype(np.float64) @ w.astype(np.float64).T
    assert np.isfinite(out).all()
    assert rel_err(out, ref) <= 1e-4
