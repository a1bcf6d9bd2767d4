"""GPU parity of the skinny tcgen05 GEMM on packed Q4_K / Q6_K weights (SMALLMIND_GEMM_SK=1;
M >= 5 rows of x through MatMul, up to 64) against the CPU oracle.

|y - y_ref| <= 1e-4 * max(max|y_ref|, rms(y_ref)) per element (FusedQ4KMatMul.cs:90-134,
FusedQ6KMatMul.cs M-blocked paths; element formulas Q4KTensor.cs:129-147, Q6KTensor.cs:105-124).
Shapes cover each x-tile width (16 / 32 / 64 columns), ragged M and N (a partial 128-row
weight tile), K from one block to 22 blocks (split over up to 22 k slices, one block each),
more weight tiles than SMs (no split), and a 64-sequence batched decode of a model whose
Q|K|V stack mixes Q4_K and Q6_K rows.
"""
import numpy as np
import pytest

from conftest import cosine, rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.fixture(autouse=True)
def _skinny_on(monkeypatch):
    monkeypatch.setenv("SMALLMIND_GEMM_SK", "1")


def _run(ctx, O, scheme, m, k, n, seed=0, xscale=1.0):
    import smallmind_b200 as sm
    t = O.quantize(O.fill_normal(n * k, 700 + seed, 0.02), getattr(O, scheme), n, k)
    a = (np.random.RandomState(seed).randn(m, k) * xscale).astype(np.float32)
    ref = O.matmul(t, a, m, k, n, mode=1)
    out = np.empty((m, n), np.float32)
    sm.CudaWeightTensor.from_qtensor(ctx, t).MatMul(a, out, m, k, n)
    return out, ref


@pytest.mark.parametrize("scheme", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("m", [5, 8, 16, 17, 32, 33, 64])
@pytest.mark.parametrize("k,n", [(256, 128), (2048, 200), (5632, 384)])
def test_gemm_sk_vs_oracle(ctx, O, scheme, m, k, n):
    out, ref = _run(ctx, O, scheme, m, k, n, seed=m + k)
    assert np.isfinite(out).all()
    assert rel_err(out, ref) <= TOL


@pytest.mark.parametrize("scheme", ["Q4_K", "Q6_K"])
def test_gemm_sk_more_tiles_than_sms(ctx, O, scheme):
    # 160 weight tiles: no k split, a second wave of CTAs
    out, ref = _run(ctx, O, scheme, 24, 512, 128 * 160, seed=3)
    assert rel_err(out, ref) <= TOL


def test_gemm_sk_small_activations(ctx, O):
    # activations far below 1: the fp16 low planes of x (and of the x sums) in their subnormal range
    out, ref = _run(ctx, O, "Q4_K", 40, 1024, 256, seed=7, xscale=1e-3)
    assert rel_err(out, ref) <= TOL


@pytest.mark.parametrize("scheme", ["Q4_K", "Q6_K"])
def test_gemm_sk_off_falls_back(ctx, O, monkeypatch, scheme):
    """SMALLMIND_GEMM_SK=0 (the default when unset): the 128-row-tile GEMM on fp16 weight
    planes, same tolerance."""
    monkeypatch.setenv("SMALLMIND_GEMM_SK", "0")
    out, ref = _run(ctx, O, scheme, 33, 1024, 200, seed=9)
    assert rel_err(out, ref) <= TOL


def test_batched_decode_64_sequences_mixed_stack(ctx, O):
    """64 rows per decode step: Q|K (Q4_K) and V (Q6_K) stacked in one skinny GEMM."""
    import smallmind_b200 as sm
    cfg = dict(vocab_size=384, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_hidden=512,
               max_context=16, norm_eps=1e-5, rope_theta=10000.0)
    schemes = dict(wq=O.Q4_K, wk=O.Q4_K, wv=O.Q6_K, wo=O.Q4_K, w_gate=O.Q4_K, w_up=O.Q4_K, w_down=O.Q6_K,
                   output=O.Q6_K)
    host = O.make_model(cfg, schemes, seed=21)
    model = sm.CudaModel.from_host(ctx, host)
    n = 64
    kv = sm.KVCache(model, n, 16)
    rs = np.random.RandomState(6)
    hist, nxt = [], []
    for s in range(n):
        p = rs.randint(0, cfg["vocab_size"], 2 + s % 4).astype(np.int32)
        t, _ = kv.prefill(s, p, want_logits=False)
        hist.append(list(p) + [t])
        nxt.append(t)
    order = list(range(n))[::-1]
    toks, lg = kv.decode(order, [nxt[s] for s in order])
    for row, s in enumerate(order):
        ref = O.model_forward(host, np.array(hist[s], np.int32), 1)[0]
        assert cosine(lg[row], ref) >= 0.9999
        assert int(toks[row]) == int(np.argmax(ref))
