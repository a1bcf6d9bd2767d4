"""Pins the CPU oracle against the reference's own known-answer tests.

Every exact value asserted here comes from the reference's test suite (cited
per test); the seeded matmul tests replay the reference's inputs (System.Random(42))
at the reference's own tolerances.  Runs on CPU.
"""
import math
import os

import numpy as np
import pytest

from conftest import rel_err

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


# ---------------------------------------------------------------- exact pins
def test_q4_decode_nibble_known_answers(O):
    # tests/SmallMind.Quantization.Tests/QuantKernelsTests.cs:149-158
    L = O.lib()
    for nib, val in [(0, 0), (1, 1), (7, 7), (8, -8), (9, -7), (15, -1)]:
        assert L.or_q4_decode_nibble(nib) == val


def test_kquant_block_geometry(O):
    # KQuantTensorTests.cs:19-29 (Q4_K 256 / 144 B) and :145-155 (Q6_K 256 / 210 B);
    # tensor byte lengths :32-44, :158-170 (256x256 -> 256 blocks).
    x = np.zeros(256 * 256, np.float32)
    assert O.quantize(x, O.Q4_K, 256, 256).data.size == 256 * 144
    assert O.quantize(x, O.Q6_K, 256, 256).data.size == 256 * 210
    with pytest.raises(AssertionError):  # Columns must be divisible by 256 (:46-51, :172-177)
        O.quantize(np.zeros(256 * 100, np.float32), O.Q4_K, 256, 100)


def test_dotnet_random_seed42_sequence(O):
    # System.Random(42) legacy seeded sequence that feeds every seeded reference test.
    r = O.dotnet_random(42)
    vals = [O.lib().or_dotnet_random_next_double(r) for _ in range(3)]
    assert vals[0] == pytest.approx(0.6681064659115423, abs=1e-15)
    assert all(0.0 <= v < 1.0 for v in vals)


def test_rmsnorm_known_values(O):
    # tests/SmallMind.Tests/RMSNormOpsTests.cs:14-37 (2x3 rows), :40-61 (gamma), :128-141 (zeros), :145-166
    x = np.array([1, 2, 3, 4, 5, 6], np.float32)
    y = O.rmsnorm(x.reshape(2, 3), np.ones(3, np.float32))
    for r in range(2):
        row = x[3 * r:3 * r + 3]
        inv = np.float32(1) / np.sqrt(np.float32(np.sum(row * row)) / np.float32(3) + np.float32(1e-5))
        np.testing.assert_allclose(y[r], row * inv, rtol=1e-6)
    y = O.rmsnorm(np.array([[1, 2, 3]], np.float32), np.array([2, 3, 4], np.float32))
    inv = 1 / math.sqrt(14 / 3 + 1e-5)
    np.testing.assert_allclose(y[0], np.array([2, 6, 12]) * inv, rtol=1e-6)
    assert np.all(O.rmsnorm(np.zeros((1, 3), np.float32), np.ones(3, np.float32)) == 0)
    x = np.array([[0.5, 1.5, 2.5, 3.5]], np.float32)
    g = np.array([1.2, 0.8, 1.5, 0.5], np.float32)
    rms = math.sqrt((0.25 + 2.25 + 6.25 + 12.25) / 4 + 1e-5)
    np.testing.assert_allclose(O.rmsnorm(x, g)[0], g * x[0] / rms, rtol=1e-6)


def test_rope_known_behaviour(O):
    # tests/SmallMind.Tests/RotaryEmbeddingTests.cs:33-61 (identity at position 0),
    # :64-88 (positions differ), :91-113 (GQA head counts), :143-160 (offsets).
    s, c = O.rope_tables(512, 4)
    q = np.array([1, 0, 1, 0], np.float32)
    assert np.array_equal(O.rope_apply(q, 1, 4, 0, s, c), q)
    assert O.rope_apply(q, 1, 4, 1, s, c)[0] != q[0]
    q16 = np.arange(16, dtype=np.float32)
    assert np.array_equal(O.rope_apply(q16, 4, 4, 0, s, c), q16)
    assert O.rope_apply(q, 1, 4, 10, s, c)[0] != q[0]
    # frequency formula 1/theta^(2i/hd): position 1 rotates pair 0 by exactly 1 radian
    r = O.rope_apply(np.array([1, 0, 0, 0], np.float32), 1, 4, 1, s, c)
    assert r[0] == pytest.approx(math.cos(1.0), abs=1e-6) and r[1] == pytest.approx(math.sin(1.0), abs=1e-6)


def test_fast_exp_pade(O):
    # MathUtils.cs:20-32: (1 + x/2 + x^2/12) / (1 - x/2 + x^2/12), x clamped to [-87.3, 88.7]
    for x in [0.0, -0.5, -1.0, -10.0, -87.3, -200.0, 3.0]:
        xc = np.float32(max(-87.3, min(x, 88.7)))
        x2 = xc * xc
        num = np.float32(np.float32(1) + xc * np.float32(0.5)) + x2 * np.float32(0.08333333)
        den = np.float32(np.float32(1) - xc * np.float32(0.5)) + x2 * np.float32(0.08333333)
        assert O.fast_exp(float(x)) == np.float32(num / den)
    assert O.fast_exp(0.0) == 1.0
    assert abs(O.fast_exp(-10.0) - 0.3023) < 1e-3  # far from exp(-10): the reference's own approximation


# ---------------------------------------------------------------- replays of the seeded reference tests
def _matmul_float(a, b, m, k, n):
    # MatMulReference (QuantKernelsTests.cs:271-287): float32 accumulation
    c = np.zeros((m, n), np.float32)
    for i in range(m):
        for j in range(n):
            s = np.float32(0)
            for p in range(k):
                s = np.float32(s + np.float32(a[i * k + p] * b[p * n + j]))
            c[i, j] = s
    return c.reshape(-1)


def _assert_arrays_close(expected, actual, tol):
    # AssertArraysClose (QuantKernelsTests.cs:289-314)
    for e, a in zip(expected, actual):
        err = abs(a - e)
        if abs(e) < 0.1:
            assert err < tol
        else:
            assert err / abs(e) < tol


@pytest.mark.parametrize("scheme,tol", [("q8", 0.16), ("q4", 5.0)])
@pytest.mark.parametrize("m,k,n,bs", [(2, 16, 8, 8), (1, 32, 16, 16), (4, 64, 32, 64)])
def test_reference_seeded_matmul_tests(O, scheme, tol, m, k, n, bs):
    # QuantKernelsTests.cs:47-142: a, b ~ U(-1, 1) from Random(42); B quantized KxN; C = A.B literal
    r = O.dotnet_random(42)
    a = O.dotnet_random_floats(r, m * k, -1.0, 1.0)
    b = O.dotnet_random_floats(r, k * n, -1.0, 1.0)
    sch = O.Q8_0 if scheme == "q8" else O.Q4_0
    t = O.quantize(b, sch, k, n, bs)
    got = O.matmul(t, a, m, k, n, mode=0).reshape(-1)
    _assert_arrays_close(_matmul_float(a, b, m, k, n), got, tol)


@pytest.mark.parametrize("scheme,tol", [("q8", 0.16), ("q4", 5.0)])
def test_reference_quantize_roundtrip(O, scheme, tol):
    # QuantKernelsTests.cs:15-45: 4x8 values U(-10, 10), block 4
    r = O.dotnet_random(42)
    x = O.dotnet_random_floats(r, 32, -10.0, 10.0)
    t = O.quantize(x, O.Q8_0 if scheme == "q8" else O.Q4_0, 4, 8, 4)
    _assert_arrays_close(x, O.dequantize(t).reshape(-1), tol)


def test_q8_quantize_rounding_is_half_even(O):
    # Q8Tensor.cs:117 MathF.Round -> ToEven: 0.5 -> 0, 1.5 -> 2, 2.5 -> 2 with scale 1 (maxAbs 127)
    x = np.array([127.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5], np.float32)
    t = O.quantize(x, O.Q8_0, 1, 8, 8)
    assert t.scales[0] == 1.0
    assert list(t.data) == [127, 0, 2, 2, 0, -2, -2, 126]


def test_q4_packing_global_index(O):
    # Q4Tensor.cs:119-129: even linear index -> low nibble, odd -> high, even when a byte
    # straddles two scale blocks (block size 3 here).
    x = np.array([7, -7, 1, -1, 7, 7], np.float32)
    t = O.quantize(x, O.Q4_0, 1, 6, 3)
    assert list(t.scales) == [1.0, 1.0]
    assert list(t.data) == [0x97, 0xF1, 0x77]
    assert list(O.dequantize(t).reshape(-1)) == [7, -7, 1, -1, 7, 7]


# ---------------------------------------------------------------- K-quants and orientations
@pytest.mark.parametrize("scheme", ["q4_k", "q6_k", "q8_0", "q4_0"])
def test_golden_fixtures_reproduce(O, scheme):
    g = np.load(os.path.join(GOLDEN, f"quant_{scheme}.npz"))
    sch = int(g["scheme"])
    t = O.quantize(g["source"], sch, int(g["rows"]), int(g["cols"]), int(g["block_size"]))
    assert np.array_equal(t.data.view(np.uint8), g["data"].view(np.uint8))
    assert np.array_equal(O.dequantize(t).reshape(-1), g["dequant"])
    y = O.matmul(t, g["a"], g["a"].shape[0], int(g["cols"]), int(g["rows"]), mode=1)
    assert np.array_equal(y, g["y_intended"])


@pytest.mark.parametrize("scheme", ["Q4_K", "Q6_K"])
def test_kquant_element_formula_and_orders(O, scheme):
    sch = getattr(O, scheme)
    rows, cols = 16, 768
    x = O.fill_normal(rows * cols, 3, 0.02)
    t = O.quantize(x, sch, rows, cols)
    deq = O.dequantize(t)
    assert np.abs(deq.reshape(-1) - x).max() < 0.25 * np.abs(x).max()
    a = np.random.RandomState(1).randn(2, cols).astype(np.float32)
    yi, y64 = O.matmul(t, a, 2, cols, rows, mode=1, want64=True)
    assert rel_err(yi, y64) < 1e-5
    np.testing.assert_allclose(y64, a.astype(np.float64) @ deq.astype(np.float64).T, rtol=1e-9, atol=1e-9)
    # the reference fused kernels' block order (k/256)*N + n gives the same product
    lit = O.reorder_kquant_blocks_to_literal(t)
    assert np.array_equal(O.matmul(lit, a, 2, cols, rows, mode=0), yi)


def test_q4k_scale_packing_roundtrip(O):
    # 6-bit sequential scale/min packing (Q4KTensor.cs:109-126) inverted by the quantizer
    x = O.fill_normal(256, 11, 1.0)
    t = O.quantize(x, O.Q4_K, 1, 256)
    blk = t.data
    s = blk[4:16].astype(np.int32)
    sc = [s[0] & 63, (s[0] >> 6) | ((s[1] & 15) << 2), (s[1] >> 4) | ((s[2] & 3) << 4), (s[2] >> 2) & 63]
    assert all(0 <= v < 64 for v in sc)
    deq = O.dequantize(t).reshape(-1)
    d = O.lib().or_half_to_float(int(blk[0]) | (int(blk[1]) << 8))
    dmin = O.lib().or_half_to_float(int(blk[2]) | (int(blk[3]) << 8))
    q0 = blk[16] & 0xF
    expect = np.float32(np.float32(d * np.float32(sc[0])) * np.float32(q0)) - np.float32(dmin * np.float32(s[6] & 63))
    assert deq[0] == expect


def test_attention_matches_numpy_pade(O):
    T, S, nH, nKv, hd = 3, 7, 4, 2, 64
    rs = np.random.RandomState(0)
    q = rs.randn(T, nH * hd).astype(np.float32)
    k = rs.randn(S, nKv * hd).astype(np.float32)
    v = rs.randn(S, nKv * hd).astype(np.float32)
    out = O.attention(q, k, v, T, S, nH, nKv, hd)
    fe = np.vectorize(O.fast_exp)
    for i in range(T):
        for h in range(nH):
            g = h // (nH // nKv)
            valid = S - T + i + 1
            s = (k[:valid, g * hd:(g + 1) * hd] @ q[i, h * hd:(h + 1) * hd]) * 0.125
            e = fe((s - s.max()).astype(np.float32))
            p = e / e.sum()
            ref = p @ v[:valid, g * hd:(g + 1) * hd]
            np.testing.assert_allclose(out[i, h * hd:(h + 1) * hd], ref, rtol=2e-4, atol=2e-5)


def test_tiny_model_fixture_reproduces(O):
    g = np.load(os.path.join(GOLDEN, "tiny_llama_q4k.npz"))
    cfg = dict(vocab_size=384, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_hidden=512,
               max_context=48, norm_eps=1e-5, rope_theta=10000.0)
    schemes = dict(wq=O.Q4_K, wk=O.Q4_K, wv=O.Q6_K, wo=O.Q4_K, w_gate=O.Q4_K, w_up=O.Q4_K, w_down=O.Q6_K,
                   output=O.Q6_K)
    host = O.make_model(cfg, schemes, seed=int(g["seed"]))
    toks = list(g["prompt"])
    for step in range(g["logits"].shape[0]):
        lg = O.model_forward(host, np.array(toks, np.int32), 1)[0]
        assert np.array_equal(lg, g["logits"][step])
        toks.append(int(np.argmax(lg)))
    assert toks == list(g["tokens"])


def test_kv_step_twin_matches_full_recompute(O):
    cfg = dict(vocab_size=300, hidden=256, n_layers=2, n_heads=4, n_kv_heads=1, head_dim=64, ffn_hidden=256,
               max_context=32, norm_eps=1e-5, rope_theta=10000.0)
    schemes = dict(wq=O.Q8_0, wk=O.Q8_0, wv=O.Q8_0, wo=O.Q8_0, w_gate=O.Q8_0, w_up=O.Q8_0, w_down=O.Q8_0,
                   output=O.Q8_0)
    host = O.make_model(cfg, schemes, seed=9, block_size=64)
    toks = np.random.RandomState(2).randint(0, 300, 9).astype(np.int32)
    dec = O.KVDecoder(host)
    dec.step(toks[:6])
    for t in range(6, 9):
        lg = dec.step(toks[t:t + 1])
        ref = O.model_forward(host, toks[:t + 1], 1)[0]
        assert rel_err(lg, ref) < 1e-5


# ---------------------------------------------------------------- Q4_1 / Q5_0
@pytest.mark.parametrize("scheme,m,k,n,lo,tol", [("Q4_1", 4, 64, 32, 2.0, 5.0), ("Q5_0", 4, 64, 32, 3.0, 3.0),
                                                 ("Q4_1", 1, 64, 64, 1.0, 5.0), ("Q5_0", 1, 64, 64, 1.0, 3.0)])
def test_reference_fused_q41_q50_matches_dequantized(O, scheme, m, k, n, lo, tol):
    # ExpandedQuantizationTests.cs:229-300: Random(42), a ~ U(-1, 1), B ~ U(-lo, lo) quantized K x N;
    # the fused kernel against matmul over the dequantized B, percent tolerance per element
    r = O.dotnet_random(42)
    a = O.dotnet_random_floats(r, m * k, -1.0, 1.0)
    b = O.dotnet_random_floats(r, k * n, -lo, lo)
    t = O.quantize(b, getattr(O, scheme), k, n, 32)
    expected = _matmul_float(a, O.dequantize(t).reshape(-1), m, k, n)
    got = O.matmul(t, a, m, k, n, mode=0).reshape(-1)
    _assert_arrays_close(expected, got, tol)


@pytest.mark.parametrize("scheme", ["Q4_1", "Q5_0"])
@pytest.mark.parametrize("rows,cols", [(4, 64), (3, 50), (1, 7)])
def test_q41_q50_sizes_and_determinism(O, scheme, rows, cols):
    # ExpandedQuantizationTests.cs:95-193: block size fixed at 32; data (n+1)/2 bytes, one scale (and min)
    # per block, 4 high-bit bytes per block (Q5_0); the same input quantizes to the same bytes
    n, nb = rows * cols, (rows * cols + 31) // 32
    x = O.fill_normal(n, 11, 1.0)
    t1, t2 = O.quantize(x, getattr(O, scheme), rows, cols, 32), O.quantize(x.copy(), getattr(O, scheme), rows, cols, 32)
    assert t1.block_size == 32
    if scheme == "Q4_1":
        assert t1.data.size == (n + 1) // 2 and t1.scales.size == 2 * nb
    else:
        assert t1.data.size == (n + 1) // 2 + 4 * nb and t1.scales.size == nb
    assert np.array_equal(t1.data, t2.data) and np.array_equal(t1.scales, t2.scales)
    # the element formulas (Q4_1Tensor.cs:153-156, Q5_0Tensor.cs:157-172) from the packed fields
    d = O.dequantize(t1).reshape(-1)
    i = np.arange(n)
    nib = np.where(i & 1, t1.data[i >> 1] >> 4, t1.data[i >> 1] & 0xF).astype(np.int64)
    sc = t1.scales[i >> 5]
    if scheme == "Q4_1":
        want = (nib.astype(np.float32) * sc).astype(np.float32) + t1.scales[nb + (i >> 5)]
    else:
        hw = t1.data[(n + 1) // 2:].view(np.uint32).astype(np.int64)
        q = (nib | (((hw[i >> 5] >> (i & 31)) & 1) << 4)) - 16
        want = q.astype(np.float32) * sc
    assert np.array_equal(d.view(np.uint32), want.astype(np.float32).view(np.uint32))
