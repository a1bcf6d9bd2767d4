"""GPU parity of the tcgen05 GEMM (M >= 5, INTENDED layout) against the CPU oracle.

|y - y_ref| <= 1e-4 * max(max|y_ref|, rms(y_ref)) per element; the oracle follows the
reference element formulas and accumulation order (FusedQ4KMatMul.cs / MatMulF32Q8.cs).
Shapes cover ragged M and N (partial 128-row tiles), K of one to several 256-blocks and
the block sizes 32 and 64 of the scale-per-block formats.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _run(ctx, O, scheme, m, k, n, bs=32, seed=0, xscale=1.0):
    import smallmind_b200 as sm
    sch = getattr(O, scheme)
    w = O.fill_normal(n * k, 100 + seed, 0.02)
    t = O.quantize(w, sch, n, k, bs)
    a = (np.random.RandomState(seed).randn(m, k) * xscale).astype(np.float32)
    ref = O.matmul(t, a, m, k, n, mode=1)
    cw = sm.CudaWeightTensor.from_qtensor(ctx, t)
    out = np.empty((m, n), np.float32)
    cw.MatMul(a, out, m, k, n)
    return out, ref


@pytest.mark.parametrize("scheme", ["Q4_K", "Q6_K", "Q8_0", "Q4_0"])
@pytest.mark.parametrize("m,k,n", [(5, 512, 200), (9, 256, 128), (16, 256, 128), (64, 512, 200), (130, 1024, 256),
                                   (200, 768, 384)])
def test_gemm_tc_vs_oracle(ctx, O, scheme, m, k, n):
    out, ref = _run(ctx, O, scheme, m, k, n)
    assert np.isfinite(out).all()
    assert rel_err(out, ref) <= TOL


@pytest.mark.parametrize("scheme", ["Q8_0", "Q4_0"])
def test_gemm_tc_block64(ctx, O, scheme):
    out, ref = _run(ctx, O, scheme, 48, 1024, 160, bs=64, seed=3)
    assert rel_err(out, ref) <= TOL


@pytest.mark.parametrize("scheme", ["Q4_K", "Q6_K"])
def test_gemm_tc_prefill_shape(ctx, O, scheme):
    # an op-sweep K with a prefill-sized M (the oracle needs about a second)
    out, ref = _run(ctx, O, scheme, 512, 2048, 256, seed=5)
    assert rel_err(out, ref) <= TOL


def test_gemm_tc_small_activations(ctx, O):
    # activations far below 1 exercise the fp16 low planes in their subnormal range
    out, ref = _run(ctx, O, "Q4_K", 64, 512, 128, seed=7, xscale=1e-3)
    assert rel_err(out, ref) <= TOL


@pytest.mark.parametrize("scheme", ["Q4_K", "Q8_0"])
def test_gemm_tc_full_grid_no_split(ctx, O, scheme):
    # 2 x 74 output tiles fill the SMs, so K is not split
    out, ref = _run(ctx, O, scheme, 256, 256, 128 * 74, seed=9)
    assert rel_err(out, ref) <= TOL


def test_gemm_tc_long_k_many_slices(ctx, O):
    # one output tile and 32 k stages: K is split 16 ways and reduced in slice order
    # (the accumulating form, y += x W^T, runs in the model prefill tests)
    out, ref = _run(ctx, O, "Q6_K", 32, 2048, 256, seed=11)
    assert rel_err(out, ref) <= TOL


@pytest.mark.parametrize("planes", ["0", "1"])
@pytest.mark.parametrize("scheme", ["Q4_K", "Q6_K", "Q8_0", "Q4_0", "Q4_1", "Q5_0"])
@pytest.mark.parametrize("m,k,n", [(16, 512, 256), (64, 1024, 384), (128, 768, 200)])
def test_gemm_tc_one_tile_both_weight_paths(ctx, O, monkeypatch, planes, scheme, m, k, n):
    """M <= 128: with resident fp16 weight planes (SMALLMIND_WEIGHT_PLANES unset / 1) the
    weights come by TMA from the planes; with SMALLMIND_WEIGHT_PLANES=0 the loader warps
    dequantize each weight tile.  Both within 1e-4 of the oracle.  (SMALLMIND_GEMM_SK=0 keeps
    Q4_K / Q6_K with M <= 64 off the opt-in skinny GEMM.)"""
    monkeypatch.setenv("SMALLMIND_WEIGHT_PLANES", planes)
    monkeypatch.setenv("SMALLMIND_GEMM_SK", "0")
    out, ref = _run(ctx, O, scheme, m, k, n, seed=m + k)
    assert np.isfinite(out).all()
    assert rel_err(out, ref) <= TOL
