"""GPU parity of the Q4_1 and Q5_0 weight formats (block 32) through the C-ABI.

Q4_1: w = q * scale + min (Q4_1Tensor.cs:153-156); Q5_0: w = ((low | high << 4)
- 16) * scale (Q5_0Tensor.cs:157-172).  Dequant bit-exact against the oracle;
MatMul in both orientations within 1e-4 of the oracle's FusedQ4_1MatMul /
FusedQ5_0MatMul restatement (intended: y = x . W^T; literal: C = A . B with B
the K x N linear-index tensor).
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.mark.parametrize("scheme", ["Q4_1", "Q5_0"])
@pytest.mark.parametrize("rows,cols", [(7, 64), (33, 256), (5, 40), (3, 17), (128, 2048)])
def test_dequant_bit_exact(ctx, O, scheme, rows, cols):
    import smallmind_b200 as sm
    sch = getattr(O, scheme)
    t = O.quantize(O.fill_normal(rows * cols, rows + cols, 0.05), sch, rows, cols, 32)
    w = sm.CudaWeightTensor.from_qtensor(ctx, t)
    assert int(w.Scheme) == sch and w.Rows == rows and w.Cols == cols
    want = O.dequantize(t).reshape(-1)
    assert np.array_equal(w.ToFloat32().view(np.uint32), want.view(np.uint32))
    w.close()


@pytest.mark.parametrize("scheme", ["Q4_1", "Q5_0"])
@pytest.mark.parametrize("m", [1, 2, 5, 16, 33, 160])
@pytest.mark.parametrize("rows,cols", [(200, 1024), (37, 96), (19, 40)])
def test_matmul_intended_vs_oracle(ctx, O, scheme, m, rows, cols):
    import smallmind_b200 as sm
    sch = getattr(O, scheme)
    t = O.quantize(O.fill_normal(rows * cols, 5 * m + rows, 0.02), sch, rows, cols, 32)
    a = np.random.RandomState(m).randn(m, cols).astype(np.float32)
    ref = O.matmul(t, a, m, cols, rows, mode=1)
    w = sm.CudaWeightTensor.from_qtensor(ctx, t)
    out = np.empty((m, rows), np.float32)
    w.MatMul(a, out, m, cols, rows)
    assert rel_err(out, ref) <= TOL
    w.close()


@pytest.mark.parametrize("scheme", ["Q4_1", "Q5_0"])
@pytest.mark.parametrize("m,k,n", [(1, 64, 48), (3, 96, 40), (4, 33, 17)])
def test_matmul_literal_vs_oracle(ctx, O, scheme, m, k, n):
    """The reference kernels' own orientation: B is K x N, blocks of 32 along the linear index."""
    import smallmind_b200 as sm
    sch = getattr(O, scheme)
    t = O.quantize(O.fill_normal(k * n, 3 * k + n, 0.05), sch, k, n, 32)
    a = np.random.RandomState(k).randn(m, k).astype(np.float32)
    ref = O.matmul(t, a, m, k, n, mode=0)
    w = sm.CudaWeightTensor.from_qtensor(ctx, t, layout=sm.LAYOUT_REFERENCE)
    out = np.empty((m, n), np.float32)
    w.MatMul(a, out, m, k, n)
    assert rel_err(out, ref) <= TOL
    w.close()


@pytest.mark.parametrize("ttype", [3, 6])
def test_gguf_blocks_decode_on_device(ctx, O, ttype):
    """ggml Q4_1 / Q5_0 blocks -> reference layout -> device: the device decodes
    every weight to the bits of ggml's published block formula."""
    import os
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    import gguf_fixture as G

    import smallmind_b200 as sm
    from smallmind_b200 import loaders as L
    rows, cols = 24, 512
    raw = G.random_blocks(ttype, rows * cols, np.random.RandomState(ttype))
    g = L.GgufFile(3, {}, [], 0, bytes(raw))
    t = L.gguf_tensor_to_host(g, L.GgufTensorInfo("w", [cols, rows], ttype, 0))
    w = sm.CudaWeightTensor(ctx, int(t.scheme), rows, cols, t.data, t.scales, 32)
    want = G.ggml_dequant(ttype, raw)
    assert np.array_equal(w.ToFloat32().view(np.uint32), want.view(np.uint32))
    w.close()
