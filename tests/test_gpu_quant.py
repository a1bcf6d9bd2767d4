"""GPU parity of the quantized operators through the C-ABI (IWeightTensor drop-in).

Dequant and quantize: bit-exact.  GEMV/GEMM: |y - y_ref| <= 1e-4 * max(max|y_ref|, rms(y_ref)).
"""
import os

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TOL = 1e-4
SCHEMES = ["q8_0", "q4_0", "q4_k", "q6_k"]


def _golden(name):
    return np.load(os.path.join(GOLDEN, f"quant_{name}.npz"))


@pytest.mark.parametrize("name", SCHEMES)
def test_dequant_bit_exact_golden(ctx, name):
    import smallmind_b200 as sm
    g = _golden(name)
    w = sm.CudaWeightTensor(ctx, int(g["scheme"]), int(g["rows"]), int(g["cols"]), g["data"],
                            g["scales"] if "scales" in g else None, int(g["block_size"]))
    assert w.Rows == int(g["rows"]) and w.Cols == int(g["cols"]) and int(w.Scheme) == int(g["scheme"])
    assert np.array_equal(w.ToFloat32().view(np.uint32), g["dequant"].view(np.uint32))


@pytest.mark.parametrize("name", SCHEMES)
def test_matmul_golden_both_orientations(ctx, name):
    import smallmind_b200 as sm
    g = _golden(name)
    rows, cols, bs = int(g["rows"]), int(g["cols"]), int(g["block_size"])
    sc = g["scales"] if "scales" in g else None
    w = sm.CudaWeightTensor(ctx, int(g["scheme"]), rows, cols, g["data"], sc, bs)
    a = g["a"]
    m = a.shape[0]
    out = np.empty((m, rows), np.float32)
    w.MatMul(a, out, m, cols, rows)
    assert rel_err(out, g["y_intended"]) <= TOL
    if name in ("q4_k", "q6_k"):
        lk, ln = int(g["lit_k"]), int(g["lit_n"])
        wl = sm.CudaWeightTensor(ctx, int(g["scheme"]), lk, ln, g["literal_data"], None, bs,
                                 layout=sm.LAYOUT_REFERENCE)
        out2 = np.empty((m, ln), np.float32)
        wl.MatMul(g["a_literal"], out2, m, lk, ln)
        assert rel_err(out2, g["y_literal"]) <= TOL
    else:
        wl = sm.CudaWeightTensor(ctx, int(g["scheme"]), rows, cols, g["data"], sc, bs, layout=sm.LAYOUT_REFERENCE)
        a2 = g["a_literal"]
        out2 = np.empty((m, cols), np.float32)
        wl.MatMul(a2, out2, m, rows, cols)
        assert rel_err(out2, g["y_literal"]) <= TOL


@pytest.mark.parametrize("scheme", ["Q8_0", "Q4_0", "Q4_K", "Q6_K"])
@pytest.mark.parametrize("m", [1, 2, 3, 8, 9, 17])
def test_matmul_vs_oracle_ragged_m(ctx, O, scheme, m):
    import smallmind_b200 as sm
    sch = getattr(O, scheme)
    rows, cols = 200, 1024  # rows not a multiple of the per-warp row group
    x = O.fill_normal(rows * cols, 77, 0.02)
    t = O.quantize(x, sch, rows, cols, 32)
    a = np.random.RandomState(m).randn(m, cols).astype(np.float32)
    ref = O.matmul(t, a, m, cols, rows, mode=1)
    w = sm.CudaWeightTensor.from_qtensor(ctx, t)
    out = np.empty((m, rows), np.float32)
    w.MatMul(a, out, m, cols, rows)
    assert rel_err(out, ref) <= TOL


@pytest.mark.parametrize("scheme", ["Q8_0", "Q4_0"])
@pytest.mark.parametrize("m,k,n,bs", [(2, 16, 8, 8), (1, 32, 16, 16), (4, 64, 32, 64), (3, 48, 40, 4)])
def test_reference_seeded_literal_tests(ctx, O, scheme, m, k, n, bs):
    # replays QuantKernelsTests.cs:47-142 inputs (Random(42)) through the literal C = A.B path
    import smallmind_b200 as sm
    r = O.dotnet_random(42)
    a = O.dotnet_random_floats(r, m * k, -1.0, 1.0)
    b = O.dotnet_random_floats(r, k * n, -1.0, 1.0)
    t = O.quantize(b, getattr(O, scheme), k, n, bs)
    ref = O.matmul(t, a, m, k, n, mode=0)
    w = sm.CudaWeightTensor.from_qtensor(ctx, t, layout=sm.LAYOUT_REFERENCE)
    out = np.empty((m, n), np.float32)
    w.MatMul(a, out, m, k, n)
    assert rel_err(out, ref) <= TOL
    assert np.array_equal(w.ToFloat32(), O.dequantize(t).reshape(-1))


@pytest.mark.parametrize("scheme", ["Q8_0", "Q4_0", "Q4_K", "Q6_K"])
@pytest.mark.parametrize("bs", [32, 64])
def test_device_quantizer_bit_exact(ctx, O, scheme, bs):
    import torch

    import smallmind_b200 as sm
    sch = getattr(O, scheme)
    rows, cols = 64, 512
    x = O.fill_normal(rows * cols, 5 + bs, 0.02)
    x[:7] = [0.0, 0.5, -0.5, 1e-8, -3.0, 3.0, 0.0]  # ties, tiny and large values
    t = O.quantize(x, sch, rows, cols, bs)
    xd = torch.from_numpy(x).cuda()
    nbytes = t.data.size
    dd = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    sd = torch.empty(max(1, 0 if t.scales is None else t.scales.size), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    rc = sm.lib().sm_quantize(ctx.handle, sch, xd.data_ptr(), x.size, bs, dd.data_ptr(), sd.data_ptr())
    assert rc == 0, sm.last_error()
    ctx.sync()
    assert np.array_equal(dd.cpu().numpy(), t.data.view(np.uint8))
    if t.scales is not None:
        assert np.array_equal(sd.cpu().numpy().view(np.uint32), t.scales.view(np.uint32))


def test_shape_errors_like_reference(ctx, O):
    import smallmind_b200 as sm
    t = O.quantize(O.fill_normal(8 * 256, 1), O.Q4_K, 8, 256)
    w = sm.CudaWeightTensor.from_qtensor(ctx, t)
    a = np.zeros((1, 256), np.float32)
    with pytest.raises(ValueError):  # k must equal the weight's K (Q4KWeightTensor.cs:43)
        w.MatMul(a, np.empty((1, 8), np.float32), 1, 128, 8)
    with pytest.raises(ValueError):  # n must equal the weight's N (:44)
        w.MatMul(a, np.empty((1, 8), np.float32), 1, 256, 7)
    with pytest.raises(ValueError):  # output too short (:47-48)
        w.MatMul(a, np.empty((1, 4), np.float32), 1, 256, 8)
    with pytest.raises(ValueError):  # K-quant columns must be divisible by 256 (Q4KTensor.cs:44-45)
        sm.CudaWeightTensor(ctx, sm.QuantScheme.Q4_K, 8, 100, np.zeros(8 * 100 // 256 * 144 + 144, np.uint8))


@pytest.mark.parametrize("scheme", ["Q4_K", "Q6_K", "Q8_0", "Q4_0"])
@pytest.mark.parametrize("kn", [(2048, 2048), (2048, 5632), (5632, 2048), (4096, 11008)])
def test_full_size_sweep_against_device_dequant(ctx, O, scheme, kn):
    """Op-sweep shapes (K x N) at M = 1, 8, 64: y must equal x . dequant(W)^T (fp64) within 1e-4."""
    import torch

    import smallmind_b200 as sm
    K, N = kn
    sch = getattr(O, scheme)
    g = torch.Generator(device="cuda").manual_seed(K * 7 + N)
    wf = (torch.randn(N * K, generator=g, device="cuda") * 0.02).contiguous()
    bs = 32
    nbytes = {O.Q8_0: N * K, O.Q4_0: N * K // 2, O.Q4_K: N * K // 256 * 144, O.Q6_K: N * K // 256 * 210}[sch]
    data = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    scales = torch.empty(N * K // bs, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    assert sm.lib().sm_quantize(ctx.handle, sch, wf.data_ptr(), N * K, bs, data.data_ptr(), scales.data_ptr()) == 0
    ctx.sync()
    import ctypes as C
    h = C.c_void_p()
    has_sc = sch in (O.Q8_0, O.Q4_0)
    rc = sm.lib().sm_weight_upload_device(ctx.handle, sch, N, K, bs, data.data_ptr(), nbytes,
                                          scales.data_ptr() if has_sc else None, N * K // bs if has_sc else 0,
                                          0, C.byref(h))
    assert rc == 0, sm.last_error()
    deq = torch.empty(N * K, dtype=torch.float32, device="cuda")
    assert sm.lib().sm_dequant(h, deq.data_ptr(), 1) == 0
    for m in (1, 8, 64):
        a = torch.randn(m, K, generator=g, device="cuda")
        y = torch.empty(m, N, device="cuda")
        torch.cuda.synchronize()
        assert sm.lib().sm_matmul(h, a.data_ptr(), y.data_ptr(), m, K, N, 1) == 0
        ctx.sync()
        ref = (a.double() @ deq.view(N, K).double().T)
        assert rel_err(y.cpu().numpy(), ref.cpu().numpy()) <= TOL
    sm.lib().sm_weight_destroy(h)


@pytest.mark.parametrize("scheme", ["Q8_0", "Q4_0"])
@pytest.mark.parametrize("bs,k,n", [(64, 2304, 37), (32, 256, 16), (128, 1024, 300)])
def test_gemv_m1_block_sizes_vs_oracle(ctx, O, scheme, bs, k, n):
    """M = 1 (the int8 tensor-core GEMV for Q8_0 / Q4_0) at scale blocks of 32, 64 and 128."""
    import smallmind_b200 as sm
    sch = getattr(O, scheme)
    t = O.quantize(O.fill_normal(n * k, 91, 0.02), sch, n, k, bs)
    a = np.random.RandomState(bs).randn(1, k).astype(np.float32)
    ref = O.matmul(t, a, 1, k, n, mode=1)
    w = sm.CudaWeightTensor.from_qtensor(ctx, t)
    out = np.empty((1, n), np.float32)
    w.MatMul(a, out, 1, k, n)
    assert rel_err(out, ref) <= TOL
