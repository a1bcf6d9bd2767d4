"""Every environment-selected alternate kernel path against the oracle.

Each SMALLMIND_* switch below picks a kernel that is otherwise only the fallback for shapes
the default kernel does not take.  Same tolerances as the default paths:
|y - y_ref| <= 1e-4 * max(max|y_ref|, rms(y_ref)) for GEMV/GEMM and attention, and
logits cosine >= 0.9999 with the same greedy top-1 for the model step.
"""
import numpy as np
import pytest

from conftest import cosine, rel_err

pytestmark = pytest.mark.gpu


def _matmul(ctx, O, scheme, m, k, n, seed):
    import smallmind_b200 as sm
    t = O.quantize(O.fill_normal(n * k, 300 + seed, 0.02), getattr(O, scheme), n, k, 32)
    a = np.random.RandomState(seed).randn(m, k).astype(np.float32)
    ref = O.matmul(t, a, m, k, n, mode=1)
    out = np.empty((m, n), np.float32)
    sm.CudaWeightTensor.from_qtensor(ctx, t).MatMul(a, out, m, k, n)
    return out, ref


@pytest.mark.parametrize("scheme", ["Q4_K", "Q6_K", "Q8_0", "Q4_0"])
@pytest.mark.parametrize("m", [1, 4])
def test_gemv_cuda_core_path(ctx, O, monkeypatch, scheme, m):
    """SMALLMIND_GEMV_MMA=0: the CUDA-core GEMV instead of the integer tensor-core one."""
    monkeypatch.setenv("SMALLMIND_GEMV_MMA", "0")
    out, ref = _matmul(ctx, O, scheme, m, 2048, 640, seed=m)
    assert rel_err(out, ref) <= 1e-4


@pytest.mark.parametrize("scheme", ["Q4_K", "Q6_K", "Q8_0"])
def test_gemm_row_kernel_path(ctx, O, monkeypatch, scheme):
    """SMALLMIND_GEMM_TC=0: the CUDA-core row kernel instead of the tcgen05 GEMM (M >= 16)."""
    monkeypatch.setenv("SMALLMIND_GEMM_TC", "0")
    out, ref = _matmul(ctx, O, scheme, 40, 1024, 384, seed=40)
    assert rel_err(out, ref) <= 1e-4


def test_attention_prefill_cuda_core_path(ctx, O, monkeypatch):
    """SMALLMIND_ATTN_TC=0: the CUDA-core causal prefill kernel."""
    import smallmind_b200 as sm
    monkeypatch.setenv("SMALLMIND_ATTN_TC", "0")
    T, S, nH, nKv, hd = 150, 230, 32, 4, 64
    rs = np.random.RandomState(5)
    q = rs.randn(T, nH * hd).astype(np.float32)
    k = rs.randn(S, nKv * hd).astype(np.float32)
    v = rs.randn(S, nKv * hd).astype(np.float32)
    assert rel_err(sm.attention(ctx, q, k, v, T, S, nH, nKv, hd), O.attention(q, k, v, T, S, nH, nKv, hd)) < 1e-4


def test_attention_decode_split_context_path(ctx, O, monkeypatch):
    """SMALLMIND_ATTN_CLUSTER=0: the three-kernel split-context decode attention."""
    import torch

    import smallmind_b200 as sm
    monkeypatch.setenv("SMALLMIND_ATTN_CLUSTER", "0")
    B, nH, nKv, hd, max_ctx = 5, 32, 4, 64, 700
    rs = np.random.RandomState(9)
    lens = np.array([1, 64, 65, 333, 700], np.int32)
    kc = rs.randn(B, nKv, max_ctx, hd).astype(np.float32)
    vc = rs.randn(B, nKv, max_ctx, hd).astype(np.float32)
    q = rs.randn(B, nH * hd).astype(np.float32)
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, kc, vc))
    dl = torch.from_numpy(lens).cuda()
    out = torch.empty(B, nH * hd, device="cuda")
    torch.cuda.synchronize()
    rc = sm.lib().sm_attention_decode(ctx.handle, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(),
                                      dl.data_ptr(), B, max_ctx, nH, nKv, hd)
    assert rc == 0, sm.last_error()
    ctx.sync()
    got = out.cpu().numpy()
    for b in range(B):
        L = int(lens[b])
        kk = np.ascontiguousarray(kc[b, :, :L].transpose(1, 0, 2).reshape(L, nKv * hd))
        vv = np.ascontiguousarray(vc[b, :, :L].transpose(1, 0, 2).reshape(L, nKv * hd))
        assert rel_err(got[b:b + 1], O.attention(q[b:b + 1], kk, vv, 1, L, nH, nKv, hd)) < 1e-4, b


@pytest.mark.parametrize("env", [{"SMALLMIND_MEGA_MMA": "0"}, {"SMALLMIND_MEGA_SLOTS": "2"},
                                 {"SMALLMIND_MEGA_LOOKAHEAD": "0"}, {"SMALLMIND_CUDA_GRAPHS": "0"}])
def test_one_launch_decode_variants(ctx, O, monkeypatch, env):
    """The one-launch decode kernel with its dp4a GEMV phases (MEGA_MMA=0), a two-slot stage
    ring (MEGA_SLOTS=2), phase-locked staging (MEGA_LOOKAHEAD=0) and without graph capture."""
    import smallmind_b200 as sm
    for k_, v_ in env.items():
        monkeypatch.setenv(k_, v_)
    cfg = dict(vocab_size=640, hidden=512, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=64, ffn_hidden=768,
               max_context=96, norm_eps=1e-5, rope_theta=10000.0)
    schemes = dict(wq=O.Q4_K, wk=O.Q4_K, wv=O.Q6_K, wo=O.Q4_K, w_gate=O.Q4_K, w_up=O.Q4_K, w_down=O.Q6_K,
                   output=O.Q6_K)
    host = O.make_model(cfg, schemes, seed=31)
    model = sm.CudaModel.from_host(ctx, host)
    kv = sm.KVCache(model, 1, 96)
    prompt = np.random.RandomState(4).randint(0, cfg["vocab_size"], 70).astype(np.int32)
    tok, _ = kv.prefill(0, prompt)
    dec = O.KVDecoder(host)
    ref = dec.step(prompt)
    assert tok == int(np.argmax(ref))
    for _ in range(4):
        n0 = ctx.launch_count()
        toks, lg = kv.decode([0], [tok])
        assert ctx.launch_count() - n0 <= 2  # the one-launch kernel ran
        ref = dec.step([tok])
        assert cosine(lg[0], ref) >= 0.9999 and int(toks[0]) == int(np.argmax(ref))
        tok = int(toks[0])
