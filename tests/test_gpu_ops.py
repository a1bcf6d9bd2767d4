"""GPU parity of the block-level ops (RMSNorm, RoPE, SiLU-gate, attention) against the oracle."""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


def test_rmsnorm(ctx, O):
    import smallmind_b200 as sm
    for rows, F in [(1, 3), (2, 3), (5, 576), (3, 2048)]:
        x = np.random.RandomState(F).randn(rows, F).astype(np.float32)
        g = np.random.RandomState(1).rand(F).astype(np.float32) + 0.5
        y = sm.rmsnorm(ctx, x, g)
        assert rel_err(y, O.rmsnorm(x, g)) < 1e-6
    assert np.all(sm.rmsnorm(ctx, np.zeros((1, 3), np.float32), np.ones(3, np.float32)) == 0)


def test_rope_bit_exact(ctx, O):
    import smallmind_b200 as sm
    nH, hd, max_seq = 4, 64, 2048
    s, c = O.rope_tables(max_seq, hd)
    pos = np.array([0, 1, 7, 100, 2047], np.int32)
    x = np.random.RandomState(0).randn(pos.size, nH * hd).astype(np.float32)
    y = sm.rope(ctx, x, nH, hd, pos, max_seq=max_seq)
    for r, p in enumerate(pos):
        assert np.array_equal(y[r], O.rope_apply(x[r], nH, hd, int(p), s, c))
    assert np.array_equal(y[0], x[0])  # identity at position 0 (RotaryEmbeddingTests.cs:33-61)
    with pytest.raises(ValueError):  # RotaryEmbeddingTests.cs:163-173: position beyond maxSeqLen throws
        sm.rope(ctx, x[:1], nH, hd, [11], max_seq=10)
    with pytest.raises(ValueError):  # odd head dim throws (:24-30)
        sm.rope(ctx, x[:1, :63], 1, 63, [0], max_seq=10)


def test_silu_mul(ctx, O):
    import smallmind_b200 as sm
    g = (np.random.RandomState(0).randn(5632) * 8).astype(np.float32)
    u = np.random.RandomState(1).randn(5632).astype(np.float32)
    assert rel_err(sm.silu_mul(ctx, g, u), O.silu_mul(g, u)) < 1e-6


@pytest.mark.parametrize("T,S,nH,nKv", [(1, 1, 4, 2), (1, 300, 32, 4), (5, 5, 9, 3), (70, 70, 4, 4),
                                          (33, 130, 8, 2), (128, 128, 32, 4), (129, 129, 4, 1), (300, 300, 32, 4),
                                          (200, 700, 8, 2), (640, 640, 32, 4)])
def test_attention_prefill(ctx, O, T, S, nH, nKv):
    import smallmind_b200 as sm
    hd = 64
    rs = np.random.RandomState(T * 1000 + S)
    q = rs.randn(T, nH * hd).astype(np.float32)
    k = rs.randn(S, nKv * hd).astype(np.float32)
    v = rs.randn(S, nKv * hd).astype(np.float32)
    ref = O.attention(q, k, v, T, S, nH, nKv, hd)
    out = sm.attention(ctx, q, k, v, T, S, nH, nKv, hd)
    assert rel_err(out, ref) < 1e-4


@pytest.mark.parametrize("B", [8, 32, 64])
def test_attention_decode_batch_cluster_sizes(ctx, O, B):
    """Batches that select 8, 2 and 1 CTAs per (sequence, kv head), short ragged contexts."""
    import torch

    import smallmind_b200 as sm
    nH, nKv, hd, max_ctx = 32, 4, 64, 256
    rs = np.random.RandomState(B)
    lens = rs.randint(1, max_ctx + 1, B).astype(np.int32)
    lens[0] = 1
    lens[-1] = max_ctx
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
        ref = O.attention(q[b:b + 1], kk, vv, 1, L, nH, nKv, hd)
        assert rel_err(got[b:b + 1], ref) < 1e-4, b


def test_attention_decode_ragged_batch(ctx, O):
    """16 sequences, lengths U[256, 2048], head-major cache."""
    import torch

    import smallmind_b200 as sm
    B, nH, nKv, hd, max_ctx = 16, 32, 4, 64, 2048
    rs = np.random.RandomState(3)
    lens = rs.randint(256, 2049, B).astype(np.int32)
    lens[0] = 1
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
        ref = O.attention(q[b:b + 1], kk, vv, 1, L, nH, nKv, hd)
        assert rel_err(got[b:b + 1], ref) < 1e-4, b
