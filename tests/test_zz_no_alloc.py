"""The allocation-free decode attention entry point (sm_attention_decode_noalloc).

It exists for callers that cannot let the library allocate device memory, such
as a host that reserved its whole device budget up front.  It must match the
oracle's attention (MultiHeadAttention.cs:206-317 decode, FastExp softmax) and
sm_attention_decode on consecutive calls, both for shapes the scratch-free
cluster kernel takes and for shapes only the split-context kernels on the shared
static scratch serve (16 q heads per kv head).  This file is named to be
collected last.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _inputs(seed, B, nH, nKv, hd, max_ctx):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, nH * hd, generator=g, device="cuda")
    kc = torch.randn(B, nKv, max_ctx, hd, generator=g, device="cuda")
    vc = torch.randn(B, nKv, max_ctx, hd, generator=g, device="cuda")
    lens = torch.randint(1, max_ctx + 1, (B,), generator=g, device="cuda", dtype=torch.int32)
    return q, kc, vc, lens


def _oracle_rows(O, q, kc, vc, lens, nH, nKv, hd):
    q, kc, vc, lens = (t.cpu().numpy() for t in (q, kc, vc, lens))
    rows = []
    for b in range(q.shape[0]):
        L = int(lens[b])
        kk = np.ascontiguousarray(kc[b, :, :L].transpose(1, 0, 2).reshape(L, nKv * hd))
        vv = np.ascontiguousarray(vc[b, :, :L].transpose(1, 0, 2).reshape(L, nKv * hd))
        rows.append(O.attention(q[b:b + 1], kk, vv, 1, L, nH, nKv, hd))
    return np.concatenate(rows)


@pytest.mark.parametrize("nH,nKv", [(32, 4), (32, 2)])  # cluster kernel; scratch kernels only (group 16)
def test_noalloc_matches_oracle_and_allocating_entry_point_twice(ctx, O, nH, nKv):
    import torch

    import smallmind_b200 as sm
    L = sm.lib()
    B, hd, max_ctx = 6, 64, 1024
    for call, seed in enumerate((1, 2)):  # two calls in a row; the second finds the first's scratch contents
        q, kc, vc, lens = _inputs(seed, B, nH, nKv, hd, max_ctx)
        if call == 1:
            lens[0] = 3  # much shorter than the previous call's rows: stale scratch must not leak in
        ref = torch.empty(B, nH * hd, device="cuda")
        got = torch.full((B, nH * hd), float("nan"), device="cuda")
        torch.cuda.synchronize()
        rc = L.sm_attention_decode(ctx.handle, q.data_ptr(), kc.data_ptr(), vc.data_ptr(), ref.data_ptr(),
                                   lens.data_ptr(), B, max_ctx, nH, nKv, hd)
        assert rc == 0, sm.last_error()
        rc = L.sm_attention_decode_noalloc(ctx.handle, q.data_ptr(), kc.data_ptr(), vc.data_ptr(), got.data_ptr(),
                                           lens.data_ptr(), B, max_ctx, nH, nKv, hd)
        assert rc == 0, sm.last_error()
        ctx.sync()
        g, r = got.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(g).all()
        assert rel_err(g, r) < 1e-4
        assert rel_err(g, _oracle_rows(O, q, kc, vc, lens, nH, nKv, hd)) < 1e-4


def test_noalloc_rejects_sizes_beyond_the_static_scratch(ctx):
    import smallmind_b200 as sm
    L = sm.lib()
    # 16 q heads per kv head (not the cluster kernel's shape): 64 sequences x 32 heads x 4096
    # positions needs ~33 M floats > 16 MiB, refused on the host before any launch
    dummy = C.c_void_p(1)
    rc = L.sm_attention_decode_noalloc(ctx.handle, dummy, dummy, dummy, dummy, dummy, 64, 4096, 32, 2, 64)
    assert rc == -2
    assert "16 MiB" in sm.last_error()
