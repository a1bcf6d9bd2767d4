"""Tensor-parallel bookkeeping on the CPU: the byte slicing of packed weights, the
head / FFN splits, and a world-size-2 gloo run in which each rank applies its
shards of the row-split O and down projections and the all-reduced partial
outputs equal the unsharded projection (MultiHeadAttention.cs:92-93,
GatedMLP.cs:38-40 are the projections split)."""
import os

import numpy as np
import pytest

from smallmind_b200 import tp

CFG = dict(vocab_size=320, hidden=512, n_layers=1, n_heads=8, n_kv_heads=2, head_dim=64, ffn_hidden=1280,
           max_context=32, norm_eps=1e-5, rope_theta=10000.0)


def _schemes(O):
    return dict(wq=O.Q4_K, wk=O.Q4_K, wv=O.Q6_K, wo=O.Q4_K, w_gate=O.Q4_K, w_up=O.Q4_K, w_down=O.Q6_K,
                output=O.Q6_K)


@pytest.mark.parametrize("scheme,bs", [("Q4_K", 256), ("Q6_K", 256), ("Q8_0", 32), ("Q8_0", 64), ("Q4_0", 32)])
def test_slices_dequantize_to_the_same_values(O, scheme, bs):
    rows, cols = 48, 1024
    t = O.quantize(O.fill_normal(rows * cols, 9, 0.02), getattr(O, scheme), rows, cols, bs)
    full = O.dequantize(t).reshape(rows, cols)
    r = tp.slice_rows(t, 5, 29)
    assert np.array_equal(O.dequantize(O.QTensor(r.scheme, r.rows, r.cols, r.data, r.scales, r.block_size))
                          .reshape(24, cols).view(np.uint32), full[5:29].view(np.uint32))
    c = tp.slice_cols(t, 256, 768)
    assert np.array_equal(O.dequantize(O.QTensor(c.scheme, c.rows, c.cols, c.data, c.scales, c.block_size))
                          .reshape(rows, 512).view(np.uint32), full[:, 256:768].view(np.uint32))
    with pytest.raises(ValueError):
        tp.slice_cols(t, 100, 356 if scheme in ("Q4_K", "Q6_K") else 101)


def test_head_and_ffn_splits():
    assert tp.head_ranges(32, 4, 2, 1) == ((16, 32), (2, 4))
    assert tp.head_ranges(32, 4, 8, 3) == ((12, 16), (1, 2))  # two ranks per kv head, each keeps a copy
    with pytest.raises(ValueError):
        tp.head_ranges(32, 4, 3, 0)
    spans = [tp.ffn_range(5632, 4, r) for r in range(4)]
    assert spans[0][0] == 0 and spans[-1][1] == 5632 and all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert all((hi - lo) % 256 == 0 for lo, hi in spans)
    assert tp.even_split(22, 4, 3) == (17, 22)


def test_shard_configs(O):
    host = O.make_model(CFG, _schemes(O), seed=4)
    shards = [tp.shard_model(host, 2, r) for r in range(2)]
    assert [s.cfg["n_heads"] for s in shards] == [4, 4]
    assert [s.cfg["n_kv_heads"] for s in shards] == [1, 1]
    assert sum(s.cfg["ffn_hidden"] for s in shards) == CFG["ffn_hidden"]
    for s in shards:
        L = s.layers[0]
        assert L["wo"].cols == 256 and L["wo"].rows == CFG["hidden"]
        assert L["w_down"].cols == s.cfg["ffn_hidden"] and L["w_gate"].rows == s.cfg["ffn_hidden"]


def _rank_main(rank, world, port, out_path):
    import torch.distributed as dist
    import torch
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from oracle import oracle as O
    host = O.make_model(CFG, _schemes(O), seed=4)
    sh = tp.shard_model(host, world, rank)
    rs = np.random.RandomState(0)
    att = rs.randn(CFG["n_heads"] * CFG["head_dim"]).astype(np.float32)
    act = rs.randn(CFG["ffn_hidden"]).astype(np.float32)
    (q0, q1), _ = tp.head_ranges(CFG["n_heads"], CFG["n_kv_heads"], world, rank)
    f0, f1 = tp.ffn_range(CFG["ffn_hidden"], world, rank)
    L = sh.layers[0]
    wo = O.dequantize(O.QTensor(L["wo"].scheme, L["wo"].rows, L["wo"].cols, L["wo"].data, None, 256))
    wd = O.dequantize(O.QTensor(L["w_down"].scheme, L["w_down"].rows, L["w_down"].cols, L["w_down"].data, None, 256))
    po = wo.reshape(L["wo"].rows, -1).astype(np.float64) @ att[q0 * 64:q1 * 64]
    pd = wd.reshape(L["w_down"].rows, -1).astype(np.float64) @ act[f0:f1]
    t = torch.from_numpy(np.concatenate([po, pd]))
    dist.all_reduce(t)
    if rank == 0:
        full = host.layers[0]
        fo = O.dequantize(full["wo"]).reshape(CFG["hidden"], -1).astype(np.float64) @ att
        fd = O.dequantize(full["w_down"]).reshape(CFG["hidden"], -1).astype(np.float64) @ act
        np.save(out_path, np.stack([t.numpy(), np.concatenate([fo, fd])]))
    dist.destroy_process_group()


def test_gloo_world2_row_split_allreduce(tmp_path):
    import socket

    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = str(tmp_path / "r.npy")
    mp.spawn(_rank_main, args=(2, port, out), nprocs=2, join=True)
    got, ref = np.load(out)
    assert np.abs(got - ref).max() <= 1e-9 * max(1.0, np.abs(ref).max())
