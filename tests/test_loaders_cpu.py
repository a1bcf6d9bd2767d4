"""SMQ container and GGUF raw-block passthrough (host side, no GPU).

The ggml -> reference block conversion is checked bit-exactly: ggml's published
block formulas (tests/gguf_fixture.py) against the oracle's dequantization of
the converted bytes (Q4KTensor.cs:129-147, Q6KTensor.cs:105-124, Q8Tensor.cs:151,
Q4Tensor.cs:140-179).  The SMQ layout checks follow SmqFormat.cs:15-25 and
SmqWriter.cs:129-170.
"""
import json
import os
import struct
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(__file__))
import gguf_fixture as G  # noqa: E402


def _ld():
    from smallmind_b200 import loaders
    return loaders


def _tensors(O):
    L = _ld()
    rs = np.random.RandomState(0)
    out = [L.HostTensor("norm.weight", L.QuantScheme.F32, [64], rs.randn(64).astype(np.float32).view(np.uint8))]
    for name, sch, rows, cols, bs in [("q8.weight", O.Q8_0, 8, 128, 64), ("q4.weight", O.Q4_0, 6, 96, 32),
                                      ("q41.weight", O.Q4_1, 5, 64, 32), ("q50.weight", O.Q5_0, 3, 96, 32),
                                      ("q4k.weight", O.Q4_K, 4, 512, 256), ("q6k.weight", O.Q6_K, 3, 256, 256)]:
        t = O.quantize(rs.randn(rows * cols).astype(np.float32), sch, rows, cols, bs)
        sc = None if t.scales is None else np.asarray(t.scales, np.float32)
        out.append(L.HostTensor(name, sch, [rows, cols], np.asarray(t.data).view(np.uint8).copy(), sc,
                                bs if sch in (O.Q8_0, O.Q4_0, O.Q4_1, O.Q5_0) else 256))
    return out


def test_smq_round_trip_and_layout(O, tmp_path):
    L = _ld()
    ts = _tensors(O)
    meta = {"llama.block_count": 2, "general.name": "x"}
    path = tmp_path / "m.smq"
    n = L.smq_write(path, ts, meta)
    raw = path.read_bytes()
    assert len(raw) == n
    # header: magic, version 1, header size 32, tensor count, metadata length, 8 reserved bytes
    assert raw[:8] == b"SMQv0001"
    ver, hs, cnt, mlen, res = struct.unpack_from("<IIIIQ", raw, 8)
    assert (ver, hs, cnt, res) == (1, 32, len(ts), 0)
    assert json.loads(raw[32:32 + mlen]) == meta
    # directory of 156-byte entries; data then aux, in directory order, right after it
    pos = 32 + mlen
    expect = pos + 156 * len(ts)
    for t in ts:
        name = raw[pos:pos + 64].rstrip(b"\0").decode()
        dtype, rank = struct.unpack_from("<Ii", raw, pos + 64)
        doff, dl, aoff, al = struct.unpack_from("<QQQQ", raw, pos + 64 + 44)
        assert (name, dtype, rank) == (t.name, int(t.scheme), len(t.dims))
        assert doff == expect
        expect += dl
        if al:
            assert aoff == expect
            expect += al
        pos += 156
    assert expect == len(raw)
    back = L.smq_read(path)
    assert back.metadata == meta
    for t in ts:
        b = back.tensors[t.name]
        assert (b.scheme, b.dims, b.block_size) == (t.scheme, t.dims, t.block_size)
        assert np.array_equal(b.data, t.data)
        if t.scales is not None:
            assert np.array_equal(b.scales, t.scales)


def test_smq_rejects_malformed(O, tmp_path):
    L = _ld()
    ts = _tensors(O)
    raw = bytearray()
    p = tmp_path / "m.smq"
    L.smq_write(p, ts)
    raw = bytearray(p.read_bytes())
    bad = bytearray(raw)
    bad[:8] = b"SMQv0002"
    with pytest.raises(ValueError):
        L.smq_read(bytes(bad))
    bad = bytearray(raw)
    struct.pack_into("<I", bad, 8, 2)  # version
    with pytest.raises(ValueError):
        L.smq_read(bytes(bad))
    with pytest.raises(ValueError):  # truncated data
        L.smq_read(bytes(raw[:-10]))
    bad = bytearray(raw)
    struct.pack_into("<Q", bad, 32 + 64 + 44 + 8, 3)  # first tensor's data length
    with pytest.raises(ValueError):
        L.smq_read(bytes(bad))


@pytest.mark.parametrize("ttype,scheme", [(G.Q8_0, "Q8_0"), (G.Q4_0, "Q4_0"), (G.Q4_1, "Q4_1"), (G.Q5_0, "Q5_0"),
                                          (G.Q4_K, "Q4_K"), (G.Q6_K, "Q6_K")])
def test_ggml_blocks_convert_bit_exact(O, ttype, scheme):
    """Every weight decodes to the same fp32 value after the layout conversion."""
    L = _ld()
    rs = np.random.RandomState(ttype)
    rows, cols = 6, 512
    raw = G.random_blocks(ttype, rows * cols, rs)
    g = L.GgufFile(3, {}, [], 0, bytes(raw))
    t = L.gguf_tensor_to_host(g, L.GgufTensorInfo("w", [cols, rows], ttype, 0))
    qt = O.QTensor(getattr(O, scheme), rows, cols, t.data, t.scales, t.block_size or 256)
    got = O.dequantize(qt).reshape(-1)
    want = G.ggml_dequant(ttype, raw)
    assert got.dtype == np.float32
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("ttype", [G.Q4_1, G.Q5_0])
def test_rows_split_of_block32_pairs(O, ttype):
    """A merged Q|K|V of Q4_1 / Q5_0 splits by rows into tensors that decode to
    the same rows (their second per-block field travels with the rows)."""
    L = _ld()
    rs = np.random.RandomState(3)
    rows, cols = 12, 96
    raw = G.random_blocks(ttype, rows * cols, rs)
    g = L.GgufFile(3, {}, [], 0, bytes(raw))
    t = L.gguf_tensor_to_host(g, L.GgufTensorInfo("w", [cols, rows], ttype, 0))
    full = O.dequantize(O.QTensor(int(t.scheme), rows, cols, t.data, t.scales, 32))
    for r0, r1 in [(0, 5), (5, 9), (9, 12)]:
        p = L._rows(t, r0, r1)
        got = O.dequantize(O.QTensor(int(p.scheme), r1 - r0, cols, p.data, p.scales, 32))
        assert np.array_equal(got.view(np.uint32), full[r0:r1].view(np.uint32))


def test_gguf_read_and_import_to_smq(O, tmp_path):
    L = _ld()
    cfg = dict(vocab_size=64, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_hidden=512,
               max_context=32)
    gp, sp = tmp_path / "m.gguf", tmp_path / "m.smq"
    ts = G.tiny_llama_gguf(gp, cfg)
    g = L.gguf_read(gp)
    assert g.version == 3
    assert g.metadata["llama.block_count"] == 2 and g.metadata["tokenizer.ggml.tokens"][3] == "t3"
    assert g.data_offset % 32 == 0
    assert [t.name for t in g.tensors] == list(ts)
    for t in g.tensors:
        ttype, raw, dims = ts[t.name]
        assert (t.type, t.dims) == (ttype, dims)
        assert np.array_equal(g.tensor_bytes(t), raw)
    c = L.config_from_metadata(g.metadata, {t.name: L.gguf_tensor_to_host(g, t) for t in g.tensors})
    assert c == dict(cfg, norm_eps=c["norm_eps"], rope_theta=10000.0)
    L.gguf_import_to_smq(gp, sp)
    s = L.smq_read(sp)
    assert s.metadata["converted_from"] == "GGUF" and s.metadata["llama.embedding_length"] == 256
    for t in g.tensors:
        h = L.gguf_tensor_to_host(g, t)
        b = s.tensors[t.name]
        assert (b.scheme, b.dims) == (h.scheme, h.dims)
        assert np.array_equal(b.data, h.data)
    emb = s.tensors["token_embd.weight"]
    assert emb.scheme == L.QuantScheme.F32 and emb.dims == [64, 256]


def test_gguf_rejects_malformed(tmp_path):
    L = _ld()
    with pytest.raises(ValueError):
        L.gguf_read(b"GGML" + bytes(20))
    with pytest.raises(ValueError):
        L.gguf_read(b"GGUF" + struct.pack("<IQQ", 1, 0, 0))
