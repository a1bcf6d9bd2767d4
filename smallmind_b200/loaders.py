"""Model files -> device weights: the SMQ container and GGUF raw-block passthrough.

SMQ (SmallMind Quantized, version 1) follows the reference container
(src/SmallMind.Quantization/IO/Smq/SmqFormat.cs:15-25, SmqWriter.cs:37-100,
SmqReader.cs:30-230): a 32-byte header (magic ``SMQv0001``, version, header
size, tensor count, metadata JSON length, 8 reserved bytes), the metadata JSON,
a directory of 156-byte entries (64-byte name, data type, rank, 8 dimensions,
block size, data offset/length, aux offset/length, 16 reserved bytes), then each
tensor's data followed by its aux blob.  The reference writes F32, Q8_0 (int8
codes + fp32 scales per block of the linear index) and Q4_0 (nibbles packed by
global index + fp32 scales).  This module also writes and reads Q4_K and Q6_K
entries: data = the tensor's blocks in the reference byte layout (144 / 210
bytes per 256 elements, Q4KTensor.cs:84-94, Q6KTensor.cs:86-95), no aux.

GGUF (versions 2 and 3, as GgufReader.cs:39-120 reads them) holds ggml-layout
blocks.  Q8_0 / Q4_0 / Q4_1 / Q5_0 / Q4_K / Q6_K blocks are converted to the reference byte
layouts without any requantization (the conversion only moves bits: every
weight decodes to the same value), then uploaded with ``sm_weight_upload``.
F32 / F16 tensors (norms, embeddings) are read as fp32.

Tensor names follow the reference (TransformerModel.cs:545-680) and llama.cpp:
``token_embd.weight``, ``blk.{l}.attn_norm.weight``, ``blk.{l}.attn_q|k|v.weight``
or the merged ``blk.{l}.attn_qkv.weight``, ``blk.{l}.attn_output.weight``,
``blk.{l}.ffn_norm.weight``, ``blk.{l}.ffn_gate|up|down.weight``,
``output_norm.weight``, ``output.weight`` (absent: tied to the embedding).
"""
from __future__ import annotations

import io
import json
import struct
from dataclasses import dataclass, field

import numpy as np

from .api import CudaContext, CudaModel, CudaWeightTensor, QuantScheme

# ---------------------------------------------------------------- shared tensor record


@dataclass
class HostTensor:
    """One tensor as stored: reference-layout bytes (``data``), fp32 block scales
    (``scales``, Q8_0 / Q4_0) and its shape (rows = out features, cols = in)."""
    name: str
    scheme: int
    dims: list
    data: np.ndarray  # uint8 (F32: float32 viewed as bytes)
    scales: np.ndarray | None = None
    block_size: int = 0

    @property
    def rows(self) -> int:
        return int(self.dims[0]) if len(self.dims) > 1 else 1

    @property
    def cols(self) -> int:
        return int(self.dims[-1]) if len(self.dims) > 1 else int(self.dims[0])

    def floats(self) -> np.ndarray:
        if self.scheme != QuantScheme.F32:
            raise ValueError(f"{self.name}: not an F32 tensor")
        return self.data.view(np.float32)


# ---------------------------------------------------------------- SMQ

SMQ_MAGIC = b"SMQv0001"
SMQ_VERSION = 1
SMQ_HEADER = 32
SMQ_ENTRY = 156
KQ_BLOCK_BYTES = {int(QuantScheme.Q4_K): 144, int(QuantScheme.Q6_K): 210}


def _smq_data_aux_len(t: HostTensor) -> tuple[int, int]:
    n = int(np.prod(t.dims))
    s = int(t.scheme)
    if s == QuantScheme.F32:
        return 4 * n, 0
    if s == QuantScheme.Q8_0:
        return n, 4 * ((n + t.block_size - 1) // t.block_size)
    if s == QuantScheme.Q4_0:
        return (n + 1) // 2, 4 * ((n + t.block_size - 1) // t.block_size)
    if s == QuantScheme.Q4_1:  # nibbles; aux = fp32 scales then fp32 mins
        return (n + 1) // 2, 8 * ((n + 31) // 32)
    if s == QuantScheme.Q5_0:  # low nibbles then a 32-bit high-bit word per block; aux = fp32 scales
        return (n + 1) // 2 + 4 * ((n + 31) // 32), 4 * ((n + 31) // 32)
    if s in KQ_BLOCK_BYTES:
        if n % 256:
            raise ValueError(f"{t.name}: K-quant tensors need a multiple of 256 elements")
        return n // 256 * KQ_BLOCK_BYTES[s], 0
    raise ValueError(f"{t.name}: unsupported data type {s}")


def smq_write(path_or_stream, tensors: list[HostTensor], metadata: dict | None = None) -> int:
    """SmqWriter.WriteModel: returns the bytes written."""
    meta = json.dumps(metadata).encode() if metadata else b""
    entries = []
    off = SMQ_HEADER + len(meta) + SMQ_ENTRY * len(tensors)
    for t in tensors:
        dl, al = _smq_data_aux_len(t)
        if t.data.nbytes != dl:
            raise ValueError(f"{t.name}: data is {t.data.nbytes} bytes, expected {dl}")
        if al and (t.scales is None or t.scales.nbytes != al):
            raise ValueError(f"{t.name}: scales must be {al} bytes")
        entries.append((t, off, dl, off + dl if al else 0, al))
        off += dl + al
    buf = io.BytesIO()
    buf.write(SMQ_MAGIC)
    buf.write(struct.pack("<IIIIQ", SMQ_VERSION, SMQ_HEADER, len(tensors), len(meta), 0))
    buf.write(meta)
    for t, doff, dl, aoff, al in entries:
        name = t.name.encode()
        if len(name) > 64:
            raise ValueError(f"tensor name too long: {t.name}")
        dims = list(t.dims) + [0] * (8 - len(t.dims))
        buf.write(name + b"\0" * (64 - len(name)))
        buf.write(struct.pack("<Ii8iIQQQQQQ", int(t.scheme), len(t.dims), *dims, t.block_size, doff, dl, aoff, al, 0, 0))
    for t, _, _, _, al in entries:
        buf.write(t.data.tobytes())
        if al:
            buf.write(np.ascontiguousarray(t.scales, np.float32).tobytes())
    out = buf.getvalue()
    if hasattr(path_or_stream, "write"):
        path_or_stream.write(out)
    else:
        with open(path_or_stream, "wb") as f:
            f.write(out)
    return len(out)


@dataclass
class SmqFile:
    metadata: dict = field(default_factory=dict)
    tensors: dict = field(default_factory=dict)  # name -> HostTensor


def smq_read(path_or_bytes) -> SmqFile:
    """SmqReader.ReadHeader + LoadAllTensors, with the reader's checks
    (magic, version, header size, rank 0..8, positive dimensions, data and aux
    lengths of the data type): ``ValueError`` on a malformed file."""
    raw = path_or_bytes if isinstance(path_or_bytes, (bytes, bytearray)) else open(path_or_bytes, "rb").read()
    mv = memoryview(raw)
    if len(raw) < SMQ_HEADER or bytes(mv[:8]) != SMQ_MAGIC:
        raise ValueError(f"invalid SMQ magic: {bytes(mv[:8])!r}")
    version, hsize, count, mlen, _ = struct.unpack_from("<IIIIQ", raw, 8)
    if version != SMQ_VERSION:
        raise ValueError(f"unsupported SMQ version {version}")
    if hsize != SMQ_HEADER:
        raise ValueError(f"invalid SMQ header size {hsize}")
    pos = SMQ_HEADER
    meta = json.loads(bytes(mv[pos:pos + mlen]).decode()) if mlen else {}
    pos += mlen
    f = SmqFile(metadata=meta)
    for _ in range(count):
        name = bytes(mv[pos:pos + 64]).split(b"\0", 1)[0].decode()
        vals = struct.unpack_from("<Ii8iIQQQQQQ", raw, pos + 64)
        dtype, rank, dims8, bs = vals[0], vals[1], vals[2:10], vals[10]
        doff, dl, aoff, al = vals[11:15]
        pos += SMQ_ENTRY
        if not 0 <= rank <= 8:
            raise ValueError(f"{name}: invalid rank {rank}")
        dims = list(dims8[:rank])
        if any(d <= 0 for d in dims):
            raise ValueError(f"{name}: invalid dimensions {dims}")
        t = HostTensor(name, dtype, dims, np.frombuffer(raw, np.uint8, dl, doff).copy(), None, bs)
        edl, eal = _smq_data_aux_len(t)
        if dl != edl or al != eal:
            raise ValueError(f"{name}: data/aux length {dl}/{al}, expected {edl}/{eal}")
        if doff + dl > len(raw) or (al and aoff + al > len(raw)):
            raise ValueError(f"{name}: data past the end of the file")
        if al:
            t.scales = np.frombuffer(raw, np.float32, al // 4, aoff).copy()
        f.tensors[name] = t
    return f


# ---------------------------------------------------------------- GGUF

GGUF_MAGIC = b"GGUF"
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1, GGML_Q5_0, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K = 0, 1, 2, 3, 6, 8, 12, 14
GGML_BLOCK = {GGML_Q4_0: (32, 18), GGML_Q4_1: (32, 20), GGML_Q5_0: (32, 22), GGML_Q8_0: (32, 34),
              GGML_Q4_K: (256, 144), GGML_Q6_K: (256, 210)}
# value types (GgufValueType.cs): fixed-size scalars -> struct code
_GGUF_SCALAR = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}
GGUF_STRING, GGUF_ARRAY = 8, 9


@dataclass
class GgufTensorInfo:
    name: str
    dims: list  # ggml order: dims[0] is the fastest-varying (columns)
    type: int
    offset: int  # from the start of the data section


@dataclass
class GgufFile:
    version: int
    metadata: dict
    tensors: list
    data_offset: int
    raw: bytes

    def tensor_bytes(self, t: GgufTensorInfo) -> np.ndarray:
        n = int(np.prod(t.dims))
        if t.type == GGML_F32:
            nb = 4 * n
        elif t.type == GGML_F16:
            nb = 2 * n
        elif t.type in GGML_BLOCK:
            be, bb = GGML_BLOCK[t.type]
            if n % be:
                raise ValueError(f"{t.name}: {n} elements is not a whole number of blocks")
            nb = n // be * bb
        else:
            raise ValueError(f"{t.name}: unsupported ggml type {t.type}")
        start = self.data_offset + t.offset
        if start + nb > len(self.raw):
            raise ValueError(f"{t.name}: data past the end of the file")
        return np.frombuffer(self.raw, np.uint8, nb, start)


def gguf_read(path_or_bytes) -> GgufFile:
    """GgufReader.ReadModelInfo: header, key/value metadata, tensor directory and
    the aligned start of the data section (general.alignment, default 32)."""
    raw = path_or_bytes if isinstance(path_or_bytes, (bytes, bytearray)) else open(path_or_bytes, "rb").read()
    if raw[:4] != GGUF_MAGIC:
        raise ValueError(f"invalid GGUF magic: {raw[:4]!r}")
    version, = struct.unpack_from("<I", raw, 4)
    if version not in (2, 3):
        raise ValueError(f"unsupported GGUF version {version}")
    n_t, n_kv = struct.unpack_from("<QQ", raw, 8)
    pos = 24

    def rstr():
        nonlocal pos
        n, = struct.unpack_from("<Q", raw, pos)
        s = raw[pos + 8:pos + 8 + n].decode("utf-8", errors="replace")
        pos += 8 + n
        return s

    def rval(vt):
        nonlocal pos
        if vt == GGUF_STRING:
            return rstr()
        if vt == GGUF_ARRAY:
            et, cnt = struct.unpack_from("<IQ", raw, pos)
            pos += 12
            return [rval(et) for _ in range(cnt)]
        code = _GGUF_SCALAR.get(vt)
        if code is None:
            raise ValueError(f"unknown GGUF value type {vt}")
        v, = struct.unpack_from("<" + code, raw, pos)
        pos += struct.calcsize(code)
        return v

    meta = {}
    for _ in range(n_kv):
        k = rstr()
        vt, = struct.unpack_from("<I", raw, pos)
        pos += 4
        meta[k] = rval(vt)
    infos = []
    for _ in range(n_t):
        name = rstr()
        nd, = struct.unpack_from("<I", raw, pos)
        dims = list(struct.unpack_from("<" + "Q" * nd, raw, pos + 4))
        ttype, off = struct.unpack_from("<IQ", raw, pos + 4 + 8 * nd)
        pos += 4 + 8 * nd + 12
        infos.append(GgufTensorInfo(name, dims, ttype, off))
    align = int(meta.get("general.alignment", 32))
    data_off = (pos + align - 1) // align * align
    return GgufFile(version, meta, infos, data_off, bytes(raw))


# ---- ggml block layouts -> reference layouts (bit moves only)

def _f16(b: np.ndarray) -> np.ndarray:
    return b.view(np.float16).astype(np.float32)


def ggml_q8_0_to_ref(raw: np.ndarray, n: int) -> tuple[np.ndarray, np.ndarray]:
    """ggml Q8_0 (fp16 d, 32 int8) -> Q8Tensor codes + fp32 scales, block size 32."""
    b = raw.reshape(-1, 34)
    return np.ascontiguousarray(b[:, 2:]).reshape(-1)[:n], _f16(np.ascontiguousarray(b[:, :2])).reshape(-1)


def ggml_q4_0_to_ref(raw: np.ndarray, n: int) -> tuple[np.ndarray, np.ndarray]:
    """ggml Q4_0 (fp16 d, 16 bytes: element i in the low nibble of byte i, element
    i + 16 in its high nibble, value (nibble - 8) d) -> Q4Tensor: two's-complement
    nibbles packed by global index (even -> low nibble, Q4Tensor.cs:119-129) +
    fp32 scales, block size 32."""
    b = raw.reshape(-1, 18)
    qs = b[:, 2:]
    vals = np.concatenate([(qs & 0xF).astype(np.int16), (qs >> 4).astype(np.int16)], axis=1) - 8  # [blocks][32]
    nib = (vals.reshape(-1) & 0xF).astype(np.uint8)
    packed = nib[0::2] | (nib[1::2] << 4)
    return packed[: (n + 1) // 2], _f16(np.ascontiguousarray(b[:, :2])).reshape(-1)


def _ggml_nibbles_by_index(qs: np.ndarray) -> np.ndarray:
    """ggml's 16 code bytes per block (element i low nibble of byte i, element
    i + 16 high nibble) -> nibbles packed by global index, even element in the
    low nibble (Q4_1Tensor.cs / Q5_0Tensor.cs element order)."""
    v = np.concatenate([qs & 0xF, qs >> 4], axis=1).reshape(-1)
    return (v[0::2] | (v[1::2] << 4)).astype(np.uint8)


def ggml_q4_1_to_ref(raw: np.ndarray, n: int) -> tuple[np.ndarray, np.ndarray]:
    """ggml Q4_1 (fp16 d, fp16 m, 16 code bytes; value q d + m) -> Q4_1Tensor
    nibbles by global index + [fp32 scales | fp32 mins], block size 32."""
    b = raw.reshape(-1, 20)
    d = _f16(np.ascontiguousarray(b[:, 0:2])).reshape(-1)
    m = _f16(np.ascontiguousarray(b[:, 2:4])).reshape(-1)
    return _ggml_nibbles_by_index(b[:, 4:])[: (n + 1) // 2], np.concatenate([d, m])


def ggml_q5_0_to_ref(raw: np.ndarray, n: int) -> tuple[np.ndarray, np.ndarray]:
    """ggml Q5_0 (fp16 d, 32-bit qh with bit i = element i's fifth bit, 16 code
    bytes; value ((lo | hi << 4) - 16) d) -> Q5_0Tensor low nibbles by global
    index followed by the per-block high words, + fp32 scales, block size 32."""
    b = raw.reshape(-1, 22)
    d = _f16(np.ascontiguousarray(b[:, 0:2])).reshape(-1)
    hi = np.ascontiguousarray(b[:, 2:6]).reshape(-1)
    return np.concatenate([_ggml_nibbles_by_index(b[:, 6:])[: (n + 1) // 2], hi]), d


def _ggml_q4k_scale_min(sc: np.ndarray):
    """The 8 six-bit scales and mins of ggml's 12-byte Q4_K field, per block."""
    s = np.empty((sc.shape[0], 8), np.uint8)
    m = np.empty((sc.shape[0], 8), np.uint8)
    for j in range(4):
        s[:, j] = sc[:, j] & 63
        m[:, j] = sc[:, j + 4] & 63
    for j in range(4, 8):
        s[:, j] = (sc[:, j + 4] & 0xF) | ((sc[:, j - 4] >> 6) << 4)
        m[:, j] = (sc[:, j + 4] >> 4) | ((sc[:, j] >> 6) << 4)
    return s, m


def _pack6(v: np.ndarray) -> np.ndarray:
    """8 six-bit values per row -> 6 bytes, least significant bits first."""
    w = np.zeros(v.shape[0], np.uint64)
    for j in range(8):
        w |= v[:, j].astype(np.uint64) << np.uint64(6 * j)
    return np.stack([((w >> np.uint64(8 * i)) & np.uint64(0xFF)).astype(np.uint8) for i in range(6)], axis=1)


def ggml_q4_k_to_ref(raw: np.ndarray) -> np.ndarray:
    """ggml Q4_K -> Q4KTensor bytes (Q4KTensor.cs:84-147): d, dmin as they are;
    scales and mins as 8 six-bit fields each, packed in sequence (bytes 4-9 and
    10-15); codes re-ordered so byte 16 j + i holds elements 32 j + 2 i (low
    nibble) and 32 j + 2 i + 1 (high).  ggml keeps 64-element chunks: byte
    32 c + l holds element 64 c + l (low nibble) and 64 c + 32 + l (high)."""
    b = raw.reshape(-1, 144)
    s, m = _ggml_q4k_scale_min(b[:, 4:16])
    qs = b[:, 16:].reshape(-1, 4, 32)
    q = np.concatenate([qs & 0xF, qs >> 4], axis=2).reshape(-1, 256)  # element order
    codes = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    out = np.concatenate([b[:, :4], _pack6(s), _pack6(m), codes], axis=1)
    return np.ascontiguousarray(out).reshape(-1)


def ggml_q6_k_to_ref(raw: np.ndarray) -> np.ndarray:
    """ggml Q6_K -> Q6KTensor bytes (Q6KTensor.cs:86-124): the 6-bit code of
    element v becomes low nibble ``ql[v / 2]`` (even v low, odd v high) and two
    bits ``qh[v / 4] >> 2 (v % 4)``; the 16 int8 scales and d keep their places.
    ggml: per 128-element half h, for l < 32: ql[64h + l] low/high nibbles are
    elements 128h + l / 128h + 64 + l, ql[64h + 32 + l] elements 128h + 32 + l /
    128h + 96 + l, and qh[32h + l] bits 0-1, 2-3, 4-5, 6-7 are the highs of
    128h + l, + 32 + l, + 64 + l, + 96 + l."""
    b = raw.reshape(-1, 210)
    ql, qh = b[:, :128], b[:, 128:192]
    q = np.empty((b.shape[0], 256), np.uint8)
    for h in range(2):
        l0, l1 = ql[:, 64 * h:64 * h + 32], ql[:, 64 * h + 32:64 * h + 64]
        hh = qh[:, 32 * h:32 * h + 32]
        base = 128 * h
        q[:, base:base + 32] = (l0 & 0xF) | (((hh >> 0) & 3) << 4)
        q[:, base + 32:base + 64] = (l1 & 0xF) | (((hh >> 2) & 3) << 4)
        q[:, base + 64:base + 96] = (l0 >> 4) | (((hh >> 4) & 3) << 4)
        q[:, base + 96:base + 128] = (l1 >> 4) | (((hh >> 6) & 3) << 4)
    rql = (q[:, 0::2] & 0xF) | ((q[:, 1::2] & 0xF) << 4)
    hi = q >> 4
    rqh = hi[:, 0::4] | (hi[:, 1::4] << 2) | (hi[:, 2::4] << 4) | (hi[:, 3::4] << 6)
    out = np.concatenate([rql.astype(np.uint8), rqh.astype(np.uint8), b[:, 192:210]], axis=1)
    return np.ascontiguousarray(out).reshape(-1)


def gguf_tensor_to_host(g: GgufFile, t: GgufTensorInfo) -> HostTensor:
    """One GGUF tensor in the reference layout (rows = dims[1], cols = dims[0])."""
    raw = g.tensor_bytes(t)
    n = int(np.prod(t.dims))
    dims = [int(d) for d in reversed(t.dims)]  # reference order: rows first
    if t.type == GGML_F32:
        return HostTensor(t.name, QuantScheme.F32, dims, raw.copy())
    if t.type == GGML_F16:
        return HostTensor(t.name, QuantScheme.F32, dims, raw.view(np.float16).astype(np.float32).view(np.uint8))
    if t.type == GGML_Q8_0:
        d, s = ggml_q8_0_to_ref(raw, n)
        return HostTensor(t.name, QuantScheme.Q8_0, dims, d, s, 32)
    if t.type == GGML_Q4_0:
        d, s = ggml_q4_0_to_ref(raw, n)
        return HostTensor(t.name, QuantScheme.Q4_0, dims, d, s, 32)
    if t.type == GGML_Q4_1:
        d, s = ggml_q4_1_to_ref(raw, n)
        return HostTensor(t.name, QuantScheme.Q4_1, dims, d, s, 32)
    if t.type == GGML_Q5_0:
        d, s = ggml_q5_0_to_ref(raw, n)
        return HostTensor(t.name, QuantScheme.Q5_0, dims, d, s, 32)
    if t.type == GGML_Q4_K:
        return HostTensor(t.name, QuantScheme.Q4_K, dims, ggml_q4_k_to_ref(raw))
    if t.type == GGML_Q6_K:
        return HostTensor(t.name, QuantScheme.Q6_K, dims, ggml_q6_k_to_ref(raw))
    raise ValueError(f"{t.name}: unsupported ggml type {t.type}")


def gguf_import_to_smq(gguf_path, smq_path) -> int:
    """GgufImporter.ImportToSmq with raw-block passthrough: every tensor keeps
    its quantization (no requantization to another block size) and the llama.*
    architecture keys are carried into the SMQ metadata (GgufImporter.cs:684-727)."""
    g = gguf_read(gguf_path)
    keys = ["general.architecture", "general.name", "general.quantization_version", "general.file_type",
            "llama.context_length", "llama.embedding_length", "llama.block_count", "llama.feed_forward_length",
            "llama.attention.head_count", "llama.attention.head_count_kv", "llama.rope.dimension_count",
            "llama.rope.freq_base", "llama.attention.layer_norm_rms_epsilon", "llama.vocab_size"]
    meta = {k: g.metadata[k] for k in keys if k in g.metadata}
    meta["converted_from"] = "GGUF"
    return smq_write(smq_path, [gguf_tensor_to_host(g, t) for t in g.tensors], meta)


# ---------------------------------------------------------------- model loading

def config_from_metadata(meta: dict, tensors: dict, max_context: int | None = None) -> dict:
    """ModelConfig (LLaMA) from the llama.* keys, with the shapes as fallback."""
    emb = tensors["token_embd.weight"]
    H = int(meta.get("llama.embedding_length", emb.cols))
    n_heads = int(meta["llama.attention.head_count"])
    L = int(meta.get("llama.block_count", sum(1 for k in tensors if k.endswith(".attn_norm.weight"))))
    ffn = int(meta.get("llama.feed_forward_length", tensors["blk.0.ffn_gate.weight"].rows))
    return dict(vocab_size=int(meta.get("llama.vocab_size", emb.rows)), hidden=H, n_layers=L, n_heads=n_heads,
                n_kv_heads=int(meta.get("llama.attention.head_count_kv", n_heads)), head_dim=H // n_heads,
                ffn_hidden=ffn, max_context=int(max_context or meta.get("llama.context_length", 2048)),
                norm_eps=float(meta.get("llama.attention.layer_norm_rms_epsilon", 1e-5)),
                rope_theta=float(meta.get("llama.rope.freq_base", 10000.0)))


def _rows(t: HostTensor, r0: int, r1: int) -> HostTensor:
    """Rows [r0, r1) of a weight whose rows are whole blocks (a merged Q|K|V split)."""
    if t.scheme in (QuantScheme.Q4_1, QuantScheme.Q5_0):
        if t.cols % 32:
            raise ValueError(f"{t.name}: rows are not whole blocks")
        nb, bpr, lo = t.rows * t.cols // 32, t.cols // 32, t.rows * t.cols // 2
        data = t.data[r0 * t.cols // 2:r1 * t.cols // 2]
        if t.scheme == QuantScheme.Q5_0:
            sc = t.scales[r0 * bpr:r1 * bpr]
            data = np.concatenate([data, t.data[lo + 4 * r0 * bpr:lo + 4 * r1 * bpr]])
        else:
            sc = np.concatenate([t.scales[r0 * bpr:r1 * bpr], t.scales[nb + r0 * bpr:nb + r1 * bpr]])
        return HostTensor(t.name, t.scheme, [r1 - r0, t.cols], data, sc, 32)
    per = t.data.nbytes // t.rows
    if per * t.rows != t.data.nbytes:
        raise ValueError(f"{t.name}: rows are not whole blocks")
    sc = None
    if t.scales is not None:
        spr = t.scales.size // t.rows
        if spr * t.rows != t.scales.size:
            raise ValueError(f"{t.name}: rows are not whole scale blocks")
        sc = t.scales[r0 * spr:r1 * spr]
    return HostTensor(t.name, t.scheme, [r1 - r0, t.cols], t.data[r0 * per:r1 * per], sc, t.block_size)


def _upload(ctx: CudaContext, t: HostTensor) -> CudaWeightTensor:
    if t.scheme == QuantScheme.F32:  # F32 / F16 linear weights as fp32 rows (GgufImporter converts F16 to F32)
        return CudaWeightTensor(ctx, QuantScheme.F32, t.rows, t.cols, t.data, None, 1)
    return CudaWeightTensor(ctx, t.scheme, t.rows, t.cols, t.data, t.scales, t.block_size or 32)


def _vector(ctx: CudaContext, t: HostTensor) -> np.ndarray:
    """fp32 values of a norm / embedding tensor (quantized ones dequantized on the device)."""
    if t.scheme == QuantScheme.F32:
        return t.floats()
    w = _upload(ctx, t)
    try:
        return w.ToFloat32()
    finally:
        w.close()


def build_model(ctx: CudaContext, tensors: dict, cfg: dict) -> CudaModel:
    """SmqModelLoader.LoadFromSmq for the LLaMA ModelConfig: every quantized
    linear stays quantized on the device; norms and the embedding as fp32."""
    m = CudaModel(ctx, cfg)
    H = cfg["hidden"]
    qd, kd = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]
    m.set_vector(0, "token_embd", _vector(ctx, tensors["token_embd.weight"]))
    m.set_vector(0, "out_norm", _vector(ctx, tensors["output_norm.weight"]))
    out = tensors.get("output.weight", tensors["token_embd.weight"])  # tied embeddings
    m.set_weight(0, "output", _upload(ctx, out))
    for li in range(cfg["n_layers"]):
        p = f"blk.{li}."
        m.set_vector(li, "attn_norm", _vector(ctx, tensors[p + "attn_norm.weight"]))
        m.set_vector(li, "ffn_norm", _vector(ctx, tensors[p + "ffn_norm.weight"]))
        if p + "attn_qkv.weight" in tensors:
            qkv = tensors[p + "attn_qkv.weight"]
            parts = {"wq": _rows(qkv, 0, qd), "wk": _rows(qkv, qd, qd + kd), "wv": _rows(qkv, qd + kd, qd + 2 * kd)}
        else:
            parts = {"wq": tensors[p + "attn_q.weight"], "wk": tensors[p + "attn_k.weight"],
                     "wv": tensors[p + "attn_v.weight"]}
        parts.update(wo=tensors[p + "attn_output.weight"], w_gate=tensors[p + "ffn_gate.weight"],
                     w_up=tensors[p + "ffn_up.weight"], w_down=tensors[p + "ffn_down.weight"])
        fan_in = {"wq": H, "wk": H, "wv": H, "wo": qd, "w_gate": H, "w_up": H, "w_down": cfg["ffn_hidden"]}
        for role, t in parts.items():
            if t.cols != fan_in[role]:
                raise ValueError(f"{p}{role}: {t.cols} inputs, the config needs {fan_in[role]}")
            m.set_weight(li, role, _upload(ctx, t))
    m.finalize()
    return m


def load_smq_model(ctx: CudaContext, path, cfg: dict | None = None, max_context: int | None = None):
    """(CudaModel, metadata) from an SMQ file; ``cfg`` as the reference passes a
    ModelConfig, else built from the file's llama.* metadata."""
    f = smq_read(path)
    cfg = cfg or config_from_metadata(f.metadata, f.tensors, max_context)
    return build_model(ctx, f.tensors, cfg), f.metadata


def load_gguf_model(ctx: CudaContext, path, max_context: int | None = None):
    """(CudaModel, metadata) from a GGUF file, raw blocks passed straight through."""
    g = gguf_read(path)
    tensors = {t.name: gguf_tensor_to_host(g, t) for t in g.tensors}
    cfg = config_from_metadata(g.metadata, tensors, max_context)
    return build_model(ctx, tensors, cfg), g.metadata
