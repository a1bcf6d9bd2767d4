"""Synthetic GGUF files for the loader tests: a writer for the public GGUF v3
container and random ggml-layout blocks, plus ggml's block dequantization
restated from the published block formats (the checker the layout conversion is
tested against).  Test infrastructure only."""
import struct

import numpy as np

F32, F16, Q4_0, Q4_1, Q5_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 3, 6, 8, 12, 14
BLOCK = {Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}


def _s(x: str) -> bytes:
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


def _val(v):
    """(type, payload) of a metadata value: str, bool, int (int32 / uint64), float, list."""
    if isinstance(v, str):
        return 8, _s(v)
    if isinstance(v, bool):
        return 7, struct.pack("<?", v)
    if isinstance(v, int):
        return (5, struct.pack("<i", v)) if -2**31 <= v < 2**31 else (10, struct.pack("<Q", v))
    if isinstance(v, float):
        return 6, struct.pack("<f", v)
    if isinstance(v, list):
        et, _ = _val(v[0])
        return 9, struct.pack("<IQ", et, len(v)) + b"".join(_val(e)[1] for e in v)
    raise TypeError(type(v))


def write_gguf(path, metadata: dict, tensors: list, alignment: int = 32):
    """tensors: (name, ggml dims (fastest first), ggml type, raw bytes)."""
    out = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(metadata) + 1))
    for k, v in list(metadata.items()) + [("general.alignment", alignment)]:
        t, p = _val(v)
        out += _s(k) + struct.pack("<I", t) + p
    offs, off = [], 0
    for _, _, _, raw in tensors:
        offs.append(off)
        off = (off + len(raw) + alignment - 1) // alignment * alignment
    for (name, dims, ttype, _), o in zip(tensors, offs):
        out += _s(name) + struct.pack("<I", len(dims)) + struct.pack("<" + "Q" * len(dims), *dims)
        out += struct.pack("<IQ", ttype, o)
    out += b"\0" * ((-len(out)) % alignment)
    base = len(out)
    for (_, _, _, raw), o in zip(tensors, offs):
        out += b"\0" * (base + o - len(out))
        out += bytes(raw)
    with open(path, "wb") as f:
        f.write(bytes(out))


def random_blocks(ttype: int, n: int, rs: np.random.RandomState, scale: float = 1e-3) -> np.ndarray:
    """Random ggml blocks for n elements: random codes, fp16 scales around `scale`."""
    be, bb = BLOCK[ttype]
    nb = n // be
    b = rs.randint(0, 256, (nb, bb)).astype(np.uint8)
    h = lambda a: np.asarray(a, np.float16).view(np.uint8).reshape(nb, -1)
    if ttype in (Q4_0, Q8_0, Q5_0):
        b[:, 0:2] = h(rs.randn(nb) * scale * 10)
    elif ttype == Q4_1:
        b[:, 0:2] = h(np.abs(rs.randn(nb)) * scale * 10)
        b[:, 2:4] = h(rs.randn(nb) * scale * 50)
    elif ttype == Q4_K:
        b[:, 0:2] = h(np.abs(rs.randn(nb)) * scale)
        b[:, 2:4] = h(np.abs(rs.randn(nb)) * scale)
    elif ttype == Q6_K:
        b[:, 192:208] = rs.randint(-40, 40, (nb, 16)).astype(np.int8).view(np.uint8)
        b[:, 208:210] = h(rs.randn(nb) * scale * 0.3)
    return b.reshape(-1)


def _f16(b):
    return np.ascontiguousarray(b).view(np.float16).astype(np.float32)


def ggml_dequant(ttype: int, raw: np.ndarray) -> np.ndarray:
    """fp32 values of ggml blocks (the published Q8_0 / Q4_0 / Q4_1 / Q5_0 / Q4_K / Q6_K formulas)."""
    f = np.float32
    if ttype == Q8_0:
        b = raw.reshape(-1, 34)
        return (b[:, 2:].view(np.int8).astype(f) * _f16(b[:, :2])).reshape(-1)
    if ttype == Q4_0:
        b = raw.reshape(-1, 18)
        q = np.concatenate([b[:, 2:] & 0xF, b[:, 2:] >> 4], axis=1).astype(np.int32) - 8
        return (q.astype(f) * _f16(b[:, :2])).reshape(-1)
    if ttype == Q4_1:
        b = raw.reshape(-1, 20)
        q = np.concatenate([b[:, 4:] & 0xF, b[:, 4:] >> 4], axis=1).astype(f)
        return ((q * _f16(b[:, 0:2])).astype(f) + _f16(b[:, 2:4])).reshape(-1)
    if ttype == Q5_0:
        b = raw.reshape(-1, 22)
        qh = np.ascontiguousarray(b[:, 2:6]).view(np.uint32).astype(np.int64)
        lo = np.concatenate([b[:, 6:] & 0xF, b[:, 6:] >> 4], axis=1).astype(np.int64)
        hi = (qh >> np.arange(32)) & 1
        return (((lo | (hi << 4)) - 16).astype(f) * _f16(b[:, 0:2])).reshape(-1)
    if ttype == Q4_K:
        b = raw.reshape(-1, 144)
        d, dmin = _f16(b[:, 0:2]), _f16(b[:, 2:4])
        sc = b[:, 4:16].astype(np.int32)
        y = np.empty((b.shape[0], 256), f)
        for j in range(8):
            if j < 4:
                s, m = sc[:, j] & 63, sc[:, j + 4] & 63
            else:
                s = (sc[:, j + 4] & 0xF) | ((sc[:, j - 4] >> 6) << 4)
                m = (sc[:, j + 4] >> 4) | ((sc[:, j] >> 6) << 4)
            d1 = (d[:, 0] * s.astype(f)).astype(f)
            m1 = (dmin[:, 0] * m.astype(f)).astype(f)
            c, hi = j // 2, j % 2
            qs = b[:, 16 + 32 * c:16 + 32 * c + 32]
            q = (qs >> 4) if hi else (qs & 0xF)
            y[:, 32 * j:32 * j + 32] = (d1[:, None] * q.astype(f)).astype(f) - m1[:, None]
        return y.reshape(-1)
    if ttype == Q6_K:
        b = raw.reshape(-1, 210)
        d = _f16(b[:, 208:210])[:, 0]
        sc = b[:, 192:208].view(np.int8).astype(f)
        y = np.empty((b.shape[0], 256), f)
        for h in range(2):
            ql, qh = b[:, 64 * h:64 * h + 64].astype(np.int32), b[:, 128 + 32 * h:128 + 32 * h + 32].astype(np.int32)
            for l in range(32):
                isc = 8 * h + l // 16
                q1 = ((ql[:, l] & 0xF) | (((qh[:, l] >> 0) & 3) << 4)) - 32
                q2 = ((ql[:, l + 32] & 0xF) | (((qh[:, l] >> 2) & 3) << 4)) - 32
                q3 = ((ql[:, l] >> 4) | (((qh[:, l] >> 4) & 3) << 4)) - 32
                q4 = ((ql[:, l + 32] >> 4) | (((qh[:, l] >> 6) & 3) << 4)) - 32
                for k, q in enumerate((q1, q2, q3, q4)):
                    y[:, 128 * h + 32 * k + l] = ((d * sc[:, isc + 2 * k]).astype(f) * q.astype(f)).astype(f)
        return y.reshape(-1)
    raise ValueError(ttype)


DEFAULT_TYPES = dict(q=Q4_K, k=Q4_K, v=Q6_K, o=Q4_K, gate=Q4_K, up=Q4_K, down=Q6_K, output=Q6_K)


def tiny_llama_gguf(path, cfg: dict, seed: int = 5, types: dict | None = None):
    """A LLaMA-shaped GGUF: by default Q4_K q/k/o/gate/up, Q6_K v/down/output
    (``types`` overrides per role), F32 norms, F16 embedding.  Returns
    {name: (ggml type, raw bytes, ggml dims)}."""
    ty = dict(DEFAULT_TYPES, **(types or {}))
    rs = np.random.RandomState(seed)
    H, F, V = cfg["hidden"], cfg["ffn_hidden"], cfg["vocab_size"]
    qd, kd = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]
    meta = {"general.architecture": "llama", "general.name": "tiny", "llama.context_length": cfg["max_context"],
            "llama.embedding_length": H, "llama.block_count": cfg["n_layers"], "llama.feed_forward_length": F,
            "llama.attention.head_count": cfg["n_heads"], "llama.attention.head_count_kv": cfg["n_kv_heads"],
            "llama.rope.freq_base": float(cfg.get("rope_theta", 10000.0)),
            "llama.attention.layer_norm_rms_epsilon": float(cfg.get("norm_eps", 1e-5)),
            "tokenizer.ggml.tokens": [f"t{i}" for i in range(8)]}
    ts = {}

    def add(name, ttype, rows, cols):
        if ttype == F32:
            raw = (1.0 + 0.05 * rs.randn(rows * cols)).astype(np.float32).view(np.uint8)
        elif ttype == F16:  # the embedding at 0.5, linear weights at 0.02
            sd = 0.5 if name == "token_embd.weight" else 0.02
            raw = (sd * rs.randn(rows * cols)).astype(np.float16).view(np.uint8)
        else:
            raw = random_blocks(ttype, rows * cols, rs)
        ts[name] = (ttype, raw, [cols] if rows == 1 else [cols, rows])

    add("token_embd.weight", F16, V, H)
    for l in range(cfg["n_layers"]):
        p = f"blk.{l}."
        add(p + "attn_norm.weight", F32, 1, H)
        add(p + "attn_q.weight", ty["q"], qd, H)
        add(p + "attn_k.weight", ty["k"], kd, H)
        add(p + "attn_v.weight", ty["v"], kd, H)
        add(p + "attn_output.weight", ty["o"], H, qd)
        add(p + "ffn_norm.weight", F32, 1, H)
        add(p + "ffn_gate.weight", ty["gate"], F, H)
        add(p + "ffn_up.weight", ty["up"], F, H)
        add(p + "ffn_down.weight", ty["down"], H, F)
    add("output_norm.weight", F32, 1, H)
    add("output.weight", ty["output"], V, H)
    write_gguf(path, meta, [(n, dims, t, raw) for n, (t, raw, dims) in ts.items()])
    return ts
