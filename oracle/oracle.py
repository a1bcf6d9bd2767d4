"""ctypes wrapper of the CPU oracle (test infrastructure only).

The oracle is a C++17 restatement of the reference's C# arithmetic for the
quantized decode/prefill path (see oracle.h for the per-function citations).
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it, as
the checker or the timed CPU baseline — never as the product path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

F32, F16, Q8_0, Q4_0, Q4_1, Q5_0, Q4_K, Q6_K = range(8)
BYTES_PER_BLOCK = {Q4_K: 144, Q6_K: 210}


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


class DotnetRandom(C.Structure):
    _fields_ = [("seed_array", C.c_int32 * 56), ("inext", C.c_int), ("inextp", C.c_int)]


class ModelConfig(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_int), ("hidden", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int),
        ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("ffn_hidden", C.c_int), ("max_context", C.c_int),
        ("norm_eps", C.c_float), ("rope_theta", C.c_float),
    ]


class Linear(C.Structure):
    _fields_ = [("scheme", C.c_int), ("block_size", C.c_int), ("data", C.c_void_p), ("scales", C.c_void_p)]


class Layer(C.Structure):
    _fields_ = [("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p)] + [
        (n, Linear) for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")
    ]


class Model(C.Structure):
    _fields_ = [("cfg", ModelConfig), ("token_embd", C.c_void_p), ("out_norm", C.c_void_p),
                ("output", Linear), ("layers", C.c_void_p)]


def _declare(L):
    vp, i, i64, f = C.c_void_p, C.c_int, C.c_int64, C.c_float
    sig = {
        "or_dotnet_random_init": (None, [C.POINTER(DotnetRandom), C.c_int32]),
        "or_dotnet_random_next_double": (C.c_double, [C.POINTER(DotnetRandom)]),
        "or_dotnet_random_floats": (None, [C.POINTER(DotnetRandom), vp, i, f, f]),
        "or_half_to_float": (f, [C.c_uint16]),
        "or_float_to_half_rne": (C.c_uint16, [f]),
        "or_q8_quantize": (i, [vp, i64, i, vp, vp]),
        "or_q8_dequantize": (None, [vp, vp, i64, i, vp]),
        "or_q4_decode_nibble": (i, [i]),
        "or_q4_quantize": (i, [vp, i64, i, vp, vp]),
        "or_q41_quantize": (i, [vp, i64, vp, vp, vp]),
        "or_q41_dequantize": (None, [vp, vp, vp, i64, vp]),
        "or_q50_quantize": (i, [vp, i64, vp, vp, vp]),
        "or_q50_dequantize": (None, [vp, vp, vp, i64, vp]),
        "or_q4_dequantize": (None, [vp, vp, i64, i, vp]),
        "or_q4k_quantize": (None, [vp, i64, vp]),
        "or_q4k_dequantize": (None, [vp, i64, vp]),
        "or_q6k_quantize": (None, [vp, i64, vp]),
        "or_q6k_dequantize": (None, [vp, i64, vp]),
        "or_matmul": (i, [i, i, vp, vp, i, vp, vp, vp, i, i, i]),
        "or_rmsnorm": (None, [vp, vp, vp, i, i, f]),
        "or_rope_tables": (None, [i, i, f, vp, vp]),
        "or_rope_apply": (None, [vp, i, i, i, vp, vp]),
        "or_fast_exp": (f, [f]),
        "or_silu_mul": (None, [vp, vp, vp, i]),
        "or_attention": (None, [vp, vp, vp, vp, i, i, i, i, i, i]),
        "or_model_forward": (i, [C.POINTER(Model), vp, i, i, vp, i]),
        "or_model_step": (i, [C.POINTER(Model), vp, i, vp, i, vp, i]),
        "or_fill_normal": (None, [vp, i64, C.c_uint64, f, i]),
        "or_set_linear_threads": (None, [i]),
        "or_sample": (i, [vp, i, C.c_double, i, C.c_double, C.c_double, f, f, f, i, vp, i, C.c_double, vp]),
        "or_deterministic_rng_doubles": (None, [C.c_int32, i, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- random
def dotnet_random(seed: int) -> DotnetRandom:
    r = DotnetRandom()
    lib().or_dotnet_random_init(C.byref(r), seed)
    return r


def dotnet_random_floats(r: DotnetRandom, count: int, lo: float, hi: float) -> np.ndarray:
    out = np.empty(count, np.float32)
    lib().or_dotnet_random_floats(C.byref(r), _p(out), count, lo, hi)
    return out


def fill_normal(n: int, seed: int, std: float = 0.02, threads: int = 8) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().or_fill_normal(_p(out), n, seed, std, threads)
    return out


# ---------------------------------------------------------------- quantizers
@dataclass
class QTensor:
    """Packed weight in the reference layout: rows x cols, linear index order."""
    scheme: int
    rows: int
    cols: int
    data: np.ndarray                 # uint8 / int8 packed bytes
    scales: np.ndarray | None = None  # fp32 block scales (Q8_0 / Q4_0)
    block_size: int = 256


def quantize(x: np.ndarray, scheme: int, rows: int, cols: int, block_size: int = 32) -> QTensor:
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    n = rows * cols
    assert x.size == n
    L = lib()
    if scheme == Q8_0:
        data = np.empty(n, np.int8)
        scales = np.empty((n + block_size - 1) // block_size, np.float32)
        assert L.or_q8_quantize(_p(x), n, block_size, _p(data), _p(scales)) == 0
        return QTensor(scheme, rows, cols, data, scales, block_size)
    if scheme == Q4_0:
        data = np.zeros((n + 1) // 2, np.uint8)
        scales = np.empty((n + block_size - 1) // block_size, np.float32)
        assert L.or_q4_quantize(_p(x), n, block_size, _p(data), _p(scales)) == 0
        return QTensor(scheme, rows, cols, data, scales, block_size)
    if scheme == Q4_1:
        # QTensor convention: data = nibbles, scales = block scales then block mins (block 32)
        nb = (n + 31) // 32
        data = np.zeros((n + 1) // 2, np.uint8)
        sc = np.empty(2 * nb, np.float32)
        assert L.or_q41_quantize(_p(x), n, _p(data), _p(sc[:nb]), sc[nb:].ctypes.data_as(C.c_void_p)) == 0
        return QTensor(scheme, rows, cols, data, sc, 32)
    if scheme == Q5_0:
        # QTensor convention: data = low nibbles then the 4-byte high-bit words, scales (block 32)
        nb = (n + 31) // 32
        data = np.zeros((n + 1) // 2 + 4 * nb, np.uint8)
        sc = np.empty(nb, np.float32)
        assert L.or_q50_quantize(_p(x), n, _p(data), data[(n + 1) // 2:].ctypes.data_as(C.c_void_p), _p(sc)) == 0
        return QTensor(scheme, rows, cols, data, sc, 32)
    if scheme == Q4_K:
        assert cols % 256 == 0
        data = np.empty(n // 256 * 144, np.uint8)
        L.or_q4k_quantize(_p(x), n, _p(data))
        return QTensor(scheme, rows, cols, data)
    if scheme == Q6_K:
        assert cols % 256 == 0
        data = np.empty(n // 256 * 210, np.uint8)
        L.or_q6k_quantize(_p(x), n, _p(data))
        return QTensor(scheme, rows, cols, data)
    if scheme == F32:
        return QTensor(scheme, rows, cols, x.copy().view(np.uint8), None, 1)
    raise ValueError(scheme)


def dequantize(t: QTensor) -> np.ndarray:
    n = t.rows * t.cols
    out = np.empty(n, np.float32)
    L = lib()
    if t.scheme == Q8_0:
        L.or_q8_dequantize(_p(t.data), _p(t.scales), n, t.block_size, _p(out))
    elif t.scheme == Q4_0:
        L.or_q4_dequantize(_p(t.data), _p(t.scales), n, t.block_size, _p(out))
    elif t.scheme == Q4_1:
        nb = (n + 31) // 32
        L.or_q41_dequantize(_p(t.data), _p(t.scales), t.scales[nb:].ctypes.data_as(C.c_void_p), n, _p(out))
    elif t.scheme == Q5_0:
        L.or_q50_dequantize(_p(t.data), t.data[(n + 1) // 2:].ctypes.data_as(C.c_void_p), _p(t.scales), n, _p(out))
    elif t.scheme == Q4_K:
        L.or_q4k_dequantize(_p(t.data), n, _p(out))
    elif t.scheme == Q6_K:
        L.or_q6k_dequantize(_p(t.data), n, _p(out))
    elif t.scheme == F32:
        out[:] = t.data.view(np.float32)
    else:
        raise ValueError(t.scheme)
    return out.reshape(t.rows, t.cols)


def reorder_kquant_blocks_to_literal(t: QTensor) -> QTensor:
    """GGUF/linear block order [N][K/256] -> the reference fused kernels' order
    [K/256][N] (FusedQ4KMatMul.cs:122,127): same blocks, transposed block grid."""
    bpb = BYTES_PER_BLOCK[t.scheme]
    nb = t.cols // 256
    blocks = t.data.reshape(t.rows, nb, bpb).transpose(1, 0, 2)
    return QTensor(t.scheme, t.cols, t.rows, np.ascontiguousarray(blocks).reshape(-1), None, t.block_size)


def matmul(t: QTensor, a: np.ndarray, m: int, k: int, n: int, mode: int, want64: bool = False):
    a = np.ascontiguousarray(a, np.float32)
    c = np.empty((m, n), np.float32)
    c64 = np.empty((m, n), np.float64) if want64 else None
    rc = lib().or_matmul(t.scheme, mode, _p(t.data), _p(t.scales) if t.scales is not None else None,
                         t.block_size, _p(a), _p(c), _p(c64) if want64 else None, m, k, n)
    if rc != 0:
        raise ValueError(f"or_matmul rc={rc}")
    return (c, c64) if want64 else c


# ---------------------------------------------------------------- model ops
def set_linear_threads(n: int) -> None:
    """0: quantized linears split rows over the caller's threads; 1: single-threaded,
    the reference's own threading for MatMulF32Q8 / FusedQ4KMatMul / FusedQ6KMatMul."""
    lib().or_set_linear_threads(int(n))


def rmsnorm(x: np.ndarray, gamma: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    rows, feat = x.reshape(-1, x.shape[-1]).shape
    y = np.empty_like(x)
    lib().or_rmsnorm(_p(x), _p(np.ascontiguousarray(gamma, np.float32)), _p(y), rows, feat, eps)
    return y


def rope_tables(max_seq: int, head_dim: int, theta: float = 10000.0):
    s = np.empty((max_seq, head_dim // 2), np.float32)
    c = np.empty_like(s)
    lib().or_rope_tables(max_seq, head_dim, theta, _p(s), _p(c))
    return s, c


def rope_apply(x: np.ndarray, n_heads: int, head_dim: int, pos: int, sin_t, cos_t) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).copy()
    lib().or_rope_apply(_p(x), n_heads, head_dim, pos, _p(sin_t), _p(cos_t))
    return x


def fast_exp(x: float) -> float:
    return lib().or_fast_exp(x)


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    out = np.empty_like(g)
    lib().or_silu_mul(_p(g), _p(u), _p(out), g.size)
    return out


def attention(q, k, v, T: int, S: int, n_heads: int, n_kv: int, head_dim: int, threads: int = 8):
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    out = np.empty((T, n_heads * head_dim), np.float32)
    lib().or_attention(_p(q), _p(k), _p(v), _p(out), T, S, n_heads, n_kv, head_dim, threads)
    return out


# ---------------------------------------------------------------- model
@dataclass
class HostModel:
    """Synthetic LLaMA-shaped model with packed weights (intended orientation:
    each linear is W[out][in], quantized along `in`)."""
    cfg: dict
    token_embd: np.ndarray
    out_norm: np.ndarray
    output: QTensor
    layers: list = field(default_factory=list)  # dicts: attn_norm, ffn_norm, wq..w_down
    _keep: list = field(default_factory=list)

    def as_ctypes(self) -> Model:
        c = self.cfg
        m = Model()
        m.cfg = ModelConfig(c["vocab_size"], c["hidden"], c["n_layers"], c["n_heads"], c["n_kv_heads"],
                            c["head_dim"], c["ffn_hidden"], c["max_context"], c["norm_eps"], c["rope_theta"])
        m.token_embd = self.token_embd.ctypes.data
        m.out_norm = self.out_norm.ctypes.data
        m.output = _lin(self.output)
        arr = (Layer * len(self.layers))()
        for i, L in enumerate(self.layers):
            arr[i].attn_norm = L["attn_norm"].ctypes.data
            arr[i].ffn_norm = L["ffn_norm"].ctypes.data
            for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"):
                setattr(arr[i], n, _lin(L[n]))
        m.layers = C.cast(arr, C.c_void_p)
        self._keep = [arr]
        return m


def _lin(t: QTensor) -> Linear:
    return Linear(t.scheme, t.block_size, t.data.ctypes.data, t.scales.ctypes.data if t.scales is not None else None)


LINEAR_NAMES = ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")


def make_model(cfg: dict, schemes: dict, seed: int = 1234, std: float = 0.02, block_size: int = 32,
               threads: int = 8) -> HostModel:
    """Random-init N(0, std) model; `schemes` maps linear name (+ 'output') to a scheme."""
    H, F, V = cfg["hidden"], cfg["ffn_hidden"], cfg["vocab_size"]
    qd = cfg["n_heads"] * cfg["head_dim"]
    kd = cfg["n_kv_heads"] * cfg["head_dim"]
    shapes = {"wq": (qd, H), "wk": (kd, H), "wv": (kd, H), "wo": (H, qd), "w_gate": (F, H), "w_up": (F, H),
              "w_down": (H, F)}
    ctr = [seed]

    def nxt(n):
        ctr[0] += 1
        return fill_normal(n, ctr[0], std, threads)

    emb = nxt(V * H).reshape(V, H)
    layers = []
    for _ in range(cfg["n_layers"]):
        L = {"attn_norm": np.ones(H, np.float32), "ffn_norm": np.ones(H, np.float32)}
        for n in LINEAR_NAMES:
            r, c = shapes[n]
            L[n] = quantize(nxt(r * c), schemes[n], r, c, block_size)
        layers.append(L)
    out = quantize(nxt(V * H), schemes["output"], V, H, block_size)
    return HostModel(cfg, emb, np.ones(H, np.float32), out, layers)


def model_forward(m: HostModel, tokens, n_last: int = 1, threads: int = 8) -> np.ndarray:
    toks = np.ascontiguousarray(tokens, np.int32)
    cm = m.as_ctypes()
    out = np.empty((n_last, m.cfg["vocab_size"]), np.float32)
    rc = lib().or_model_forward(C.byref(cm), _p(toks), toks.size, n_last, _p(out), threads)
    if rc:
        raise ValueError(f"or_model_forward rc={rc}")
    return out


class KVDecoder:
    """KV-cached step-by-step twin (the CPU baseline's timed loop)."""

    def __init__(self, m: HostModel, threads: int = 8):
        c = m.cfg
        self.m, self.threads = m, threads
        self.cm = m.as_ctypes()
        self.kv = np.zeros(c["n_layers"] * 2 * c["max_context"] * c["n_kv_heads"] * c["head_dim"], np.float32)
        self.pos = 0

    def step(self, tokens) -> np.ndarray:
        toks = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(self.m.cfg["vocab_size"], np.float32)
        rc = lib().or_model_step(C.byref(self.cm), _p(self.kv), self.pos, _p(toks), toks.size, _p(out),
                                 self.threads)
        if rc:
            raise ValueError(f"or_model_step rc={rc}")
        self.pos += toks.size
        return out


# ---------------------------------------------------------------- sampling
def sample(logits: np.ndarray, target: float, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0,
           min_p: float = 0.0, repetition_penalty: float = 1.0, presence_penalty: float = 0.0,
           frequency_penalty: float = 0.0, repetition_window: int = 0, context=()):
    """(token, probs) of one row through the reference sampling pipeline (or_sample)."""
    lg = np.array(logits, np.float32).reshape(-1)
    ctx = np.ascontiguousarray(np.asarray(context, np.int32).reshape(-1))
    probs = np.empty_like(lg)
    t = lib().or_sample(_p(lg), lg.size, temperature, top_k, top_p, min_p, repetition_penalty, presence_penalty,
                        frequency_penalty, repetition_window, _p(ctx) if ctx.size else None, ctx.size, target,
                        _p(probs))
    return t, probs


def deterministic_rng_doubles(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float64)
    lib().or_deterministic_rng_doubles(seed, n, _p(out))
    return out
