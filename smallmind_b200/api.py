"""Host-side mirror of the reference's operator API for the quantized hot path.

``CudaWeightTensor`` implements the reference ``IWeightTensor`` contract
(src/SmallMind.Quantization/Abstractions/IWeightTensor.cs:7-42): ``Rows``,
``Cols``, ``Scheme``, ``MatMul(activations, output, m, k, n)`` and
``ToFloat32()``, with the reference's ArgumentException rules surfaced as
``ValueError`` (``ShapeError``).  ``CudaModel`` / ``InferenceSession`` mirror the
generation loop around it (TransformerModel.Forward, InferenceSession
.GenerateNextTokenAsync) on the device-resident model and HBM KV cache.

Everything runs in libsmallmind_cuda.so; there is no CPU path.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from enum import IntEnum

import numpy as np

from . import _lib as L


class QuantScheme(IntEnum):
    """IWeightTensor.cs:47-72."""
    F32 = 0
    F16 = 1
    Q8_0 = 2
    Q4_0 = 3
    Q4_1 = 4
    Q5_0 = 5
    Q4_K = 6
    Q6_K = 7


def _p(a: np.ndarray):
    if not a.flags["C_CONTIGUOUS"]:
        raise ValueError("arrays must be C-contiguous")
    return a.ctypes.data_as(C.c_void_p)


class CudaContext:
    """One device + one CUDA stream (sm_ctx)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        L.check(L.lib().sm_ctx_create(device, C.byref(h)), "sm_ctx_create")
        self.handle = h
        self.device = device

    def sync(self):
        L.check(L.lib().sm_stream_sync(self.handle), "sm_stream_sync")

    def set_stream(self, stream_ptr: int | None):
        L.check(L.lib().sm_ctx_set_stream(self.handle, C.c_void_p(stream_ptr or 0)), "sm_ctx_set_stream")

    def launch_count(self) -> int:
        v = C.c_int64()
        L.check(L.lib().sm_ctx_launch_count(self.handle, C.byref(v)))
        return v.value

    def device_status(self) -> int:
        return L.lib().sm_ctx_device_status(self.handle)

    def close(self):
        if self.handle:
            L.lib().sm_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CudaWeightTensor:
    """IWeightTensor on the GPU (Q8WeightTensor / Q4WeightTensor / Q4KWeightTensor / Q6KWeightTensor).

    ``layout`` LAYOUT_INTENDED (default): Rows = out features N, Cols = in
    features K, MatMul computes output = activations x weights^T.
    ``layout`` LAYOUT_REFERENCE: the reference kernels as written, Rows = K,
    Cols = N, MatMul computes C = A x B.
    """

    def __init__(self, ctx: CudaContext, scheme: int, rows: int, cols: int, data: np.ndarray,
                 scales: np.ndarray | None = None, block_size: int = 64, layout: int = L.LAYOUT_INTENDED):
        data = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        sc = None if scales is None else np.ascontiguousarray(scales, np.float32)
        h = C.c_void_p()
        L.check(L.lib().sm_weight_upload(ctx.handle, int(scheme), rows, cols, block_size, _p(data), data.size,
                                         _p(sc) if sc is not None else None, 0 if sc is None else sc.size,
                                         layout, C.byref(h)), "sm_weight_upload")
        self.ctx, self.handle = ctx, h
        self._rows, self._cols, self._scheme, self.layout = rows, cols, QuantScheme(scheme), layout

    @classmethod
    def from_qtensor(cls, ctx: CudaContext, t, layout: int = L.LAYOUT_INTENDED) -> "CudaWeightTensor":
        """From any object with scheme/rows/cols/data/scales/block_size (e.g. a packed host tensor)."""
        return cls(ctx, t.scheme, t.rows, t.cols, t.data, t.scales, t.block_size, layout)

    # IWeightTensor.cs:12-22
    @property
    def Rows(self) -> int:
        return self._rows

    @property
    def Cols(self) -> int:
        return self._cols

    @property
    def Scheme(self) -> QuantScheme:
        return self._scheme

    def nbytes(self) -> int:
        v = C.c_size_t()
        L.check(L.lib().sm_weight_nbytes(self.handle, C.byref(v)))
        return v.value

    def MatMul(self, activations: np.ndarray, output: np.ndarray, m: int, k: int, n: int) -> None:
        """IWeightTensor.MatMul (IWeightTensor.cs:33); output is overwritten."""
        a = np.ascontiguousarray(activations, np.float32).reshape(-1)
        if a.size < m * k:
            raise L.ShapeError(-2, f"activations.Length {a.size} < m*k {m * k}")
        if output.dtype != np.float32 or not output.flags["C_CONTIGUOUS"] or output.size < m * n:
            raise L.ShapeError(-2, f"output.Length {output.size} < m*n {m * n}")
        L.check(L.lib().sm_matmul(self.handle, _p(a), _p(output), m, k, n, L.PTR_HOST), "MatMul")

    def matmul_device(self, a_ptr: int, c_ptr: int, m: int) -> None:
        """Device-pointer variant (asynchronous on the context stream)."""
        k = self._cols if self.layout == L.LAYOUT_INTENDED else self._rows
        n = self._rows if self.layout == L.LAYOUT_INTENDED else self._cols
        L.check(L.lib().sm_matmul(self.handle, C.c_void_p(a_ptr), C.c_void_p(c_ptr), m, k, n, L.PTR_DEVICE),
                "matmul_device")

    def ToFloat32(self) -> np.ndarray:
        """IWeightTensor.ToFloat32 (IWeightTensor.cs:41): bit-exact dequantization."""
        out = np.empty(self._rows * self._cols, np.float32)
        L.check(L.lib().sm_dequant(self.handle, _p(out), L.PTR_HOST), "ToFloat32")
        return out

    def close(self):
        if self.handle:
            L.lib().sm_weight_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------- ops
def rmsnorm(ctx: CudaContext, x: np.ndarray, gamma: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """RMSNormOps.RMSNorm (RMSNormOps.cs:28-220)."""
    x = np.ascontiguousarray(x, np.float32)
    g = np.ascontiguousarray(gamma, np.float32)
    rows = x.size // g.size
    y = np.empty_like(x)
    L.check(L.lib().sm_op_rmsnorm(ctx.handle, _p(x), _p(g), _p(y), rows, g.size, eps, L.PTR_HOST), "rmsnorm")
    return y


def rope(ctx: CudaContext, x: np.ndarray, n_heads: int, head_dim: int, positions, theta: float = 10000.0,
         max_seq: int = 2048) -> np.ndarray:
    """RotaryEmbedding.ApplyInPlace (RotaryEmbedding.cs:69-121) on token rows [rows][n_heads*head_dim]."""
    x = np.ascontiguousarray(x, np.float32).copy()
    pos = np.ascontiguousarray(positions, np.int32)
    L.check(L.lib().sm_op_rope(ctx.handle, _p(x), pos.size, n_heads, head_dim, _p(pos), theta, max_seq,
                               L.PTR_HOST), "rope")
    return x


def silu_mul(ctx: CudaContext, gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """ActivationOps.FusedSiLUMul (ActivationOps.cs:565-580)."""
    g = np.ascontiguousarray(gate, np.float32)
    u = np.ascontiguousarray(up, np.float32)
    out = np.empty_like(g)
    L.check(L.lib().sm_op_silu_mul(ctx.handle, _p(g), _p(u), _p(out), g.size, L.PTR_HOST), "silu_mul")
    return out


def attention(ctx: CudaContext, q, k, v, T: int, S: int, n_heads: int, n_kv: int, head_dim: int) -> np.ndarray:
    """Causal GQA attention with the reference's Pade softmax (MultiHeadAttention.cs:676-744, 810-844)."""
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    out = np.empty((T, n_heads * head_dim), np.float32)
    L.check(L.lib().sm_attention(ctx.handle, _p(q), _p(k), _p(v), _p(out), T, S, n_heads, n_kv, head_dim,
                                 L.PTR_HOST), "attention")
    return out


# ---------------------------------------------------------------- model
ROLE_OF = {"wq": L.ROLE_WQ, "wk": L.ROLE_WK, "wv": L.ROLE_WV, "wo": L.ROLE_WO, "w_gate": L.ROLE_W_GATE,
           "w_up": L.ROLE_W_UP, "w_down": L.ROLE_W_DOWN}


class CudaModel:
    """new TransformerModel(ModelConfig) (TransformerModel.cs:163-259) resident on one GPU."""

    def __init__(self, ctx: CudaContext, cfg: dict):
        self.ctx, self.cfg = ctx, dict(cfg)
        c = L.ModelConfig(cfg["vocab_size"], cfg["hidden"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv_heads"],
                          cfg["head_dim"], cfg["ffn_hidden"], cfg["max_context"], cfg.get("norm_eps", 1e-5),
                          cfg.get("rope_theta", 10000.0))
        h = C.c_void_p()
        L.check(L.lib().sm_model_create(ctx.handle, C.byref(c), C.byref(h)), "sm_model_create")
        self.handle = h
        self._weights = []  # keeps borrowed weights alive

    def set_weight(self, layer: int, name: str, w: CudaWeightTensor):
        role = L.ROLE_OUTPUT if name == "output" else ROLE_OF[name]
        L.check(L.lib().sm_model_set_weight(self.handle, layer, role, w.handle), f"set_weight {name}")
        self._weights.append(w)

    def set_vector(self, layer: int, name: str, data: np.ndarray):
        role = {"attn_norm": L.ROLE_ATTN_NORM, "ffn_norm": L.ROLE_FFN_NORM, "token_embd": L.ROLE_TOKEN_EMBD,
                "out_norm": L.ROLE_OUT_NORM}[name]
        d = np.ascontiguousarray(data, np.float32).reshape(-1)
        L.check(L.lib().sm_model_set_vector(self.handle, layer, role, _p(d), d.size), f"set_vector {name}")

    def finalize(self):
        L.check(L.lib().sm_model_finalize(self.handle), "sm_model_finalize")

    @classmethod
    def from_host(cls, ctx: CudaContext, host_model) -> "CudaModel":
        """Upload a packed host model (token_embd, out_norm, output, layers[...] dicts)."""
        m = cls(ctx, host_model.cfg)
        m.set_vector(0, "token_embd", host_model.token_embd)
        m.set_vector(0, "out_norm", host_model.out_norm)
        m.set_weight(0, "output", CudaWeightTensor.from_qtensor(ctx, host_model.output))
        for li, layer in enumerate(host_model.layers):
            m.set_vector(li, "attn_norm", layer["attn_norm"])
            m.set_vector(li, "ffn_norm", layer["ffn_norm"])
            for n in ROLE_OF:
                m.set_weight(li, n, CudaWeightTensor.from_qtensor(ctx, layer[n]))
        m.finalize()
        m._owns_weights = True
        return m

    def nbytes(self) -> int:
        v = C.c_size_t()
        L.check(L.lib().sm_model_nbytes(self.handle, C.byref(v)))
        return v.value

    def close(self):
        """Releases the model; weights uploaded by from_host go with it (weights passed to
        set_weight by the caller stay the caller's)."""
        if self.handle:
            L.lib().sm_model_destroy(self.handle)
            self.handle = None
        if getattr(self, "_owns_weights", False):
            for w in self._weights:
                w.close()
            self._weights = []


class KVCache:
    """HBM KV cache for many sequences (sm_kv)."""

    def __init__(self, model: CudaModel, max_seqs: int, max_tokens: int):
        h = C.c_void_p()
        L.check(L.lib().sm_kv_create(model.handle, max_seqs, max_tokens, C.byref(h)), "sm_kv_create")
        self.model, self.handle = model, h
        self.max_seqs, self.max_tokens = max_seqs, max_tokens

    def reset(self, seq: int):
        L.check(L.lib().sm_kv_reset(self.handle, seq), "sm_kv_reset")

    def length(self, seq: int) -> int:
        v = C.c_int()
        L.check(L.lib().sm_kv_length(self.handle, seq, C.byref(v)), "sm_kv_length")
        return v.value

    def truncate(self, seq: int, length: int):
        """Keep the first ``length`` cached tokens of ``seq``."""
        L.check(L.lib().sm_kv_truncate(self.handle, seq, length), "sm_kv_truncate")

    def slide(self, seq: int, window: int):
        """KvCacheEntry.Slide: keep the last ``window`` tokens, moved to the front."""
        L.check(L.lib().sm_kv_slide(self.handle, seq, window), "sm_kv_slide")

    def read(self, layer: int, seq: int, start: int, count: int):
        """KvCacheEntry.GetKeys / GetValues: (keys, values), each [count, n_kv_heads * head_dim]."""
        width = self.model.cfg["n_kv_heads"] * self.model.cfg["head_dim"]
        k = np.empty((count, width), np.float32)
        v = np.empty((count, width), np.float32)
        L.check(L.lib().sm_kv_read(self.handle, layer, seq, start, count, _p(k), _p(v)), "sm_kv_read")
        return k, v

    def prefill(self, seq: int, tokens, want_logits: bool = True):
        toks = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(self.model.cfg["vocab_size"], np.float32) if want_logits else None
        nxt = np.zeros(1, np.int32)
        L.check(L.lib().sm_prefill(self.model.handle, self.handle, seq, _p(toks), toks.size,
                                   _p(logits) if want_logits else None, _p(nxt)), "sm_prefill")
        return int(nxt[0]), logits

    def prefill_batch(self, seq_ids, prompts, want_logits: bool = True):
        """Several prompts in one pass (sm_prefill_batch): returns (next tokens [n], logits [n, vocab])."""
        s = np.ascontiguousarray(seq_ids, np.int32)
        ps = [np.asarray(p, np.int32).reshape(-1) for p in prompts]
        lens = np.array([p.size for p in ps], np.int32)
        toks = np.ascontiguousarray(np.concatenate(ps))
        n = s.size
        logits = np.empty((n, self.model.cfg["vocab_size"]), np.float32) if want_logits else None
        nxt = np.zeros(n, np.int32)
        L.check(L.lib().sm_prefill_batch(self.model.handle, self.handle, _p(s), _p(toks), _p(lens), n,
                                         _p(logits) if want_logits else None, _p(nxt)), "sm_prefill_batch")
        return nxt, logits

    def decode(self, seq_ids, tokens, want_logits: bool = True):
        s = np.ascontiguousarray(seq_ids, np.int32)
        t = np.ascontiguousarray(tokens, np.int32)
        n = s.size
        logits = np.empty((n, self.model.cfg["vocab_size"]), np.float32) if want_logits else None
        nxt = np.zeros(n, np.int32)
        L.check(L.lib().sm_decode(self.model.handle, self.handle, _p(s), _p(t), n,
                                  _p(logits) if want_logits else None, _p(nxt), L.PTR_HOST), "sm_decode")
        return nxt, logits

    def decode_device(self, seq_ptr: int, tok_ptr: int, n: int, logits_ptr: int | None, next_ptr: int | None):
        """All-device step (no host sync): inputs/outputs are device pointers."""
        L.check(L.lib().sm_decode(self.model.handle, self.handle, C.c_void_p(seq_ptr), C.c_void_p(tok_ptr), n,
                                  C.c_void_p(logits_ptr or 0), C.c_void_p(next_ptr or 0), L.PTR_DEVICE),
                "sm_decode")

    def close(self):
        if self.handle:
            L.lib().sm_kv_destroy(self.handle)
            self.handle = None


@dataclass
class SamplingOptions:
    """The sampling fields of the reference's ProductionInferenceOptions as
    InferenceSession.SampleNextToken reads them (InferenceSession.cs:565-606).
    ``seed`` set: targets come from DeterministicRng(seed) (:104-105)."""
    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 1.0
    min_p: float = 0.0
    repetition_penalty: float = 1.0
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    repetition_window: int = 0
    seed: int | None = None

    def params(self) -> L.SamplingParams:
        return L.SamplingParams(self.temperature, self.top_k, self.top_p, self.min_p, self.repetition_penalty,
                                self.presence_penalty, self.frequency_penalty, self.repetition_window)

    @property
    def penalized(self) -> bool:
        return not (self.repetition_penalty == 1.0 and self.presence_penalty == 0.0 and self.frequency_penalty == 0.0)


class DeterministicRng:
    """DeterministicRng (src/SmallMind.Core/Rng/DeterministicRng.cs): SplitMix64
    seeding of a xoroshiro128+ generator; NextDouble keeps 53 bits."""
    _M = (1 << 64) - 1

    def __init__(self, seed: int):
        s = seed & self._M  # (ulong)seed of an int: sign-extended

        def splitmix():
            nonlocal s
            s = (s + 0x9E3779B97F4A7C15) & self._M
            z = s
            z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & self._M
            z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & self._M
            return z ^ (z >> 31)

        self.s0, self.s1 = splitmix(), splitmix()
        if self.s0 == 0 and self.s1 == 0:
            self.s0 = self.s1 = 1

    def next_ulong(self) -> int:
        s0, s1 = self.s0, self.s1
        r = (s0 + s1) & self._M
        s1 ^= s0
        self.s0 = (((s0 << 24) | (s0 >> 40)) & self._M) ^ s1 ^ ((s1 << 16) & self._M)
        self.s1 = ((s1 << 37) | (s1 >> 27)) & self._M
        return r

    def next_double(self) -> float:
        return (self.next_ulong() & ((1 << 53) - 1)) * (1.0 / (1 << 53))


def sample(ctx: CudaContext, logits: np.ndarray, options: SamplingOptions, targets, context=None,
           want_probs: bool = False):
    """sm_sample over host arrays: logits [rows, vocab], targets [rows] uniform draws,
    context: per-row token histories (for the penalties).  Returns tokens (and probs)."""
    lg = np.ascontiguousarray(logits, np.float32)
    if lg.ndim == 1:
        lg = lg[None]
    rows, vocab = lg.shape
    tg = np.ascontiguousarray(np.asarray(targets, np.float64).reshape(-1))
    if tg.size != rows:
        raise ValueError("one target per row")
    ctx_arr = lens = None
    stride = 0
    if context is not None and options.penalized:
        hist = [np.asarray(c, np.int32).reshape(-1) for c in context]
        stride = max(1, max(h.size for h in hist))
        ctx_arr = np.zeros((rows, stride), np.int32)
        lens = np.zeros(rows, np.int32)
        for r, h in enumerate(hist):
            ctx_arr[r, :h.size] = h
            lens[r] = h.size
    toks = np.zeros(rows, np.int32)
    probs = np.empty((rows, vocab), np.float32) if want_probs else None
    prm = options.params()
    L.check(L.lib().sm_sample(ctx.handle, _p(lg), rows, vocab, C.byref(prm),
                              _p(ctx_arr) if ctx_arr is not None else None, _p(lens) if lens is not None else None,
                              stride, _p(tg), _p(toks), _p(probs) if want_probs else None, L.PTR_HOST), "sm_sample")
    return (toks, probs) if want_probs else toks


class InferenceSession:
    """Greedy generation loop (InferenceSession.GenerateNextTokenAsync, TopK = 1) over one sequence slot."""

    def __init__(self, kv: KVCache, seq: int = 0):
        self.kv, self.seq = kv, seq

    def generate_sampled(self, prompt_ids, max_new_tokens: int, options: SamplingOptions):
        """GenerateNextTokenAsync with the full sampling pipeline on the device
        (sm_sample); the context for the penalties is prompt + generated tokens."""
        # seed unset: the reference falls back to an unseeded System.Random (InferenceSession.cs:109)
        seed = options.seed if options.seed is not None else int.from_bytes(os.urandom(4), "little", signed=True)
        rng = DeterministicRng(seed)
        ctx = self.kv.model.ctx
        self.kv.reset(self.seq)
        context = [int(t) for t in prompt_ids]
        _, logits = self.kv.prefill(self.seq, prompt_ids, want_logits=True)
        out = []
        while True:
            t = int(sample(ctx, logits, options, [rng.next_double()], [context])[0])
            out.append(t)
            context.append(t)
            if len(out) == max_new_tokens:
                return out
            _, lg = self.kv.decode([self.seq], [t], want_logits=True)
            logits = lg[0]

    def generate(self, prompt_ids, max_new_tokens: int, return_logits: bool = False):
        self.kv.reset(self.seq)
        nxt, logits = self.kv.prefill(self.seq, prompt_ids, want_logits=return_logits)
        out, all_logits = [nxt], [logits] if return_logits else []
        for _ in range(max_new_tokens - 1):
            t, lg = self.kv.decode([self.seq], [out[-1]], want_logits=return_logits)
            out.append(int(t[0]))
            if return_logits:
                all_logits.append(lg[0])
        return (out, all_logits) if return_logits else out


def longest_common_prefix(previous, current) -> int:
    """ChatSession.CalculateLongestCommonPrefix (ChatSession.cs:1368-1383)."""
    n = 0
    for a, b in zip(previous, current):
        if a != b:
            break
        n += 1
    return n


class ChatSession:
    """Multi-turn greedy generation over one KV slot with prefix reuse.

    The reference (ChatSession.cs:270-312, 398-403) keeps a session's KV cache
    between turns and, when the new prompt's longest common prefix with the
    cached tokens covers the whole cache, prefills only the new tokens;
    otherwise it resets and prefills everything.  Here the cached tokens are
    tracked exactly (the prompt plus every generated token fed back), and a
    partial match keeps the shared prefix (``sm_kv_truncate``) instead of
    resetting.  At least one prompt token is always prefilled, so the last
    position's logits exist.  Counters mirror the reference's cache statistics.
    """

    def __init__(self, kv: KVCache, seq: int = 0, reuse: bool = True):
        self.kv, self.seq, self.reuse = kv, seq, reuse
        self.cached: list[int] = []
        self.kv_cache_hits = 0
        self.kv_cache_misses = 0
        self.tokens_from_cache = 0
        kv.reset(seq)

    def generate(self, prompt_ids, max_new_tokens: int, return_logits: bool = False):
        prompt = [int(t) for t in prompt_ids]
        keep = 0
        if self.reuse and self.cached:
            keep = min(longest_common_prefix(self.cached, prompt), len(prompt) - 1)
        if keep > 0:
            self.kv_cache_hits += 1
            self.tokens_from_cache += keep
            self.kv.truncate(self.seq, keep)
        else:
            self.kv_cache_misses += 1
            self.kv.reset(self.seq)
        nxt, logits = self.kv.prefill(self.seq, np.asarray(prompt[keep:], np.int32), want_logits=return_logits)
        self.cached = prompt[:]
        out, all_logits = [nxt], [logits] if return_logits else []
        for _ in range(max_new_tokens - 1):
            t, lg = self.kv.decode([self.seq], [out[-1]], want_logits=return_logits)
            self.cached.append(out[-1])
            out.append(int(t[0]))
            if return_logits:
                all_logits.append(lg[0])
        return (out, all_logits) if return_logits else out
