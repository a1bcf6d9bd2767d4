"""Tensor-parallel decode: one model split over a group of GPUs (one process each).

Which projection is split how (the reference runs one CPU process and has no
such split; the projections are those of MultiHeadAttention.cs:92-93 and
GatedMLP.cs:38-40):

* column-split (output rows): Wq and Wk / Wv by heads, gate and up by FFN units;
* row-split (input columns, whole 256-weight blocks): Wo over the rank's q heads,
  down over the rank's FFN units; after each, the ranks all-reduce their partial
  outputs before the residual add (``sm_model_set_tp``);
* replicated: token embedding, RMSNorm weights, final norm and LM head, so every
  rank produces the same logits.

With more ranks than kv heads, ranks whose q heads share a kv head each keep a
copy of it.  Packed weights are sliced as bytes: rows of the INTENDED layout are
contiguous, and a column range of whole blocks is a byte range of every row
(plus the matching slice of the per-block scales for Q8_0 / Q4_0).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib as L
from .api import QuantScheme

# bytes per 256 weights of the block formats, and block granularity of a column slice
_KQ_BYTES = {int(QuantScheme.Q4_K): 144, int(QuantScheme.Q6_K): 210}


@dataclass
class PackedWeight:
    """A packed weight in the reference layout (the fields CudaWeightTensor.from_qtensor reads)."""
    scheme: int
    rows: int
    cols: int
    data: np.ndarray
    scales: np.ndarray | None = None
    block_size: int = 256


@dataclass
class ShardModel:
    """One rank's model: the same fields CudaModel.from_host reads."""
    cfg: dict
    token_embd: np.ndarray
    out_norm: np.ndarray
    output: object
    layers: list = field(default_factory=list)
    tp_size: int = 1
    tp_rank: int = 0


def even_split(n: int, parts: int, rank: int) -> tuple[int, int]:
    """[lo, hi) of rank's share when n units are split as evenly as possible (first ranks get one more)."""
    if parts <= 0 or not 0 <= rank < parts:
        raise ValueError(f"bad rank {rank} of {parts}")
    base, extra = divmod(n, parts)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def _row_bytes(w) -> int:
    s = int(w.scheme)
    if s in _KQ_BYTES:
        return w.cols // 256 * _KQ_BYTES[s]
    if s == QuantScheme.Q8_0:
        return w.cols
    if s == QuantScheme.Q4_0:
        return w.cols // 2
    if s == QuantScheme.F32:
        return 4 * w.cols
    raise NotImplementedError(f"tensor-parallel slicing of {QuantScheme(s).name} weights")


def _col_unit(w) -> int:
    """Smallest column slice that keeps whole blocks (and byte boundaries)."""
    s = int(w.scheme)
    if s in _KQ_BYTES:
        return 256
    if s in (QuantScheme.Q8_0, QuantScheme.Q4_0):
        if w.cols % w.block_size:
            raise NotImplementedError("Q8_0 / Q4_0 blocks that straddle rows")
        return w.block_size
    return 1


def slice_rows(w, r0: int, r1: int) -> PackedWeight:
    """Output rows [r0, r1) of a packed INTENDED-layout weight."""
    if not 0 <= r0 < r1 <= w.rows:
        raise ValueError(f"row range [{r0}, {r1}) outside {w.rows} rows")
    rb = _row_bytes(w)
    data = np.ascontiguousarray(np.asarray(w.data).view(np.uint8).reshape(w.rows, rb)[r0:r1]).reshape(-1)
    scales = None
    if w.scales is not None and int(w.scheme) in (QuantScheme.Q8_0, QuantScheme.Q4_0):
        per_row = w.cols // w.block_size
        scales = np.ascontiguousarray(np.asarray(w.scales, np.float32).reshape(w.rows, per_row)[r0:r1]).reshape(-1)
    return PackedWeight(int(w.scheme), r1 - r0, w.cols, data, scales, w.block_size)


def slice_cols(w, c0: int, c1: int) -> PackedWeight:
    """Input columns [c0, c1) (whole blocks) of a packed INTENDED-layout weight."""
    unit = _col_unit(w)
    if c0 % unit or c1 % unit or not 0 <= c0 < c1 <= w.cols:
        raise ValueError(f"column range [{c0}, {c1}) is not whole {unit}-column blocks of {w.cols}")
    rb = _row_bytes(w)
    b0, b1 = c0 * rb // w.cols, c1 * rb // w.cols
    data = np.ascontiguousarray(np.asarray(w.data).view(np.uint8).reshape(w.rows, rb)[:, b0:b1]).reshape(-1)
    scales = None
    if w.scales is not None and int(w.scheme) in (QuantScheme.Q8_0, QuantScheme.Q4_0):
        per_row = w.cols // w.block_size
        sc = np.asarray(w.scales, np.float32).reshape(w.rows, per_row)
        scales = np.ascontiguousarray(sc[:, c0 // w.block_size:c1 // w.block_size]).reshape(-1)
    return PackedWeight(int(w.scheme), w.rows, c1 - c0, data, scales, w.block_size)


def head_ranges(n_heads: int, n_kv: int, tp: int, rank: int) -> tuple[tuple[int, int], tuple[int, int]]:
    """(q heads [lo, hi), kv heads [lo, hi)) of a rank.  q heads split evenly (n_heads % tp == 0);
    kv heads split when n_kv % tp == 0, else (tp % n_kv == 0) each rank keeps the one its q heads read."""
    if n_heads % tp:
        raise ValueError(f"{n_heads} q heads do not split over {tp} ranks")
    q0, q1 = rank * n_heads // tp, (rank + 1) * n_heads // tp
    group = n_heads // n_kv
    k0, k1 = q0 // group, (q1 - 1) // group + 1
    whole = q0 % group == 0 and (q1 - q0) % group == 0   # whole kv groups: kv heads split
    inside = k1 - k0 == 1                               # part of one kv group: that kv head copied
    if not (whole or inside):
        raise ValueError(f"{n_heads} q / {n_kv} kv heads cannot be split over {tp} ranks")
    return (q0, q1), (k0, k1)


def ffn_range(ffn: int, tp: int, rank: int, unit: int = 256) -> tuple[int, int]:
    """FFN units [lo, hi) of a rank, in whole `unit`-column blocks of the down projection."""
    if ffn % unit:
        raise ValueError(f"FFN width {ffn} is not whole {unit}-column blocks")
    b0, b1 = even_split(ffn // unit, tp, rank)
    if b1 <= b0:
        raise ValueError(f"{tp} ranks leave rank {rank} without FFN blocks")
    return b0 * unit, b1 * unit


def shard_model(host, tp: int, rank: int) -> ShardModel:
    """This rank's shard of a packed host model (cfg, token_embd, out_norm, output,
    layers[...] dicts of wq..w_down, attn_norm, ffn_norm)."""
    c = dict(host.cfg)
    hd = c["head_dim"]
    (q0, q1), (k0, k1) = head_ranges(c["n_heads"], c["n_kv_heads"], tp, rank)
    unit = 256 if int(host.layers[0]["w_down"].scheme) in _KQ_BYTES else max(
        1, getattr(host.layers[0]["w_down"], "block_size", 32))
    f0, f1 = ffn_range(c["ffn_hidden"], tp, rank, unit)
    cfg = dict(c, n_heads=q1 - q0, n_kv_heads=k1 - k0, ffn_hidden=f1 - f0)
    layers = []
    for L_ in host.layers:
        layers.append({
            "attn_norm": L_["attn_norm"], "ffn_norm": L_["ffn_norm"],
            "wq": slice_rows(L_["wq"], q0 * hd, q1 * hd),
            "wk": slice_rows(L_["wk"], k0 * hd, k1 * hd),
            "wv": slice_rows(L_["wv"], k0 * hd, k1 * hd),
            "wo": slice_cols(L_["wo"], q0 * hd, q1 * hd),
            "w_gate": slice_rows(L_["w_gate"], f0, f1),
            "w_up": slice_rows(L_["w_up"], f0, f1),
            "w_down": slice_cols(L_["w_down"], f0, f1),
        })
    return ShardModel(cfg, host.token_embd, host.out_norm, host.output, layers, tp, rank)


class TensorParallelGroup:
    """Joins a CudaContext to a tensor-parallel group; the 128-byte id travels over
    the default torch.distributed process group (any backend)."""

    def __init__(self, ctx, tp: int, rank: int):
        import torch
        import torch.distributed as dist
        buf = (C.c_uint8 * 128)()
        if rank == 0:
            L.check(L.lib().sm_tp_unique_id(buf, 128), "sm_tp_unique_id")
        if tp > 1:
            obj = [bytes(buf) if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            C.memmove(buf, obj[0], 128)
        torch.cuda.synchronize()
        L.check(L.lib().sm_tp_init(ctx.handle, tp, rank, buf, 128), "sm_tp_init")
        self.ctx, self.tp, self.rank = ctx, tp, rank

    def allreduce_(self, ptr: int, n: int) -> None:
        """In-place float32 sum of n elements at device pointer ptr, on the context stream."""
        L.check(L.lib().sm_tp_allreduce(self.ctx.handle, C.c_void_p(ptr), n), "sm_tp_allreduce")

    def shard(self, model) -> None:
        """Marks a CudaModel built from this rank's shard as tensor-parallel."""
        L.check(L.lib().sm_model_set_tp(model.handle, 1), "sm_model_set_tp")
