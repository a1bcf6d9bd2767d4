"""Generates tests/golden/*.npz from the CPU oracle (run once; outputs are committed).

The reference (C#/.NET) cannot run in this environment, so these vectors come
from the oracle, a restatement of the reference arithmetic that is itself
pinned by tests/test_oracle_golden.py against the reference's own
known-answer tests.  They freeze the packed bytes, the bit-exact dequantized
values and the matmul outputs so the GPU parity tests compare against fixed
data, independent of later oracle edits.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402

NAMES = {O.Q8_0: "q8_0", O.Q4_0: "q4_0", O.Q4_K: "q4_k", O.Q6_K: "q6_k"}


def main():
    rows, cols, m = 24, 512, 3
    for scheme, name in NAMES.items():
        x = O.fill_normal(rows * cols, 1000 + scheme, 0.02)
        bs = 32
        t = O.quantize(x, scheme, rows, cols, bs)
        deq = O.dequantize(t).reshape(-1)
        a = np.random.RandomState(scheme).randn(m, cols).astype(np.float32)
        y_int = O.matmul(t, a, m, cols, rows, mode=1)
        out = dict(scheme=scheme, rows=rows, cols=cols, block_size=bs, source=x, data=t.data, dequant=deq, a=a,
                   y_intended=y_int)
        if t.scales is not None:
            out["scales"] = t.scales
        # reference-literal orientation: B = K x N; K-quant blocks (k/256)*N + n
        if scheme in (O.Q4_K, O.Q6_K):
            # the reference's Q4KTensor/Q6KTensor need Cols (= N here) % 256 == 0 too
            lk, ln = 512, 256
            tl = O.quantize(O.fill_normal(ln * lk, 2000 + scheme, 0.02), scheme, ln, lk)
            lit = O.reorder_kquant_blocks_to_literal(tl)
            a3 = np.random.RandomState(20 + scheme).randn(m, lk).astype(np.float32)
            out.update(literal_data=lit.data, a_literal=a3, lit_k=lk, lit_n=ln,
                       y_literal=O.matmul(lit, a3, m, lk, ln, mode=0))
        else:
            # literal B[K][N] with the same bytes read as a K x N tensor (rows=cols_int, cols=rows_int)
            a2 = np.random.RandomState(10 + scheme).randn(m, rows).astype(np.float32)
            lit = O.QTensor(scheme, rows, cols, t.data, t.scales, bs)
            out["a_literal"] = a2
            out["y_literal"] = O.matmul(lit, a2, m, rows, cols, mode=0)
        np.savez_compressed(os.path.join(HERE, f"quant_{name}.npz"), **out)

    # tiny LLaMA-shaped model: the logits of a greedy continuation
    cfg = dict(vocab_size=384, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_hidden=512,
               max_context=48, norm_eps=1e-5, rope_theta=10000.0)
    schemes = dict(wq=O.Q4_K, wk=O.Q4_K, wv=O.Q6_K, wo=O.Q4_K, w_gate=O.Q4_K, w_up=O.Q4_K, w_down=O.Q6_K,
                   output=O.Q6_K)
    host = O.make_model(cfg, schemes, seed=4242)
    prompt = np.random.RandomState(5).randint(0, cfg["vocab_size"], 10).astype(np.int32)
    toks = list(prompt)
    logits = []
    for _ in range(4):
        lg = O.model_forward(host, np.array(toks, np.int32), 1)[0]
        logits.append(lg)
        toks.append(int(np.argmax(lg)))
    np.savez_compressed(os.path.join(HERE, "tiny_llama_q4k.npz"), prompt=prompt, tokens=np.array(toks, np.int32),
                        logits=np.stack(logits), seed=4242)


if __name__ == "__main__":
    main()
