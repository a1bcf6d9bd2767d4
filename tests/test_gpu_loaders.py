"""A GGUF / SMQ file -> device model -> greedy decode, against the oracle model
built from the same (converted) tensors.  Logits cosine >= 0.9999 and the same
greedy tokens at every step (the model-level parity bar)."""
import os
import sys

import numpy as np
import pytest

from conftest import cosine

sys.path.insert(0, os.path.dirname(__file__))
import gguf_fixture as G  # noqa: E402

pytestmark = pytest.mark.gpu

CFG = dict(vocab_size=384, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_hidden=512,
           max_context=48, norm_eps=1e-5, rope_theta=10000.0)


def _oracle_model(O, L, tensors, cfg):
    """The oracle HostModel from loader tensors (reference layouts, no requantization)."""
    def q(t):
        return O.QTensor(int(t.scheme), t.rows, t.cols, t.data, t.scales, t.block_size or 256)
    layers = []
    for li in range(cfg["n_layers"]):
        p = f"blk.{li}."
        layers.append({"attn_norm": tensors[p + "attn_norm.weight"].floats().copy(),
                       "ffn_norm": tensors[p + "ffn_norm.weight"].floats().copy(),
                       "wq": q(tensors[p + "attn_q.weight"]), "wk": q(tensors[p + "attn_k.weight"]),
                       "wv": q(tensors[p + "attn_v.weight"]), "wo": q(tensors[p + "attn_output.weight"]),
                       "w_gate": q(tensors[p + "ffn_gate.weight"]), "w_up": q(tensors[p + "ffn_up.weight"]),
                       "w_down": q(tensors[p + "ffn_down.weight"])})
    emb = tensors["token_embd.weight"].floats().reshape(cfg["vocab_size"], cfg["hidden"]).copy()
    return O.HostModel(dict(cfg), emb, tensors["output_norm.weight"].floats().copy(),
                       q(tensors["output.weight"]), layers)


TYPES = {"kquant": None,
         "q4_1": dict(q=G.Q4_1, k=G.Q4_1, v=G.Q4_1, o=G.Q4_1, gate=G.Q4_1, up=G.Q4_1, down=G.Q4_1, output=G.Q4_1),
         "q5_0": dict(q=G.Q5_0, k=G.Q5_0, v=G.Q5_0, o=G.Q5_0, gate=G.Q5_0, up=G.Q5_0, down=G.Q5_0, output=G.Q5_0),
         "mixed": dict(q=G.Q5_0, k=G.Q5_0, v=G.Q8_0, o=G.F16, gate=G.Q4_1, up=G.Q4_1, down=G.Q5_0, output=G.Q4_0)}


@pytest.mark.parametrize("via,types", [("gguf", "kquant"), ("smq", "kquant"), ("gguf", "q4_1"), ("smq", "q5_0"),
                                       ("gguf", "mixed"), ("smq", "mixed")])
def test_file_model_greedy_matches_oracle(ctx, O, tmp_path, via, types):
    import smallmind_b200 as sm
    from smallmind_b200 import loaders as L
    gp = tmp_path / "tiny.gguf"
    G.tiny_llama_gguf(gp, CFG, types=TYPES[types])
    g = L.gguf_read(gp)
    tensors = {t.name: L.gguf_tensor_to_host(g, t) for t in g.tensors}
    if via == "gguf":
        model, meta = L.load_gguf_model(ctx, gp)
    else:
        sp = tmp_path / "tiny.smq"
        L.gguf_import_to_smq(gp, sp)
        model, meta = L.load_smq_model(ctx, sp)
    assert {k: v for k, v in model.cfg.items() if k != "norm_eps"} == {k: v for k, v in CFG.items() if k != "norm_eps"}
    assert abs(model.cfg["norm_eps"] - CFG["norm_eps"]) < 1e-9
    host = _oracle_model(O, L, tensors, CFG)
    kv = sm.KVCache(model, 1, 40)
    prompt = np.random.RandomState(1).randint(0, CFG["vocab_size"], 9).astype(np.int32)
    toks, logits = sm.InferenceSession(kv).generate(prompt, 4, return_logits=True)
    hist = list(prompt)
    for step, lg in enumerate(logits):
        ref = O.model_forward(host, np.array(hist, np.int32), 1)[0]
        assert cosine(lg, ref) >= 0.9999, step
        assert toks[step] == int(np.argmax(ref)), step
        hist.append(toks[step])
    kv.close()
    model.close()
