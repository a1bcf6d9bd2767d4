"""End-to-end parity of the device-resident LLaMA path: logits cosine >= 0.9999 with
greedy top-1 agreement on every step, against the CPU oracle and the golden fixture."""
import os

import numpy as np
import pytest

from conftest import cosine

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")

TINY = dict(vocab_size=384, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_hidden=512,
            max_context=48, norm_eps=1e-5, rope_theta=10000.0)


def _kq_schemes(O):
    return dict(wq=O.Q4_K, wk=O.Q4_K, wv=O.Q6_K, wo=O.Q4_K, w_gate=O.Q4_K, w_up=O.Q4_K, w_down=O.Q6_K,
                output=O.Q6_K)


def test_golden_tiny_model_greedy(ctx, O):
    import smallmind_b200 as sm
    g = np.load(os.path.join(GOLDEN, "tiny_llama_q4k.npz"))
    host = O.make_model(TINY, _kq_schemes(O), seed=int(g["seed"]))
    model = sm.CudaModel.from_host(ctx, host)
    kv = sm.KVCache(model, 2, 48)
    sess = sm.InferenceSession(kv, seq=1)
    toks, logits = sess.generate(g["prompt"], g["logits"].shape[0], return_logits=True)
    for step, lg in enumerate(logits):
        assert cosine(lg, g["logits"][step]) >= 0.9999
    assert toks == list(g["tokens"][len(g["prompt"]):])


@pytest.mark.parametrize("mix", ["q8", "kq"])
def test_batched_decode_matches_oracle(ctx, O, mix):
    import smallmind_b200 as sm
    cfg = dict(TINY, n_heads=9, n_kv_heads=3, hidden=576, ffn_hidden=512, vocab_size=400, max_context=40)
    if mix == "q8":
        schemes = {k: O.Q8_0 for k in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down", "output")}
        cfg = dict(cfg, hidden=576)
    else:
        cfg = dict(cfg, hidden=512, n_heads=8, n_kv_heads=2)
        schemes = _kq_schemes(O)
    host = O.make_model(cfg, schemes, seed=11, block_size=64)
    model = sm.CudaModel.from_host(ctx, host)
    kv = sm.KVCache(model, 4, 40)
    rs = np.random.RandomState(0)
    prompts = [rs.randint(0, cfg["vocab_size"], n).astype(np.int32) for n in (5, 9, 1, 13)]
    hist = []
    nxt = []
    for s, p in enumerate(prompts):
        t, lg = kv.prefill(s, p)
        ref = O.model_forward(host, p, 1)[0]
        assert cosine(lg, ref) >= 0.9999 and t == int(np.argmax(ref))
        hist.append(list(p) + [t])
        nxt.append(t)
    order = [2, 0, 3, 1]  # batch rows in a different order than the slots
    for step in range(4):
        toks, lg = kv.decode(order, [nxt[s] for s in order])
        for row, s in enumerate(order):
            ref = O.model_forward(host, np.array(hist[s], np.int32), 1)[0]
            assert cosine(lg[row], ref) >= 0.9999
            assert int(toks[row]) == int(np.argmax(ref))
            hist[s].append(int(toks[row]))
            nxt[s] = int(toks[row])
    for s in range(4):
        assert kv.length(s) == len(hist[s]) - 1


def test_graph_and_eager_agree_and_limits(ctx, O, monkeypatch):
    import smallmind_b200 as sm
    host = O.make_model(TINY, _kq_schemes(O), seed=3)
    model = sm.CudaModel.from_host(ctx, host)
    prompt = np.arange(7, dtype=np.int32)
    outs = []
    for graphs in ("1", "0"):
        monkeypatch.setenv("SMALLMIND_CUDA_GRAPHS", graphs)
        kv = sm.KVCache(model, 1, 12)
        out = sm.InferenceSession(kv).generate(prompt, 5)
        outs.append(out)
        # prefill 7 + 4 decodes = 11 cached; one more fills the 12-token context, the next is refused
        kv.decode([0], [out[-1]])
        with pytest.raises(ValueError):
            kv.decode([0], [out[-1]])
        kv.close()
    assert outs[0] == outs[1]
    kv = sm.KVCache(model, 1, 12)
    with pytest.raises(ValueError):
        kv.prefill(0, np.zeros(13, np.int32))  # Sequence length exceeds block size (TransformerModel.cs:280-283)
    with pytest.raises(ValueError):
        kv.prefill(0, np.array([TINY["vocab_size"]], np.int32))
    with pytest.raises(ValueError):
        kv.decode([0, 0], [1, 2])  # the same sequence twice in one step


def test_device_mode_decode_loop(ctx, O):
    """All-device greedy loop (tokens fed back on the GPU) equals the host loop."""
    import torch

    import smallmind_b200 as sm
    host = O.make_model(TINY, _kq_schemes(O), seed=21)
    model = sm.CudaModel.from_host(ctx, host)
    prompt = np.array([3, 1, 4, 1, 5], np.int32)
    ref = sm.InferenceSession(sm.KVCache(model, 1, 30)).generate(prompt, 8)
    kv = sm.KVCache(model, 1, 30)
    t0, _ = kv.prefill(0, prompt, want_logits=False)
    seq = torch.zeros(1, dtype=torch.int32, device="cuda")
    tok = torch.tensor([t0], dtype=torch.int32, device="cuda")
    nxt = torch.empty(1, dtype=torch.int32, device="cuda")
    got = [t0]
    torch.cuda.synchronize()
    for _ in range(7):
        kv.decode_device(seq.data_ptr(), tok.data_ptr(), 1, None, nxt.data_ptr())
        ctx.sync()
        got.append(int(nxt.item()))
        tok.copy_(nxt)
        torch.cuda.synchronize()
    assert got == ref
    assert kv.length(0) == len(prompt) + 7


@pytest.mark.parametrize("n_prompt", [40, 160])
def test_long_prefill_tensor_core_path(ctx, O, n_prompt):
    # prompts of >= 16 rows run the tcgen05 GEMMs (Q|K|V and gate|up as one stacked-weight
    # GEMM each; > 128 rows through the fp16 weight planes) and the tcgen05 prefill attention
    import smallmind_b200 as sm
    cfg = dict(TINY, max_context=200)
    host = O.make_model(cfg, _kq_schemes(O), seed=5)
    model = sm.CudaModel.from_host(ctx, host)
    kv = sm.KVCache(model, 1, 200)
    prompt = np.random.RandomState(n_prompt).randint(0, cfg["vocab_size"], n_prompt).astype(np.int32)
    t, lg = kv.prefill(0, prompt)
    ref = O.model_forward(host, prompt, 1)[0]
    assert cosine(lg, ref) >= 0.9999 and t == int(np.argmax(ref))
    # one decode step on top of the long prefix
    toks, lg2 = kv.decode([0], [t])
    ref2 = O.model_forward(host, np.append(prompt, t).astype(np.int32), 1)[0]
    assert cosine(lg2[0], ref2) >= 0.9999 and int(toks[0]) == int(np.argmax(ref2))


def test_batched_decode_20_sequences(ctx, O):
    # 20 rows per decode step: the batched forward runs the tcgen05 GEMM with split K
    import smallmind_b200 as sm
    cfg = dict(TINY, max_context=24)
    host = O.make_model(cfg, _kq_schemes(O), seed=8)
    model = sm.CudaModel.from_host(ctx, host)
    n = 20
    kv = sm.KVCache(model, n, 24)
    rs = np.random.RandomState(4)
    hist, nxt = [], []
    for s in range(n):
        p = rs.randint(0, cfg["vocab_size"], 3 + s % 5).astype(np.int32)
        t, _ = kv.prefill(s, p, want_logits=False)
        hist.append(list(p) + [t])
        nxt.append(t)
    toks, lg = kv.decode(list(range(n)), nxt)
    for s in range(n):
        ref = O.model_forward(host, np.array(hist[s], np.int32), 1)[0]
        assert cosine(lg[s], ref) >= 0.9999
        assert int(toks[s]) == int(np.argmax(ref))


def test_q8_model_hidden_576_bs1_decode_matches_oracle(ctx, O):
    """SmolLM-shaped widths (hidden 576 = 18 units, 9 q / 3 kv heads), bs1 greedy decode."""
    import smallmind_b200 as sm
    cfg = dict(TINY, hidden=576, n_heads=9, n_kv_heads=3, ffn_hidden=1536, vocab_size=400, max_context=40)
    schemes = {k: O.Q8_0 for k in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down", "output")}
    host = O.make_model(cfg, schemes, seed=21, block_size=64)
    model = sm.CudaModel.from_host(ctx, host)
    kv = sm.KVCache(model, 1, 40)
    prompt = np.random.RandomState(4).randint(0, cfg["vocab_size"], 11).astype(np.int32)
    toks, logits = sm.InferenceSession(kv).generate(prompt, 5, return_logits=True)
    hist = list(prompt)
    for step, lg in enumerate(logits):
        ref = O.model_forward(host, np.array(hist, np.int32), 1)[0]
        assert cosine(lg, ref) >= 0.9999, step
        assert toks[step] == int(np.argmax(ref)), step
        hist.append(toks[step])
