"""Session reuse over the HBM KV cache: prefix reuse across turns (ChatSession.cs:270-312),
KvCacheEntry.Slide / GetKeys / GetValues (KvCacheEntry.cs:155-229).

A turn that reuses the cached prefix prefills only the new tokens at their
positions (prefill with a non-zero offset); its logits must match the oracle's
full recompute of the whole history (cosine >= 0.9999, same greedy tokens)."""
import numpy as np
import pytest

from conftest import cosine

pytestmark = pytest.mark.gpu

CFG = dict(vocab_size=384, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_hidden=512,
           max_context=96, norm_eps=1e-5, rope_theta=10000.0)


def _model(ctx, O):
    import smallmind_b200 as sm
    schemes = dict(wq=O.Q4_K, wk=O.Q4_K, wv=O.Q6_K, wo=O.Q4_K, w_gate=O.Q4_K, w_up=O.Q4_K, w_down=O.Q6_K,
                   output=O.Q6_K)
    host = O.make_model(CFG, schemes, seed=21)
    return host, sm.CudaModel.from_host(ctx, host)


def _check_turn(O, host, history, toks, logits):
    hist = list(history)
    for step, lg in enumerate(logits):
        ref = O.model_forward(host, np.array(hist, np.int32), 1)[0]
        assert cosine(lg, ref) >= 0.9999, step
        assert toks[step] == int(np.argmax(ref)), step
        hist.append(toks[step])


def test_lcp_helper():
    import smallmind_b200 as sm
    assert sm.longest_common_prefix([1, 2, 3], [1, 2, 4, 5]) == 2
    assert sm.longest_common_prefix([], [1]) == 0
    assert sm.longest_common_prefix([1, 2], [1, 2, 3]) == 2


def test_chat_turns_reuse_prefix_and_match_full_recompute(ctx, O):
    import smallmind_b200 as sm
    host, model = _model(ctx, O)
    kv = sm.KVCache(model, 2, 96)
    chat = sm.ChatSession(kv, seq=1)
    rs = np.random.RandomState(4)
    p1 = list(rs.randint(0, CFG["vocab_size"], 11))
    t1, lg1 = chat.generate(p1, 4, return_logits=True)
    _check_turn(O, host, p1, t1, lg1)
    assert (chat.kv_cache_hits, chat.kv_cache_misses) == (0, 1)
    # turn 2 extends the whole conversation: only the new tokens are prefilled
    p2 = p1 + t1 + list(rs.randint(0, CFG["vocab_size"], 6))
    t2, lg2 = chat.generate(p2, 4, return_logits=True)
    _check_turn(O, host, p2, t2, lg2)
    assert chat.kv_cache_hits == 1 and chat.tokens_from_cache == len(p1) + 3
    assert kv.length(1) == len(p2) + 3
    # turn 3 edits the middle of the history: the shared prefix is kept, the rest recomputed
    p3 = p2[:8] + list(rs.randint(0, CFG["vocab_size"], 5))
    t3, lg3 = chat.generate(p3, 3, return_logits=True)
    _check_turn(O, host, p3, t3, lg3)
    assert chat.kv_cache_hits == 2 and chat.tokens_from_cache == len(p1) + 3 + 8
    # turn 4 shares nothing: full prefill
    p4 = [int((p3[0] + 1) % CFG["vocab_size"])] + p3[1:4]
    t4, lg4 = chat.generate(p4, 2, return_logits=True)
    _check_turn(O, host, p4, t4, lg4)
    assert chat.kv_cache_misses == 2
    # the same prompt again: all but its last token come from the cache
    t5, lg5 = chat.generate(p4, 2, return_logits=True)
    assert t5 == t4 and all(cosine(a, b) >= 0.9999 for a, b in zip(lg5, lg4))
    kv.close()
    model.close()


def test_kv_read_slide_truncate(ctx, O):
    import smallmind_b200 as sm
    host, model = _model(ctx, O)
    kv = sm.KVCache(model, 3, 96)
    rs = np.random.RandomState(9)
    kv.prefill(2, rs.randint(0, CFG["vocab_size"], 70).astype(np.int32), want_logits=False)
    kv.prefill(0, rs.randint(0, CFG["vocab_size"], 5).astype(np.int32), want_logits=False)
    before = [kv.read(l, 2, 0, 70) for l in range(CFG["n_layers"])]
    other = [kv.read(l, 0, 0, 5) for l in range(CFG["n_layers"])]
    # reads of sub-ranges agree with the full read
    k, v = kv.read(1, 2, 13, 20)
    assert np.array_equal(k, before[1][0][13:33]) and np.array_equal(v, before[1][1][13:33])
    with pytest.raises(Exception):
        kv.read(0, 2, 60, 11)  # past the cached tokens (KvCacheEntry.cs:162-163)
    with pytest.raises(Exception):
        kv.slide(2, -1)  # KvCacheEntry.cs:205-206
    kv.slide(2, 80)  # window >= length: nothing moves
    assert kv.length(2) == 70
    kv.slide(2, 50)  # overlapping move (start 20 < keep 50)
    assert kv.length(2) == 50
    for l in range(CFG["n_layers"]):
        k, v = kv.read(l, 2, 0, 50)
        assert np.array_equal(k, before[l][0][20:]) and np.array_equal(v, before[l][1][20:])
        k0, v0 = kv.read(l, 0, 0, 5)  # the other sequence is untouched
        assert np.array_equal(k0, other[l][0]) and np.array_equal(v0, other[l][1])
    kv.slide(2, 7)  # non-overlapping move
    for l in range(CFG["n_layers"]):
        k, v = kv.read(l, 2, 0, 7)
        assert np.array_equal(k, before[l][0][63:]) and np.array_equal(v, before[l][1][63:])
    kv.truncate(2, 3)
    assert kv.length(2) == 3
    with pytest.raises(Exception):
        kv.truncate(2, 4)
    kv.slide(2, 0)
    assert kv.length(2) == 0
    kv.close()
    model.close()


def test_prefill_batch_matches_oracle(ctx, O):
    """Several prompts in one pass (sm_prefill_batch), ragged lengths, slots in any
    order, one slot already holding context: each prompt's last-position logits
    and the greedy decode that follows match the oracle's full recompute."""
    import smallmind_b200 as sm
    host, model = _model(ctx, O)
    kv = sm.KVCache(model, 5, 96)
    rs = np.random.RandomState(12)
    V = CFG["vocab_size"]
    pre = list(rs.randint(0, V, 6))
    kv.prefill(3, np.array(pre, np.int32), want_logits=False)
    seqs = [4, 0, 3, 2]
    prompts = [list(rs.randint(0, V, n)) for n in (9, 1, 5, 17)]
    nxt, logits = kv.prefill_batch(seqs, prompts)
    hist = {}
    for i, s in enumerate(seqs):
        h = (pre if s == 3 else []) + prompts[i]
        ref = O.model_forward(host, np.array(h, np.int32), 1)[0]
        assert cosine(logits[i], ref) >= 0.9999, s
        assert nxt[i] == int(np.argmax(ref)), s
        hist[s] = h + [int(nxt[i])]
        assert kv.length(s) == len(h)
    # decode all four together from there
    toks = [hist[s][-1] for s in seqs]
    for step in range(3):
        t, lg = kv.decode(seqs, toks)
        for i, s in enumerate(seqs):
            ref = O.model_forward(host, np.array(hist[s], np.int32), 1)[0]
            assert cosine(lg[i], ref) >= 0.9999 and t[i] == int(np.argmax(ref)), (step, s)
            hist[s].append(int(t[i]))
        toks = [int(x) for x in t]
    with pytest.raises(Exception):
        kv.prefill_batch([1, 1], [[1, 2], [3]])  # a slot twice
    with pytest.raises(Exception):
        kv.prefill_batch([1], [list(range(100))])  # past the slot's capacity
    kv.close()
    model.close()
