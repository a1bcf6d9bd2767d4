"""ChatSession's prefix reuse (ChatSession.cs:270-312, 398-403) as host logic, on
CPU: a fake KV cache records which tokens each turn prefills, truncates or resets,
so the bookkeeping is checked without a GPU."""
import numpy as np


class FakeKV:
    """Stands in for KVCache: tracks the token ids held by each slot."""

    def __init__(self):
        self.slots = {}
        self.log = []

    def reset(self, seq):
        self.slots[seq] = []
        self.log.append(("reset", seq))

    def truncate(self, seq, n):
        assert 0 <= n <= len(self.slots[seq])
        self.slots[seq] = self.slots[seq][:n]
        self.log.append(("truncate", seq, n))

    def prefill(self, seq, tokens, want_logits=True):
        toks = [int(t) for t in tokens]
        assert toks, "at least one token is prefilled"
        self.slots[seq] += toks
        self.log.append(("prefill", seq, len(toks)))
        return (sum(self.slots[seq]) * 7 + 3) % 101, None

    def decode(self, seq_ids, tokens, want_logits=True):
        s = int(seq_ids[0])
        self.slots[s].append(int(tokens[0]))
        return np.array([(sum(self.slots[s]) * 7 + 3) % 101]), None


def test_prefix_reuse_bookkeeping():
    from smallmind_b200.api import ChatSession
    kv = FakeKV()
    chat = ChatSession(kv, seq=2)
    p1 = [5, 6, 7, 8]
    t1 = chat.generate(p1, 3)
    assert kv.slots[2] == p1 + t1[:-1]  # the last generated token is output only
    assert (chat.kv_cache_hits, chat.kv_cache_misses) == (0, 1)
    # the whole conversation extended: only the new tokens are prefilled
    p2 = p1 + t1 + [9, 10]
    kv.log.clear()
    t2 = chat.generate(p2, 2)
    assert kv.log[0] == ("truncate", 2, len(p1) + 2) and kv.log[1] == ("prefill", 2, 3)
    assert kv.slots[2] == p2 + t2[:-1]
    assert chat.kv_cache_hits == 1 and chat.tokens_from_cache == len(p1) + 2
    # an edit in the middle keeps the shared prefix
    p3 = p2[:3] + [99, 98]
    kv.log.clear()
    chat.generate(p3, 1)
    assert kv.log[0] == ("truncate", 2, 3) and kv.log[1] == ("prefill", 2, 2)
    # nothing shared: a reset and a full prefill
    kv.log.clear()
    chat.generate([1, 2], 1)
    assert kv.log[0] == ("reset", 2) and kv.log[1] == ("prefill", 2, 2)
    assert chat.kv_cache_misses == 2
    # the same prompt again: all but its last token reused
    kv.log.clear()
    chat.generate([1, 2], 1)
    assert kv.log[0] == ("truncate", 2, 1) and kv.log[1] == ("prefill", 2, 1)


def test_reuse_off_always_resets():
    from smallmind_b200.api import ChatSession
    kv = FakeKV()
    chat = ChatSession(kv, seq=0, reuse=False)
    chat.generate([1, 2, 3], 2)
    kv.log.clear()
    chat.generate([1, 2, 3, 4], 2)
    assert kv.log[0] == ("reset", 0) and kv.log[1] == ("prefill", 0, 4)
