"""`NativeEngine`'s run loop on the CPU, over a fake engine whose greedy token is a function of the
whole sequence: the reference engine's run semantics (`qwen_vk.cpp:588-613`) — every sampled token
emitted and counted, the stop token with empty text; the last sampled token kept in the session
unprocessed (state: position = processed + 1) and processed first by the next request; text still
held by the incremental decoder flushed as a token -1 line; decode_tok_s = generated / decode_s;
the chat turn layout of `qwen_vk.cpp:615-620`; numeric stop entries; `special=False` tokenizing."""
import pytest
import torch

from seedplane_b200 import native as nat

V = 97


def f(seq):
    return (sum(seq) * 31 + 7 * len(seq)) % V


class FakeKV:
    def __init__(self, capacity):
        self.capacity, self.length, self.cache = capacity, 0, []

    def close(self):
        pass


class FakeEngine:
    device = torch.device("cpu")
    cfg = type("C", (), {"vocab": V, "max_positions": 4096})()

    def new_kv(self, capacity):
        return FakeKV(capacity)

    def forward(self, kv, ids, positions=None, want_logits=False, last_only=False):
        ids = [int(t) for t in ids]
        del kv.cache[kv.length:]
        out = []
        for t in ids:
            kv.cache.append(t)
            out.append(f(kv.cache))
        kv.length = len(kv.cache)
        return None, torch.tensor(out)

    def decode(self, kv, token, pos, n, want_logits=False):
        assert pos == kv.length
        out = []
        for _ in range(n):
            _, am = self.forward(kv, [token])
            token = int(am[-1])
            out.append(token)
        return torch.tensor(out), None


class FakeTok:
    """id 90: an open multi-byte character (decodes to U+FFFD until 91 closes it); 95: special."""

    def __init__(self):
        self.encode_special_tokens = False

    def decode(self, ids, skip_special_tokens=True):
        s = ""
        for i in ids:
            if i == 95 and skip_special_tokens:
                continue
            s = s[:-1] + "é" if (i == 91 and s.endswith("�")) else s + ("�" if i == 90 else chr(65 + i % 26))
        return s

    def token_to_id(self, text):
        return {"<|im_end|>": 95, "<|endoftext|>": 96}.get(text)

    def encode(self, text, add_special_tokens=False):
        class E:
            pass
        e = E()
        if self.encode_special_tokens:
            e.ids = [ord(c) % 90 for c in text]
        else:
            e.ids = [95 if c == "|" else ord(c) % 90 for c in text]
        return e


def bare(tok=None, capacity=64, engine=None):
    eng = nat.NativeEngine.__new__(nat.NativeEngine)
    eng.cfg = type("C", (), {"vocab": V})()
    eng._engine, eng._tok = engine or FakeEngine(), tok
    eng._session = nat.WindowSession(eng._engine, "full", None, capacity)
    eng.capacity = capacity
    eng._stop_ids = {95, 96} if tok is not None else set()
    eng.defaults = {"temperature": None, "top_k": None, "top_p": None, "seed": None, "max_new_tokens": 256}
    eng.system = nat.DEFAULT_SYSTEM
    eng.last, eng.last_tokens, eng.on_token, eng.bundle = None, [], None, "fake"
    return eng


def greedy(seq, n):
    seq, out = list(seq), []
    for _ in range(n):
        out.append(f(seq))
        seq.append(out[-1])
    return out


def test_length_run_keeps_the_last_token_unprocessed():
    eng = bare()
    prompt = [3, 1, 4, 1, 5]
    list(eng.generate(ids=prompt, max_new_tokens=40))
    assert eng.last_tokens == greedy(prompt, 40)
    last = eng.last
    assert last["reason"] == "length" and last["generated"] == 40 and last["position"] == len(prompt) + 40
    assert last["decode_tok_s"] == pytest.approx(40 / max(last["decode_s"], 1e-9))
    st = eng.state()
    assert st["position"] == len(prompt) + 40 and st["processed"] == len(prompt) + 39
    assert st["tokens"] == prompt + greedy(prompt, 40)


def test_stop_token_is_emitted_counted_and_processed_by_the_next_request():
    eng = bare()
    prompt = [2, 7, 1, 8]
    want = greedy(prompt, 30)
    k = 6
    seen = []
    eng.on_token = lambda t, piece: seen.append((t, piece))
    list(eng.generate(ids=prompt, max_new_tokens=30, stop=[float(want[k])]))   # a JSON float stop entry
    j = want.index(want[k])
    assert eng.last_tokens == want[:j + 1] and [t for t, _ in seen] == want[:j + 1]
    assert seen[-1] == (want[j], "") and eng.last["reason"] == "stop" and eng.last["generated"] == j + 1
    st = eng.state()
    assert st["tokens"] == prompt + want[:j + 1] and st["processed"] == len(prompt) + j
    more = [11, 12]
    list(eng.generate(ids=more, reset=False, max_new_tokens=5))
    assert eng.last_tokens == greedy(prompt + want[:j + 1] + more, 5)
    assert eng.state()["processed"] == len(prompt) + j + 1 + len(more) + 4


def test_decoder_flush_is_a_token_minus_one_emission():
    s = nat._TextStream(FakeTok())
    assert s.push(90) == "" and s.push(91) == "é" and s.flush() == ""

    class OpenChars(FakeEngine):        # every greedy token opens a character that never closes
        def forward(self, kv, ids, positions=None, want_logits=False, last_only=False):
            _, am = super().forward(kv, ids, positions, want_logits)
            return None, torch.full_like(am, 90)

    eng = bare(FakeTok(), engine=OpenChars())
    seen = []
    eng.on_token = lambda t, piece: seen.append((t, piece))
    pieces = list(eng.generate(ids=[1, 2, 3], max_new_tokens=4))
    assert seen == [(90, "")] * 4 + [(-1, "����")] and pieces == ["����"]
    assert eng.last_tokens == [90] * 4 + [-1] and eng.last["generated"] == 4


def test_chat_turns_follow_the_reference_layout():
    tok = FakeTok()
    eng = bare(tok, capacity=512)
    sent = []
    real = eng._run
    eng._run = lambda ids, sampling: (sent.append(list(ids)), real(ids, sampling))[1]
    list(eng.chat("hi", max_new_tokens=3))
    first = tok.encode(f"<|im_start|>system\n{nat.DEFAULT_SYSTEM}<|im_end|>\n<|im_start|>user\nhi<|im_end|>\n"
                       "<|im_start|>assistant\n").ids
    assert sent[0] == first
    closed = eng._history[-1] == 95
    list(eng.chat("again", max_new_tokens=2))
    want = ("" if closed else "<|im_end|>") + "\n<|im_start|>user\nagain<|im_end|>\n<|im_start|>assistant\n"
    assert sent[1] == tok.encode(want).ids


def test_tokenize_special_flag():
    eng = bare(FakeTok())
    assert 95 in eng.tokenize("a|b") and 95 not in eng.tokenize("a|b", special=False)
    assert eng._tok.encode_special_tokens is False
