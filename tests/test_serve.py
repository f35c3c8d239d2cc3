"""The `--serve` JSON-lines loop (`seedplane_b200.serve`, the reference's `qwen_vk.cpp:810-855`)
on the CPU with a fake engine: the ready line, each op's answer, one token line per emitted token
then the done line, error lines that keep the loop alive; the token and text lines parsed the way
the reference's subprocess client reads them (`seedplane/native.py:51-61`). And the executable's
start-up failure path (no GPU needed)."""
import io
import json
import subprocess
import sys
from pathlib import Path

from seedplane_b200.serve import serve

ROOT = Path(__file__).resolve().parents[1]


class FakeEngine:
    def __init__(self):
        self.info = {"ready": True, "device": "fake", "mode": "full", "plan": {"shard": 0, "halo": 0, "sinks": 0},
                     "positions": 64, "window_slots": 64, "engine": "fake"}
        self.on_token = None
        self.last = None
        self.hist = []
        self.calls = []

    def _run(self, ids, sampling):
        self.calls.append(dict(sampling))
        out = [(i * 7 + len(self.hist)) % 50 for i in range(int(sampling.get("max_new_tokens", 3)))]
        for t in out:
            piece = f"<{t}>" if t % 2 == 0 else ""
            if self.on_token:
                self.on_token(t, piece)
            if piece:
                yield piece
        self.hist += list(ids) + out
        self.last = {"done": True, "reason": "length", "generated": len(out), "prompt_tokens": len(ids),
                     "prefill_s": 0.0, "decode_s": 0.0, "decode_tok_s": 0.0, "position": len(self.hist)}

    def generate(self, text=None, ids=None, reset=True, **sampling):
        if reset:
            self.reset()
        if ids is None:
            raise RuntimeError("no tokenizer")
        yield from self._run(ids, sampling)

    def chat(self, content, system=None, reset=False, **sampling):
        raise RuntimeError("no tokenizer")
        yield

    def tokenize(self, text, special=True):
        return [ord(c) for c in text]

    def detokenize(self, ids, skip_special=False):
        return "".join(chr(i) for i in ids)

    def state(self):
        return {"position": len(self.hist), "processed": len(self.hist), "tokens": list(self.hist), "capacity": 64}

    def reset(self):
        self.hist = []


def run(reqs):
    eng = FakeEngine()
    out = io.StringIO()
    inp = io.StringIO("".join((r if isinstance(r, str) else json.dumps(r)) + "\n" for r in reqs))
    assert serve(eng, inp, out) == 0
    return eng, [json.loads(l) for l in out.getvalue().splitlines()]


def client_stream(lines):
    """The reference client's reading of one generate / chat answer."""
    tokens, text = [], []
    for r in lines:
        if "error" in r:
            raise RuntimeError(r["error"])
        if r.get("done"):
            return tokens, "".join(text), r
        if "token" in r:
            tokens.append(int(r["token"]))
        if r["text"]:
            text.append(r["text"])
    raise AssertionError("no done line")


def test_serve_protocol():
    eng, lines = run([{"op": "generate", "ids": [1, 2, 3], "max_new_tokens": 4, "temperature": 0.5, "top_k": 3},
                      {"op": "state"}, {"op": "tokenize", "text": "ab"}, {"op": "detokenize", "ids": [104, 105]},
                      {"op": "generate", "ids": [9], "reset": 1, "max_new_tokens": 2, "stop": [5]},
                      {"op": "chat", "content": "hi"}, "not json", {"op": "nope"}, {"op": "reset"}, {"op": "state"}])
    assert lines[0] == {"ready": True, "device": "fake", "mode": "full", "plan": {"shard": 0, "halo": 0, "sinks": 0},
                        "positions": 64, "window_slots": 64}
    toks, text, done = client_stream(lines[1:6])
    assert toks == [0, 7, 14, 21] and text == "<0><14>" and done["generated"] == 4 and done["position"] == 7
    assert eng.calls[0] == {"max_new_tokens": 4, "temperature": 0.5, "top_k": 3}
    assert lines[6] == {"position": 7, "processed": 7, "tokens": [1, 2, 3, 0, 7, 14, 21]}
    assert lines[7] == {"ids": [97, 98]} and lines[8] == {"text": "hi"}
    toks, _, done = client_stream(lines[9:12])
    assert toks == [0, 7] and done["prompt_tokens"] == 1 and eng.calls[1]["stop"] == [5]
    assert "error" in lines[12] and "error" in lines[13] and "error" in lines[14]
    assert lines[15] == {"ok": True} and lines[16]["position"] == 0
    assert len(lines) == 17 and eng.on_token is None


def test_serve_generate_continues_without_reset():
    _, lines = run([{"op": "generate", "ids": [1], "max_new_tokens": 1}, {"op": "generate", "ids": [2], "max_new_tokens": 1},
                    {"op": "state"}])
    assert lines[-1]["position"] == 4              # reset defaults to 0 in the serve protocol


def test_executable_reports_a_bad_bundle():
    exe = ROOT / "seedplane_b200" / "qwen_serve"
    assert exe.stat().st_mode & 0o111
    r = subprocess.run([sys.executable, str(exe), str(ROOT / "no-such-bundle"), "--serve"], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 1 and r.stdout == "" and "seedplane-b200 serve:" in r.stderr
