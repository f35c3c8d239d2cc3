"""The reference engine's `--serve` loop (`native/vulkan_decode/qwen_vk.cpp:810-855`) over this
repository's engine, so the reference's own subprocess client (`seedplane/native.py:25-90`,
`NativeEngine`) drives it unchanged: point `SEEDPLANE_NATIVE_ENGINE` (or its `engine=` argument)
at the executable `seedplane_b200/qwen_serve`.

Protocol: one JSON object per line in, JSON lines out. First line out: the ready line
(`{"ready": true, "device", "mode", "plan", "positions", "window_slots"}`). Requests: `reset`
-> `{"ok": true}`; `tokenize` {text, special} -> `{"ids"}`; `detokenize` {ids, skip_special} ->
`{"text"}`; `state` -> `{"position", "processed", "tokens"}`; `generate` {ids | text, reset,
temperature, top_k, top_p, seed, stop, max_new_tokens} and `chat` {content, system, reset, ...}
-> one `{"token", "text"}` line per emitted token, then `{"done": true, "reason", "generated",
"prompt_tokens", "prefill_s", "decode_s", "decode_tok_s", "position"}`. A failed request answers
`{"error": message}` and the loop goes on; end of input ends it.
"""
from __future__ import annotations

import argparse
import json
import sys
from typing import IO, List, Optional

_SAMPLING = ("temperature", "top_k", "top_p", "seed", "stop", "max_new_tokens")


def _line(out: IO[str], obj) -> None:
    out.write(json.dumps(obj, ensure_ascii=False) + "\n")
    out.flush()


def serve(eng, inp: IO[str], out: IO[str]) -> int:
    """Answer the requests of `inp` on `out` with `eng` (the `NativeEngine` interface: info,
    generate, chat, tokenize, detokenize, state, reset, last, on_token)."""
    info = eng.info
    _line(out, {"ready": True, "device": info.get("device"), "mode": info.get("mode"), "plan": info.get("plan"),
                "positions": info.get("positions"), "window_slots": info.get("window_slots")})
    for raw in inp:
        raw = raw.rstrip("\r\n")
        if not raw:
            continue
        try:
            q = json.loads(raw)
            if not isinstance(q, dict):
                raise ValueError("a request is a JSON object")
            op = q.get("op", "")
            if op == "reset":
                eng.reset()
                _line(out, {"ok": True})
            elif op == "tokenize":
                _line(out, {"ids": list(eng.tokenize(q.get("text", ""), bool(q.get("special", 1))))})
            elif op == "detokenize":
                _line(out, {"text": eng.detokenize(q.get("ids") or [], bool(q.get("skip_special", 0)))})
            elif op == "state":
                st = eng.state()
                _line(out, {"position": st["position"], "processed": st["processed"], "tokens": st["tokens"]})
            elif op in ("generate", "chat"):
                sampling = {k: q[k] for k in _SAMPLING if q.get(k) is not None}
                reset = bool(q.get("reset", 0))
                eng.on_token = lambda t, piece: _line(out, {"token": int(t), "text": piece})
                try:
                    if op == "chat":
                        it = eng.chat(q.get("content", ""), system=q.get("system"), reset=reset, **sampling)
                    elif q.get("ids") is not None:
                        it = eng.generate(ids=[int(t) for t in q["ids"]], reset=reset, **sampling)
                    else:
                        it = eng.generate(text=q.get("text", ""), reset=reset, **sampling)
                    for _ in it:
                        pass
                finally:
                    eng.on_token = None
                _line(out, dict(eng.last))
            else:
                raise ValueError(f"unknown op {op}")
        except Exception as exc:   # the reference answers every failure with an error line
            _line(out, {"error": str(exc)})
    return 0


def main(argv: Optional[List[str]] = None) -> int:
    ap = argparse.ArgumentParser(description="JSON-lines serve loop of the reference engine over seedplane-b200")
    ap.add_argument("bundle")
    ap.add_argument("--serve", action="store_true", required=True)
    ap.add_argument("--mode")
    ap.add_argument("--full", action="store_true")
    ap.add_argument("--ctx", type=int)
    ap.add_argument("--temperature", type=float)
    ap.add_argument("--top-k", type=int)
    ap.add_argument("--top-p", type=float)
    ap.add_argument("--seed", type=int)
    ap.add_argument("-n", "--max-new-tokens", type=int)
    ap.add_argument("--system")
    a = ap.parse_args(argv)
    from . import _native as N
    from .native import NativeEngine
    try:
        eng = NativeEngine(a.bundle, engine=str(N.LIB_PATH), mode=a.mode, full=a.full, ctx=a.ctx,
                           temperature=a.temperature, top_k=a.top_k, top_p=a.top_p, seed=a.seed,
                           max_new_tokens=a.max_new_tokens, system=a.system)
    except Exception as exc:
        print(f"seedplane-b200 serve: {exc}", file=sys.stderr)
        return 1
    try:
        return serve(eng, sys.stdin, sys.stdout)
    finally:
        eng.close()


if __name__ == "__main__":
    sys.exit(main())
