"""Drop-in for `seedplane.native.NativeEngine` (`seedplane/native.py:25-90`) on the B200 engine.

The reference drives `qwen_vk <bundle> --serve`, a subprocess speaking JSON lines. Here the same
surface drives the CUDA engine in this process, so `NativeEngine` keeps the reference's
constructor, `info`, `generate` / `chat` generators of text pieces, `last`, `last_tokens`,
`tokenize`, `detokenize`, `state`, `reset`, `close` and the context manager, with the same error
types: a failed request raises `RuntimeError(message)`, a missing engine `FileNotFoundError`.

* `bundle`: a seedplane-bundle/2 directory or an HF checkpoint directory (`bundle.load_checkpoint`).
  Text operations need a `tokenizer.json` beside the weights; without one, `generate(ids=...)`
  still works and yields no text (the token ids are in `last_tokens`).
* `engine`: the engine library (`libseedplane_cuda.so`) in place of the reference's executable:
  the explicit path, `$SEEDPLANE_NATIVE_ENGINE`, or the in-tree build.
* Greedy decoding runs on the device in blocks (the argmax is fed back without a host round trip);
  the host sees each block's tokens, cuts at a stop token or the length limit and rolls the cache
  back to it. The token sequence is the same as one-at-a-time decoding.
* Run semantics are the reference engine's (`qwen_vk.cpp:588-613`): every sampled token, a stop
  token included, is emitted (a stop token with empty text) and counted in `generated`; the last
  sampled token stays in the session unprocessed (so `state()` reports position = processed + 1
  and a chat turn's `<|im_end|>` becomes history); text still held by the incremental decoder at
  the end is flushed as one more emission with token -1, and the reference's client appends that
  -1 to `last_tokens`, as this class does.
* Attention follows the reference's modes (`qwen_vk.cpp:235,257,285-301`): `full=True` or
  `mode="full"` is one window over all positions (default `ctx` 8192); otherwise the bundle's shard
  plan (`seedplane.json`, overridable by `--shard/--halo/--sinks` in `extra_args`) with `mode` one
  of rebuild, rebuild-batch, shadow, shadow-batch (the default) or reuse, and `ctx` positions
  (default: the checkpoint's maximum) over windows of S + H + sinks slots (`windows.py`).
* Sampling: temperature > 0 draws each token on the device from softmax(logits / temperature) with
  a counter-based RNG (`seed`, then one counter step per token), so a seed reproduces a run; the
  distribution is the reference's, the random stream is not its mt19937_64 (`sampler.hpp`).
  `top_k` (> 0) / `top_p` (< 1) filter the row on the device first (`sp_sample_filter`, the
  reference's rule of `sampler.hpp:2-3` and `qwen_engine.py:147-156`), then the same draw runs on
  the filtered row.

`last` (`qwen_vk.cpp:848-850`): {done, reason in {stop, length, context}, generated, prompt_tokens,
prefill_s, decode_s, decode_tok_s, position}.
"""
from __future__ import annotations

import os
import time
from pathlib import Path
from typing import Iterable, List, Optional

import torch

from . import _native as N
from .windows import DEFAULT_MODE, MODES, ShardPlan, WindowSession

QWEN_STOP_TOKENS = ("<|im_end|>", "<|endoftext|>")
DEFAULT_SYSTEM = "You are a helpful assistant."      # qwen_vk.cpp:664
_DECODE_BLOCK = 32


class _TextStream:
    """Incremental detokenizer: `push(id)` returns the text that became complete (nothing while a
    multi-byte character is still open), `flush()` whatever is left. Special tokens add no text."""

    def __init__(self, tok):
        self.tok = tok
        self.ids: List[int] = []
        self.shown = ""

    def push(self, t: int) -> str:
        if self.tok is None:
            return ""
        self.ids.append(int(t))
        full = self.tok.decode(self.ids, skip_special_tokens=True)
        if full.endswith("\ufffd") or len(full) <= len(self.shown):
            return ""
        piece, self.shown = full[len(self.shown):], full
        return piece

    def flush(self) -> str:
        if self.tok is None or not self.ids:
            return ""
        full = self.tok.decode(self.ids, skip_special_tokens=True)
        rest = full[len(self.shown):] if full.startswith(self.shown) else ""
        self.shown = full
        return rest


def _sync(dev) -> None:
    if getattr(dev, "type", None) == "cuda":
        torch.cuda.synchronize(dev)


def find_engine(explicit=None) -> str:
    """Engine library: explicit path, $SEEDPLANE_NATIVE_ENGINE, then the in-tree build. The variable
    may name the serve executable instead (for the reference's subprocess client); a candidate
    that is not a shared library is passed over."""
    for cand in (explicit, os.environ.get("SEEDPLANE_NATIVE_ENGINE"), N.LIB_PATH):
        if cand and Path(cand).is_file() and ".so" in Path(cand).name:
            return str(cand)
    raise FileNotFoundError("native engine not found: build it with `python -m seedplane_b200.build` "
                            "or set SEEDPLANE_NATIVE_ENGINE")


class NativeEngine:
    def __init__(self, bundle, engine=None, mode=None, full=False, ctx=None, temperature=None, top_k=None,
                 top_p=None, seed=None, max_new_tokens=None, system=None, extra_args=()):
        lib_path = find_engine(engine)
        if Path(lib_path).resolve() != N.LIB_PATH.resolve() and N._lib is None:
            N.load(Path(lib_path))
        device = "cuda"
        overrides = {}
        args = list(extra_args)
        while args:
            flag = args.pop(0)
            if flag == "--device" and args:
                device = args.pop(0)
            elif flag == "--shaders" and args:
                args.pop(0)                      # the Vulkan build's shader directory: nothing to load here
            elif flag in ("--shard", "--halo", "--sinks") and args:
                try:
                    overrides[flag[2:]] = int(args.pop(0))
                except ValueError as exc:
                    raise RuntimeError(f"engine failed to start: {flag} needs an integer") from exc
            else:
                raise RuntimeError(f"engine failed to start: unknown argument {flag!r}")
        from .bundle import bundle_plan, load_checkpoint, plan_of
        # a SeedPlane bundle decodes under its plan (shadow-batch unless told otherwise, as the
        # reference engine); a plain checkpoint without a plan defaults to full attention
        mode = "full" if full else (mode or (DEFAULT_MODE if bundle_plan(bundle) is not None else "full"))
        if mode not in MODES:
            raise RuntimeError(f"engine failed to start: bad --mode {mode!r}")
        from .engine import CudaQwen2
        self.bundle = Path(bundle)
        try:
            cfg, weights, fmt = load_checkpoint(self.bundle)
            plan = ShardPlan(**{**plan_of(self.bundle), **overrides})
        except (OSError, ValueError, KeyError, TypeError) as exc:
            raise RuntimeError(f"engine failed to start: {exc}") from exc
        self.cfg = cfg
        # positions: qwen_vk.cpp:785 (full attention defaults to 8192, windows to the model's maximum)
        self.capacity = int(min(ctx or (8192 if mode == "full" else cfg.max_positions), cfg.max_positions))
        self._engine = CudaQwen2(cfg, weights, device=device, weight_format=fmt)
        del weights
        try:
            self._session = WindowSession(self._engine, mode, plan, self.capacity)
        except ValueError as exc:
            self._engine.close()
            raise RuntimeError(f"engine failed to start: {exc}") from exc
        self._tok = self._load_tokenizer(self.bundle)
        self._stop_ids = set()
        if self._tok is not None:
            for s in QWEN_STOP_TOKENS:
                i = self._tok.token_to_id(s)
                if i is not None:
                    self._stop_ids.add(int(i))
        self.defaults = {"temperature": temperature, "top_k": top_k, "top_p": top_p, "seed": seed,
                         "max_new_tokens": max_new_tokens if max_new_tokens is not None else 256}
        self.system = DEFAULT_SYSTEM if system is None else system
        dev = self._engine.device
        ses = self._session
        self.info = {"ready": True, "device": torch.cuda.get_device_name(dev), "engine": "seedplane-b200",
                     "mode": ses.mode, "plan": ses.plan, "positions": ses.P, "window_slots": ses.W, "weights": fmt}
        self.last = None
        self.last_tokens: List[int] = []
        self.on_token = None                    # callable(token, text piece or "") per emitted token

    @staticmethod
    def _load_tokenizer(path: Path):
        f = path / "tokenizer.json"
        if not f.is_file():
            return None
        from tokenizers import Tokenizer
        return Tokenizer.from_file(str(f))

    def _need_tokenizer(self):
        if self._tok is None:
            raise RuntimeError(f"{self.bundle}: the bundle has no tokenizer.json (use generate(ids=...))")

    # ---- requests --------------------------------------------------------------------------
    def tokenize(self, text, special=True):
        """Token ids of `text`. With `special` (the default), special tokens written in the text
        (`<|im_start|>`, ...) become their ids; without it they are encoded as plain text, like
        the reference engine's `encode(text, allow_special)`."""
        self._need_tokenizer()
        self._tok.encode_special_tokens = not special
        try:
            return self._tok.encode(text, add_special_tokens=False).ids
        finally:
            self._tok.encode_special_tokens = False

    def detokenize(self, ids, skip_special=False):
        self._need_tokenizer()
        return self._tok.decode(list(ids), skip_special_tokens=skip_special)

    @property
    def _history(self) -> List[int]:
        """The session's token sequence; the first `_session.done` of them are processed (after a
        run, every token but the last sampled one)."""
        return self._session.seq

    def state(self):
        """The serve loop's `state` answer (`qwen_vk.cpp:828-831`): position = tokens in the
        session, processed = tokens whose K/V the windows hold, and the token ids."""
        return {"position": len(self._history), "processed": self._session.done, "tokens": list(self._history),
                "capacity": self.capacity, "mode": self._session.mode}

    def reset(self):
        self._session.reset()

    def generate(self, text=None, ids=None, reset=True, **sampling):
        """Raw continuation of `text` or of token `ids`; yields text pieces."""
        if reset:
            self.reset()
        prompt = list(ids) if ids is not None else self.tokenize(text or "")
        yield from self._run(prompt, sampling)

    def chat(self, content, system=None, reset=False, **sampling):
        """One user turn in ChatML (`qwen_vk.cpp:615-620`); the conversation stays in the session.
        The first turn opens with the system block; a later one closes the previous assistant turn
        (with `<|im_end|>` unless that was its last token) before the user block."""
        self._need_tokenizer()
        if reset:
            self.reset()
        tail = f"<|im_start|>user\n{content}<|im_end|>\n<|im_start|>assistant\n"
        if not self._history:
            sys_prompt = system if system is not None else self.system
            text = f"<|im_start|>system\n{sys_prompt}<|im_end|>\n" + tail
        else:
            closed = self._history[-1] == self._tok.token_to_id("<|im_end|>")
            text = ("" if closed else "<|im_end|>") + "\n" + tail
        yield from self._run(self.tokenize(text), sampling)

    # ---- the loop ----------------------------------------------------------------------------
    def _options(self, sampling):
        allowed = {"max_new_tokens", "temperature", "top_k", "top_p", "seed", "stop"}
        unknown = set(sampling) - allowed
        if unknown:
            raise RuntimeError(f"unknown request field(s): {sorted(unknown)}")
        opt = {k: v for k, v in self.defaults.items()}
        opt.update({k: v for k, v in sampling.items() if v is not None})
        temp = float(opt.get("temperature") or 0.0)
        if temp < 0.0:
            raise RuntimeError("temperature must be >= 0")
        top_k, top_p = int(opt.get("top_k") or 0), float(1.0 if opt.get("top_p") is None else opt["top_p"])
        if top_k < 0 or not 0.0 <= top_p <= 1.0:
            raise RuntimeError("top_k must be >= 0 and top_p in [0, 1]")
        # a request's stop list replaces the default stop tokens (`qwen_vk.cpp:839-840`)
        stops = set(self._stop_ids) if opt.get("stop") is None else set()
        for s in opt.get("stop") or ():
            if isinstance(s, (int, float)) and not isinstance(s, bool):
                stops.add(int(s))             # JSON numbers (151645 or 151645.0), as qwen_vk.cpp:844 casts them
            elif self._tok is not None:
                i = self._tok.token_to_id(str(s))
                if i is not None:
                    stops.add(int(i))
        return int(opt["max_new_tokens"]), stops, temp, int(opt.get("seed") or 0), top_k, top_p

    def _catch_up(self, ids: List[int], want_logits: bool = False):
        """Append `ids` to the session and process every pending token (the previous run's last
        sampled token, then `ids`); returns (logits of the last or None, its argmax)."""
        self._history.extend(int(t) for t in ids)
        return self._session.catch_up(want_logits)

    def _emit(self, t: int, piece: str):
        self.last_tokens.append(int(t))
        if self.on_token is not None:
            self.on_token(int(t), piece)

    def _finish(self, reason, generated, n_prompt, prefill_s, decode_s, stream: _TextStream):
        rest = stream.flush()
        if rest:
            self._emit(-1, rest)
        self.last = {"done": True, "reason": reason, "generated": generated, "prompt_tokens": n_prompt,
                     "prefill_s": prefill_s, "decode_s": decode_s,
                     "decode_tok_s": generated / max(decode_s, 1e-9), "position": len(self._history)}
        return rest

    def _check_prompt(self, prompt: List[int]) -> bool:
        if not prompt:
            raise RuntimeError("empty prompt")
        if any(t < 0 or t >= self.cfg.vocab for t in prompt):
            raise RuntimeError("token id outside the vocabulary")
        if len(self._history) + len(prompt) > self.capacity:
            self.last = {"done": True, "reason": "context", "generated": 0, "prompt_tokens": len(prompt),
                         "prefill_s": 0.0, "decode_s": 0.0, "decode_tok_s": 0.0, "position": len(self._history)}
            return False
        return True

    def _run(self, prompt: List[int], sampling) -> Iterable[str]:
        max_new, stops, temp, seed, top_k, top_p = self._options(sampling)
        self.last_tokens = []
        self.last = None
        if not self._check_prompt(prompt):
            return
        if temp > 0.0:
            yield from self._run_sampled(prompt, max_new, stops, temp, seed, top_k, top_p)
            return
        dev = self._engine.device
        stream = _TextStream(self._tok)
        t0 = time.perf_counter()
        _, first = self._catch_up(prompt)
        _sync(dev)
        prefill_s = time.perf_counter() - t0
        t1 = time.perf_counter()
        ses = self._session
        queue = [first]                         # sampled tokens not emitted yet (the first is unprocessed)
        in_block = False                        # queue came from a device decode block
        generated, reason = 0, "length"
        while True:
            done, kept = False, len(queue)
            for i, t in enumerate(queue):
                self._history.append(t)
                generated += 1
                is_stop = t in stops
                piece = "" if is_stop else stream.push(t)
                self._emit(t, piece)
                if piece:
                    yield piece
                if is_stop:
                    reason, done = "stop", True
                elif generated >= max_new:
                    reason, done = "length", True
                if done:
                    kept = i + 1
                    break
            if in_block:
                # the block processed the fed token and queue[:-1]; keep them up to queue[kept - 2]
                ses.commit_block(kept)
            if done:
                break
            room = ses.P - ses.done
            if room < 1:
                reason = "context"
                break
            out, _ = ses.decode_block(min(_DECODE_BLOCK, max_new - generated, room))
            queue, in_block = out.tolist(), True
        decode_s = time.perf_counter() - t1
        rest = self._finish(reason, generated, len(prompt), prefill_s, decode_s, stream)
        if rest:
            yield rest

    def _run_sampled(self, prompt: List[int], max_new: int, stops, temp: float, seed: int, top_k: int = 0,
                     top_p: float = 1.0) -> Iterable[str]:
        """Temperature sampling (top-k / top-p filtered when set, as the reference's sample()): one
        decode step with logits per token, the filter and the draw on the device."""
        from .speculative import sample_token
        dev = self._engine.device
        stream = _TextStream(self._tok)
        t0 = time.perf_counter()
        logits, _ = self._catch_up(prompt, want_logits=True)
        counter = 0
        tok = sample_token(self._engine, logits[-1:], temp, seed, counter, top_k, top_p)
        prefill_s = time.perf_counter() - t0
        t1 = time.perf_counter()
        generated, reason = 0, "length"
        while True:
            self._history.append(tok)
            generated += 1
            is_stop = tok in stops
            piece = "" if is_stop else stream.push(tok)
            self._emit(tok, piece)
            if piece:
                yield piece
            if is_stop:
                reason = "stop"
                break
            if generated >= max_new:
                break
            if self._session.P - self._session.done < 1:
                reason = "context"
                break
            _, lg = self._session.decode_block(1, want_logits=True)
            self._session.commit_block(1)
            counter += 1
            tok = sample_token(self._engine, lg, temp, seed, counter, top_k, top_p)
        _sync(dev)
        decode_s = time.perf_counter() - t1
        rest = self._finish(reason, generated, len(prompt), prefill_s, decode_s, stream)
        if rest:
            yield rest

    # ---- lifetime ----------------------------------------------------------------------------
    def close(self):
        if getattr(self, "_session", None) is not None:
            self._session.close()
            self._session = None
        if getattr(self, "_engine", None) is not None:
            self._engine.close()
            self._engine = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
