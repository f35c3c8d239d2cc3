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
  the host sees each block's tokens, cuts at a stop token and rolls the cache back to it. The
  token sequence is the same as one-at-a-time decoding.
* Only full attention (`mode` None / "full") is built; shard windows raise `RuntimeError`.
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

QWEN_STOP_TOKENS = ("<|endoftext|>", "<|im_end|>")
_DECODE_BLOCK = 32


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
        args = list(extra_args)
        while args:
            flag = args.pop(0)
            if flag == "--device" and args:
                device = args.pop(0)
            elif flag == "--shaders" and args:
                args.pop(0)                      # the Vulkan build's shader directory: nothing to load here
            else:
                raise RuntimeError(f"engine failed to start: unknown argument {flag!r}")
        if mode not in (None, "full") and not full:
            raise RuntimeError(f"engine failed to start: attention mode {mode!r} is not built (full attention only)")
        from .bundle import load_checkpoint, plan_of
        from .engine import CudaQwen2
        self.bundle = Path(bundle)
        try:
            cfg, weights, fmt = load_checkpoint(self.bundle)
        except (OSError, ValueError, KeyError) as exc:
            raise RuntimeError(f"engine failed to start: {exc}") from exc
        self.cfg = cfg
        self._engine = CudaQwen2(cfg, weights, device=device, weight_format=fmt)
        del weights
        self.capacity = int(min(ctx or 4096, cfg.max_positions))
        self._kv = self._engine.new_kv(self.capacity)
        self._tok = self._load_tokenizer(self.bundle)
        self._stop_ids = set()
        if self._tok is not None:
            for s in QWEN_STOP_TOKENS:
                i = self._tok.token_to_id(s)
                if i is not None:
                    self._stop_ids.add(int(i))
        self.defaults = {"temperature": temperature, "top_k": top_k, "top_p": top_p, "seed": seed,
                         "max_new_tokens": max_new_tokens if max_new_tokens is not None else 256}
        self.system = system
        self._history: List[int] = []           # token ids whose K/V the cache holds
        dev = self._engine.device
        self.info = {"ready": True, "device": torch.cuda.get_device_name(dev), "engine": "seedplane-b200",
                     "mode": "full", "plan": plan_of(self.bundle), "positions": self.capacity,
                     "window_slots": self.capacity, "weights": fmt}
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
        """Token ids of `text`; special tokens written in the text are recognised (the tokenizer's
        added tokens), as the reference engine's `special=True` default does."""
        self._need_tokenizer()
        return self._tok.encode(text, add_special_tokens=False).ids

    def detokenize(self, ids, skip_special=False):
        self._need_tokenizer()
        return self._tok.decode(list(ids), skip_special_tokens=skip_special)

    def state(self):
        """The serve loop's `state` answer (`qwen_vk.cpp:828-831`): position, processed (every
        position of the cache is processed here) and the token ids the cache holds."""
        return {"position": self._kv.length, "processed": self._kv.length, "tokens": list(self._history),
                "capacity": self.capacity, "mode": "full"}

    def reset(self):
        self._kv.length = 0
        self._history = []

    def generate(self, text=None, ids=None, reset=True, **sampling):
        """Raw continuation of `text` or of token `ids`; yields text pieces."""
        if reset:
            self.reset()
        prompt = list(ids) if ids is not None else self.tokenize(text or "")
        yield from self._run(prompt, sampling)

    def chat(self, content, system=None, reset=False, **sampling):
        """One user turn in ChatML; the conversation stays in the cache."""
        self._need_tokenizer()
        if reset:
            self.reset()
        text = ""
        sys_prompt = system if system is not None else self.system
        if not self._history and sys_prompt:
            text += f"<|im_start|>system\n{sys_prompt}<|im_end|>\n"
        elif self._history:
            text += "\n"                        # closes the previous assistant turn's <|im_end|>
        text += f"<|im_start|>user\n{content}<|im_end|>\n<|im_start|>assistant\n"
        yield from self._run(self.tokenize(text), sampling)
        # close the assistant turn in the cache: its last token (when cut by length) and <|im_end|>
        tail = []
        if self.last and self.last["reason"] == "length" and self.last_tokens:
            tail.append(self.last_tokens[-1])
        end = self._tok.token_to_id("<|im_end|>")
        if end is not None:
            tail.append(int(end))
        if tail and self._kv.length + len(tail) < self.capacity:
            self._feed(tail)

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
            if isinstance(s, int):
                stops.add(int(s))
            elif self._tok is not None:
                i = self._tok.token_to_id(str(s))
                if i is not None:
                    stops.add(int(i))
        return int(opt["max_new_tokens"]), stops, temp, int(opt.get("seed") or 0), top_k, top_p

    def _feed(self, ids: List[int]):
        """Prefill ids into the cache; returns the argmax after the last one."""
        _, am = self._engine.forward(self._kv, torch.tensor(ids, dtype=torch.int32), want_logits=False)
        self._history.extend(ids)
        return int(am[-1])

    def _run(self, prompt: List[int], sampling) -> Iterable[str]:
        max_new, stops, temp, seed, top_k, top_p = self._options(sampling)
        self.last_tokens = []
        self.last = None
        if not prompt:
            raise RuntimeError("empty prompt")
        if any(t < 0 or t >= self.cfg.vocab for t in prompt):
            raise RuntimeError("token id outside the vocabulary")
        if self._kv.length + len(prompt) >= self.capacity:
            self.last = {"done": True, "reason": "context", "generated": 0, "prompt_tokens": len(prompt),
                         "prefill_s": 0.0, "decode_s": 0.0, "decode_tok_s": 0.0, "position": self._kv.length}
            return
        dev = self._engine.device
        if temp > 0.0:
            yield from self._run_sampled(prompt, max_new, stops, temp, seed, top_k, top_p)
            return
        t0 = time.perf_counter()
        queue = [self._feed(prompt)]            # generated tokens not yet checked (none is in the cache)
        torch.cuda.synchronize(dev)
        prefill_s = time.perf_counter() - t0
        t1 = time.perf_counter()
        produced: List[int] = []
        shown = ""
        reason = "length"
        fed_at = None                           # cache slot of the token fed to the last decode block
        while True:
            done = False
            for i, t in enumerate(queue):
                if t in stops:
                    reason, done = "stop", True
                else:
                    produced.append(t)
                    self.last_tokens.append(t)
                    piece = ""
                    if self._tok is not None:
                        full = self._tok.decode(produced)
                        if not full.endswith("\ufffd") and len(full) > len(shown):
                            piece, shown = full[len(shown):], full
                    if self.on_token is not None:
                        self.on_token(t, piece)
                    if piece:
                        yield piece
                    if len(produced) >= max_new:
                        reason, done = "length", True
                if done:
                    if fed_at is not None:      # the cache holds the fed token and queue[:-1]: keep queue[:i]
                        self._kv.length = fed_at + 1 + i
                        del self._history[self._kv.length:]
                    break
            if done:
                break
            room = self.capacity - self._kv.length
            if room < 1:
                reason = "context"
                break
            token = queue[-1]
            n = min(_DECODE_BLOCK, max_new - len(produced), room)
            fed_at = self._kv.length
            out, _ = self._engine.decode(self._kv, token, fed_at, n)
            queue = out.tolist()
            self._history.append(token)
            self._history.extend(queue[:-1])
        decode_s = time.perf_counter() - t1
        gen = len(produced)
        self.last = {"done": True, "reason": reason, "generated": gen, "prompt_tokens": len(prompt),
                     "prefill_s": prefill_s, "decode_s": decode_s,
                     "decode_tok_s": (gen - 1) / decode_s if gen > 1 and decode_s > 0 else 0.0,
                     "position": self._kv.length}

    def _run_sampled(self, prompt: List[int], max_new: int, stops, temp: float, seed: int, top_k: int = 0,
                     top_p: float = 1.0) -> Iterable[str]:
        """Temperature sampling (top-k / top-p filtered when set, as the reference's sample()): one
        decode step with logits per token, the filter and the draw on the device."""
        from .speculative import sample_token
        dev = self._engine.device
        t0 = time.perf_counter()
        logits, _ = self._engine.forward(self._kv, torch.tensor(prompt, dtype=torch.int32))
        self._history.extend(prompt)
        counter = 0
        tok = sample_token(self._engine, logits, temp, seed, counter, top_k, top_p)
        prefill_s = time.perf_counter() - t0
        t1 = time.perf_counter()
        produced: List[int] = []
        shown = ""
        reason = "length"
        while True:
            if tok in stops:
                reason = "stop"
                break
            produced.append(tok)
            self.last_tokens.append(tok)
            piece = ""
            if self._tok is not None:
                full = self._tok.decode(produced)
                if not full.endswith("\ufffd") and len(full) > len(shown):
                    piece, shown = full[len(shown):], full
            if self.on_token is not None:
                self.on_token(tok, piece)
            if piece:
                yield piece
            if len(produced) >= max_new:
                break
            if self.capacity - self._kv.length < 1:
                reason = "context"
                break
            _, lg = self._engine.decode(self._kv, tok, self._kv.length, 1, want_logits=True)
            self._history.append(tok)
            counter += 1
            tok = sample_token(self._engine, lg, temp, seed, counter, top_k, top_p)
        torch.cuda.synchronize(dev)
        decode_s = time.perf_counter() - t1
        gen = len(produced)
        self.last = {"done": True, "reason": reason, "generated": gen, "prompt_tokens": len(prompt),
                     "prefill_s": prefill_s, "decode_s": decode_s,
                     "decode_tok_s": (gen - 1) / decode_s if gen > 1 and decode_s > 0 else 0.0,
                     "position": self._kv.length}

    # ---- lifetime ----------------------------------------------------------------------------
    def close(self):
        if getattr(self, "_kv", None) is not None:
            self._kv.close()
            self._kv = None
        if getattr(self, "_engine", None) is not None:
            self._engine.close()
            self._engine = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
