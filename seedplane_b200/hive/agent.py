"""One persistent HIVE pull agent per GPU (`seedplane/hive/agent.py:12-48` of the reference).

The reference runs one agent per host around a `NativeEngine` subprocess; here every GPU of the
box gets its own agent (worker id `gpu<k>`), each bound to the engine on its device, and requests
partition across the GPUs with no collective. A request's result carries the generated token ids
and their sha256 over the compact JSON list, so identical requests on different GPUs can be
checked for identical output.

    python -m seedplane_b200.hive.agent --bundle DIR --model-id qwen2-1.5b --connect 127.0.0.1:PORT --device 0
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
from typing import List

from .pool import HiveAgent

ALLOWED = {"max_new_tokens", "temperature", "top_k", "top_p", "seed", "stop"}


def token_sha256(tokens: List[int]) -> str:
    return hashlib.sha256(json.dumps(list(tokens), separators=(",", ":")).encode("utf-8")).hexdigest()


def native_generate(engine, payload: dict) -> dict:
    """A `generate` request on a `NativeEngine` (text or token ids), the reference agent's result."""
    options = {k: v for k, v in payload.items() if k in ALLOWED}
    if "ids" in payload:
        pieces = list(engine.generate(ids=payload["ids"], reset=True, **options))
    else:
        pieces = list(engine.generate(text=payload.get("text", ""), reset=True, **options))
    return {"text": "".join(pieces), "tokens": engine.last_tokens, "token_sha256": token_sha256(engine.last_tokens),
            "stats": engine.last, "device": engine.info.get("device")}


class GreedyExecutor:
    """`execute` of a GPU agent over an engine in this process: greedy generation of token ids.

    Payload: {"ids": [...], "max_new_tokens": n}. Prefill, then the device decode loop (argmax fed
    back on the GPU); one host sync per request, to read the first token. A grouped lease,
    {"batch": [payload, ...]}, runs its requests together (`batch.generate_batch`: one batched pass
    per decode step for all of them) and answers {"batch": [result, ...]}. Optional `timer`
    (callable(start: bool)) brackets the device work of each lease."""

    def __init__(self, engine, capacity: int, timer=None):
        self.engine = engine
        self.capacity = capacity
        self.kv = engine.new_kv(capacity)
        self.batch_kvs = []
        self.timer = timer

    def _batch(self, items) -> dict:
        from ..batch import MAX_BATCH, generate_batch
        prompts, limits = [], []
        for it in items:
            ids = [int(t) for t in it["ids"]]
            n = int(it.get("max_new_tokens", 32))
            if not ids or n < 1:
                raise ValueError("a request needs prompt ids and max_new_tokens >= 1")
            if len(ids) + n > self.capacity:
                raise ValueError("request exceeds the agent's KV capacity")
            prompts.append(ids)
            limits.append(n)
        while len(self.batch_kvs) < min(len(items), MAX_BATCH):
            self.batch_kvs.append(self.engine.new_kv(self.capacity))
        out = []
        for c0 in range(0, len(items), MAX_BATCH):
            out += generate_batch(self.engine, prompts[c0:c0 + MAX_BATCH], limits[c0:c0 + MAX_BATCH],
                                  kvs=self.batch_kvs, timer=self.timer)
        dev = str(self.engine.device)
        return {"batch": [{"tokens": t, "token_sha256": token_sha256(t), "device": dev} for t in out]}

    def __call__(self, payload: dict) -> dict:
        import torch
        if "batch" in payload:
            return self._batch(payload["batch"])
        ids = [int(t) for t in payload["ids"]]
        n = int(payload.get("max_new_tokens", 32))
        if not ids or n < 1:
            raise ValueError("a request needs prompt ids and max_new_tokens >= 1")
        if len(ids) + n > self.kv.capacity:
            raise ValueError("request exceeds the agent's KV capacity")
        dev = self.engine.device
        torch.cuda.set_device(dev)
        self.kv.length = 0
        if self.timer:
            self.timer(True)
        _, am = self.engine.forward(self.kv, torch.tensor(ids, dtype=torch.int32), want_logits=False, last_only=True)
        first = int(am[-1])
        tokens = [first]
        if n > 1:
            out, _ = self.engine.decode(self.kv, first, len(ids), n - 1)
            tokens += out.tolist()
        if self.timer:
            self.timer(False)
        return {"tokens": tokens, "token_sha256": token_sha256(tokens), "device": str(dev)}


def main(argv=None):
    ap = argparse.ArgumentParser(description="Persistent pull-based SeedPlane HIVE agent for one GPU")
    ap.add_argument("--bundle", required=True, help="seedplane-bundle/2 or HF checkpoint directory")
    ap.add_argument("--engine", help="engine library (default: the in-tree build)")
    ap.add_argument("--model-id", required=True, help="model identity advertised to the broker")
    ap.add_argument("--device", type=int, default=0, help="CUDA device of this agent")
    ap.add_argument("--worker-id", default=None, help="default: gpu<device>")
    ap.add_argument("--cap", action="append", default=[], help="additional execution capability (repeatable)")
    ap.add_argument("--connect", required=True, metavar="HOST:PORT", help="HIVE broker address")
    ap.add_argument("--authkey", default=os.environ.get("SEEDPLANE_AUTHKEY"),
                    help="shared secret; use only on a trusted network")
    a = ap.parse_args(argv)
    host, port = a.connect.rsplit(":", 1)
    from ..native import NativeEngine
    with NativeEngine(a.bundle, engine=a.engine, max_new_tokens=512, extra_args=("--device", f"cuda:{a.device}")) as eng:
        agent = HiveAgent(host, int(port), a.worker_id or f"gpu{a.device}",
                          caps=("generate", "throughput.generate", *a.cap), models=(a.model_id,),
                          execute=lambda payload: native_generate(eng, payload), authkey=a.authkey)
        agent.run()


if __name__ == "__main__":
    main()
