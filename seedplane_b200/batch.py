"""Runtime request batching: greedy generation of independent requests together on one engine.

The reference decodes one request per native session and its HIVE agents report `batch_size: 1`
(`seedplane/hive/pool.py:465-466`; a batched inference API is listed as not built,
`README.md:68`). Here the requests of a batch share every decode step: `sp_decode_batch` runs ONE
batched pass per step over the batch's tokens, each reading and writing its own KV cache, so the
weights stream from HBM once per step for all of them. Every request's tokens are its own greedy
continuation, the same as decoding it alone.

`generate_batch` packs the requests' prompts into batched passes (`sp_prefill_batch`: every token
writes and reads its own request's cache), then decodes the batch in device blocks (each block's
argmaxes are fed back on the GPU); after a block the host cuts each request at its stop token or
length limit and drops finished requests from the batch.
"""
from __future__ import annotations

from typing import Iterable, List, Optional, Sequence

import torch

MAX_BATCH = 64                          # requests per sp_decode_batch call
MAX_PREFILL_BATCH = 256                 # prompts per sp_prefill_batch call


def generate_batch(engine, prompts: Sequence[Sequence[int]], max_new_tokens, stop: Iterable[int] = (),
                   block: int = 16, kvs: Optional[Sequence] = None, timer=None) -> List[List[int]]:
    """Greedy tokens of every prompt (each up to max_new_tokens, ending at the first stop token,
    which is included). `max_new_tokens` is one limit or one per request. `kvs`: caches to use (one
    per request, each with room for its prompt and tokens; their contents are replaced), else new
    ones for this call. `timer(start: bool)` brackets the device work."""
    n_req = len(prompts)
    if n_req == 0:
        return []
    limits = [int(max_new_tokens)] * n_req if isinstance(max_new_tokens, int) else [int(m) for m in max_new_tokens]
    if len(limits) != n_req or any(m < 1 for m in limits):
        raise ValueError("every request needs max_new_tokens >= 1")
    stops = {int(s) for s in stop}
    prompts = [[int(t) for t in p] for p in prompts]
    if any(not p for p in prompts):
        raise ValueError("empty prompt")
    own = kvs is None
    if own:
        kvs = [engine.new_kv(len(p) + m) for p, m in zip(prompts, limits)]
    elif len(kvs) < n_req or any(kv.capacity < len(p) + m for kv, p, m in zip(kvs, prompts, limits)):
        raise ValueError("a request does not fit its cache")
    try:
        if timer:
            timer(True)
        firsts = []
        for kv in kvs[:n_req]:
            kv.length = 0
        for c0 in range(0, n_req, MAX_PREFILL_BATCH):      # the prompts packed into batched passes
            firsts.append(engine.prefill_batch(kvs[c0:c0 + MAX_PREFILL_BATCH], prompts[c0:c0 + MAX_PREFILL_BATCH]))
        out = [[t] for t in torch.cat(firsts).cpu().tolist()]
        done = [o[0] in stops or m == 1 for o, m in zip(out, limits)]
        while True:
            active = [b for b in range(n_req) if not done[b]]
            if not active:
                break
            for c0 in range(0, len(active), MAX_BATCH):
                group = active[c0:c0 + MAX_BATCH]
                n = max(1, min(block, min(limits[b] - len(out[b]) for b in group)))
                toks = engine.decode_batch([kvs[b] for b in group], [out[b][-1] for b in group],
                                           [len(prompts[b]) + len(out[b]) - 1 for b in group], n)
                rows = toks.cpu().tolist()               # [n][len(group)]
                for j, b in enumerate(group):
                    for i in range(n):
                        t = rows[i][j]
                        out[b].append(t)
                        if t in stops or len(out[b]) >= limits[b]:
                            done[b] = True
                            break
        if timer:
            timer(False)
        return out
    finally:
        if own:
            for kv in kvs:
                kv.close()
