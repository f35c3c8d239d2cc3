"""`NativeEngine` and the per-GPU HIVE executor on the GPU: greedy tokens identical to the oracle,
the reference engine's run semantics (`qwen_vk.cpp:588-613`: the stop token emitted and counted,
the last sampled token kept unprocessed in the session and processed by the next request), reset;
temperature sampling (the device draw bit-exact with its CPU restatement, runs reproducible from
the seed)."""
import pytest
import torch

from oracle.qwen_oracle import OracleQwen2
from seedplane_b200.config import PRESETS
from seedplane_b200.randinit import TEST_INIT, make_weights, random_prompt

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bundle(tmp_path_factory):
    from safetensors.torch import save_file
    import json
    cfg = PRESETS["tiny-hd128"]
    w = make_weights(cfg, seed=0, dtype=torch.float16, **TEST_INIT)
    d = tmp_path_factory.mktemp("tiny-bundle")
    (d / "config.json").write_text(json.dumps(cfg.to_hf()))
    save_file({k: v.contiguous() for k, v in w.items()}, str(d / "model.safetensors"))
    return d, cfg, w


def test_native_engine_generate_matches_oracle(bundle):
    from seedplane_b200.native import NativeEngine
    d, cfg, w = bundle
    prompt = random_prompt(cfg.vocab, 11, seed=5)
    want = OracleQwen2(cfg, w, kv_fp16=True).greedy(prompt, 40)[0]
    with NativeEngine(d, ctx=256) as eng:
        assert eng.info["ready"] and eng.info["mode"] == "full" and eng.info["positions"] == 256
        pieces = list(eng.generate(ids=prompt, max_new_tokens=40))
        assert pieces == []                       # no tokenizer.json: ids only
        assert eng.last_tokens == want
        last = eng.last
        assert last["done"] and last["reason"] == "length" and last["generated"] == 40
        assert last["prompt_tokens"] == len(prompt) and last["position"] == len(prompt) + 40
        st = eng.state()
        assert st["position"] == len(prompt) + 40 and st["processed"] == len(prompt) + 39
        # a stop token ends the run: emitted and counted, kept in the session unprocessed
        k = want.index(want[5])
        list(eng.generate(ids=prompt, max_new_tokens=40, stop=[want[5]]))
        assert eng.last_tokens == want[:k + 1] and eng.last["reason"] == "stop" and eng.last["generated"] == k + 1
        st = eng.state()
        assert st["tokens"] == prompt + want[:k + 1] and st["processed"] == len(prompt) + k
        # a request without reset continues the session: the pending stop token is processed first
        more = random_prompt(cfg.vocab, 3, seed=9)
        list(eng.generate(ids=more, reset=False, max_new_tokens=6))
        assert eng.last_tokens == OracleQwen2(cfg, w, kv_fp16=True).greedy(prompt + want[:k + 1] + more, 6)[0]
        # reset=True starts over: same tokens again
        list(eng.generate(ids=prompt, max_new_tokens=7))
        assert eng.last_tokens == want[:7]
        with pytest.raises(RuntimeError):
            list(eng.generate(ids=prompt, temperature=0.7, top_p=1.5))
        with pytest.raises(RuntimeError):
            eng.tokenize("hello")


def test_gpu_agent_executor_matches_oracle(bundle):
    from seedplane_b200.engine import CudaQwen2
    from seedplane_b200.hive.agent import GreedyExecutor, token_sha256
    d, cfg, w = bundle
    eng = CudaQwen2(cfg, w, device="cuda:0")
    ex = GreedyExecutor(eng, 128)
    o = OracleQwen2(cfg, w, kv_fp16=True)
    for seed in (1, 2):
        prompt = random_prompt(cfg.vocab, 20 + seed, seed=seed)
        r = ex({"ids": prompt, "max_new_tokens": 9})
        want = o.greedy(prompt, 9)[0]
        assert r["tokens"] == want and r["token_sha256"] == token_sha256(want)
    eng.close()


def test_device_temperature_draw_matches_restatement(bundle):
    """One draw from softmax(logits / T) on the device equals the CPU restatement's on the same logits."""
    from oracle import speculative_oracle as so
    from seedplane_b200.engine import CudaQwen2
    from seedplane_b200.speculative import sample_token
    d, cfg, w = bundle
    eng = CudaQwen2(cfg, w, device="cuda:0")
    kv = eng.new_kv(64)
    logits, _ = eng.forward(kv, random_prompt(cfg.vocab, 9, seed=2))
    host = logits.cpu().numpy()
    for temp in (0.5, 1.0, 3.0):
        for seed, counter in [(0, 0), (1, 0), (7, 3), (12345, 99), (2 ** 40 + 5, 7)]:
            got = sample_token(eng, logits, temp, seed, counter)
            emitted, _ = so.accept_stochastic([], [], host, host, temp, seed, counter)
            assert got == emitted[0], (temp, seed, counter)
    eng.close()


def test_native_engine_temperature_sampling(bundle):
    from seedplane_b200.native import NativeEngine
    d, cfg, w = bundle
    prompt = random_prompt(cfg.vocab, 11, seed=5)
    with NativeEngine(d, ctx=256) as eng:
        list(eng.generate(ids=prompt, max_new_tokens=24, temperature=5.0, seed=11))
        a = list(eng.last_tokens)
        assert len(a) == 24 and all(0 <= t < cfg.vocab for t in a)
        assert eng.last["reason"] == "length" and eng.last["position"] == len(prompt) + 24
        list(eng.generate(ids=prompt, max_new_tokens=24, temperature=5.0, seed=11))
        assert eng.last_tokens == a                      # the seed reproduces the run
        list(eng.generate(ids=prompt, max_new_tokens=24, temperature=5.0, seed=12))
        assert eng.last_tokens != a                      # another seed, another run
        # a stop token ends the run with it
        list(eng.generate(ids=prompt, max_new_tokens=24, temperature=5.0, seed=11, stop=[a[4]]))
        assert eng.last_tokens == a[:a.index(a[4]) + 1] and eng.last["reason"] == "stop"


def test_native_engine_top_k_top_p_sampling(bundle):
    """top-k / top-p sampling on the device: top_k = 1 is greedy, a seed reproduces a filtered run."""
    from seedplane_b200.native import NativeEngine
    d, cfg, w = bundle
    prompt = random_prompt(cfg.vocab, 11, seed=5)
    with NativeEngine(d, ctx=256) as eng:
        list(eng.generate(ids=prompt, max_new_tokens=12))
        greedy = list(eng.last_tokens)
        list(eng.generate(ids=prompt, max_new_tokens=12, temperature=3.0, top_k=1, seed=4))
        assert eng.last_tokens == greedy
        list(eng.generate(ids=prompt, max_new_tokens=12, temperature=3.0, top_p=0.0, seed=4))
        assert eng.last_tokens == greedy
        list(eng.generate(ids=prompt, max_new_tokens=16, temperature=2.0, top_k=20, top_p=0.9, seed=8))
        a = list(eng.last_tokens)
        assert len(a) == 16 and eng.last["reason"] == "length"
        list(eng.generate(ids=prompt, max_new_tokens=16, temperature=2.0, top_k=20, top_p=0.9, seed=8))
        assert eng.last_tokens == a


def test_serve_executable_matches_in_process_engine(bundle):
    """`seedplane_b200/qwen_serve` as the reference's client runs it (`[engine, bundle, '--serve',
    ...]`, JSON lines): the ready line, greedy tokens equal to the in-process engine's, state."""
    import json
    import subprocess
    import sys
    from pathlib import Path
    from seedplane_b200.native import NativeEngine
    d, cfg, w = bundle
    prompt = random_prompt(cfg.vocab, 10, seed=3)
    with NativeEngine(d, ctx=128) as eng:
        list(eng.generate(ids=prompt, max_new_tokens=9))
        want = list(eng.last_tokens)
    exe = Path(__file__).resolve().parents[1] / "seedplane_b200" / "qwen_serve"
    p = subprocess.Popen([sys.executable, str(exe), str(d), "--serve", "--ctx", "128"], stdin=subprocess.PIPE,
                         stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
    try:
        ready = json.loads(p.stdout.readline())
        assert ready["ready"] and ready["positions"] == 128
        p.stdin.write(json.dumps({"op": "generate", "ids": prompt, "max_new_tokens": 9}) + "\n")
        p.stdin.flush()
        toks = []
        while True:
            r = json.loads(p.stdout.readline())
            assert "error" not in r, r
            if r.get("done"):
                break
            toks.append(r["token"])
        assert toks == want and r["generated"] == 9 and r["position"] == len(prompt) + 9
        p.stdin.write(json.dumps({"op": "state"}) + "\n")
        p.stdin.flush()
        st = json.loads(p.stdout.readline())
        assert st["position"] == len(prompt) + 9 and st["processed"] == len(prompt) + 8
        assert st["tokens"] == prompt + want
    finally:
        p.stdin.close()
        p.wait(timeout=60)
