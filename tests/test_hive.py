"""HIVE host logic on the CPU: wire format, pull leases, auth, cost model, batch planning, and the
per-GPU agent layout as world-size-2 `gloo` ranks (each rank one agent, rank 0 also the broker).

The planner and cost-model expectations restate the reference's own tests
(`tests/test_hive_transport.py:91-146`); the executor here is a fake (no GPU)."""
import hashlib
import json
import socket
import threading
import time

import pytest

from seedplane_b200.hive import HiveAgent, HiveBroker, MeasuredCostModel, plan_homogeneous_batch
from seedplane_b200.hive.protocol import HEADER, Frame, Message, recv_frame, send_frame


def _wait(cond, limit=3.0):
    end = time.monotonic() + limit
    while not cond() and time.monotonic() < end:
        time.sleep(0.005)
    return cond()


def test_frame_survives_fragmented_transport():
    a, b = socket.socketpair()
    try:
        frame = Frame(Message.WORK, request_id=42, sequence=9, payload=b'{"x":1}')
        raw = HEADER.pack(b"SPH1", 1, int(frame.kind), 0, 42, 9, len(frame.payload)) + frame.payload

        def dribble():
            for octet in raw:
                a.sendall(bytes([octet]))
            a.close()

        t = threading.Thread(target=dribble)
        t.start()
        assert recv_frame(b) == frame
        t.join()
    finally:
        b.close()


def test_bad_magic_and_version_are_rejected():
    for raw in (HEADER.pack(b"XXXX", 1, 5, 0, 0, 0, 0), HEADER.pack(b"SPH1", 2, 5, 0, 0, 0, 0)):
        a, b = socket.socketpair()
        a.sendall(raw)
        with pytest.raises(ValueError):
            recv_frame(b)
        a.close()
        b.close()


def _start_agents(broker, specs):
    agents = [HiveAgent(*broker.address, name, caps=caps, models=models, execute=fn) for name, caps, models, fn in specs]
    threads = [threading.Thread(target=ag.run, daemon=True) for ag in agents]
    for t in threads:
        t.start()
    assert _wait(lambda: len(broker.workers()) == len(agents))
    return agents, threads


def _stop(agents, threads):
    for ag in agents:
        ag.stop()
    for t in threads:
        t.join(timeout=3)
        assert not t.is_alive()


def test_agents_pull_only_compatible_work():
    with HiveBroker(pull_poll_s=0.03) as broker:
        agents, threads = _start_agents(broker, [
            ("draft-box", ("draft",), ("qwen-small",), lambda p: {"worker": "draft-box", "value": p["value"]}),
            ("gpu0", ("generate",), ("qwen-target",), lambda p: {"worker": "gpu0", "value": p["value"]})])
        first = broker.submit({"value": 7}, model="qwen-target", required_caps=("generate",))
        second = broker.submit({"value": 11}, model="qwen-small", required_caps=("draft",))
        assert first.result(timeout=3) == {"worker": "gpu0", "value": 7}
        assert second.result(timeout=3) == {"worker": "draft-box", "value": 11}
        assert broker.cost_model.estimate(kind="throughput.generate", model="qwen-target", worker="gpu0",
                                          token_budget=0) is None      # one sample: not trusted yet
        assert len(broker.cost_model.snapshot()) == 2
        assert _wait(lambda: all(a.completed == 1 for a in agents))
        _stop(agents, threads)


def test_failed_task_fails_its_lease_only():
    def boom(p):
        if p.get("fail"):
            raise ValueError("bad request")
        return p

    with HiveBroker(pull_poll_s=0.03) as broker:
        agents, threads = _start_agents(broker, [("gpu0", ("generate",), ("m",), boom)])
        bad = broker.submit({"fail": True}, model="m")
        good = broker.submit({"ok": 1}, model="m")
        with pytest.raises(RuntimeError, match="bad request"):
            bad.result(timeout=3)
        assert good.result(timeout=3) == {"ok": 1}
        _stop(agents, threads)


def test_hmac_auth_and_external_bind_guard():
    with pytest.raises(ValueError):
        HiveBroker(host="0.0.0.0")
    with HiveBroker(authkey="local-test-secret", pull_poll_s=0.03) as broker:
        ag = HiveAgent(*broker.address, "auth-agent", caps=("run",), models=("m",), execute=lambda p: p,
                       authkey="local-test-secret")
        t = threading.Thread(target=ag.run, daemon=True)
        t.start()
        assert _wait(lambda: bool(broker.workers()))
        assert broker.submit({"ok": True}, model="m", required_caps=("run",)).result(timeout=3) == {"ok": True}
        _stop([ag], [t])


def test_cost_model_quantiles_and_lease_sizing():
    m = MeasuredCostModel(min_samples=3, history=4)
    for v in (10, 12, 11, 100):
        m.observe(kind="decode", model="qwen", worker="gpu-a", token_budget=16, duration_ms=v)
    e = m.estimate(kind="decode", model="qwen", worker="gpu-a", token_budget=16)
    assert (e.samples, e.p50_ms, e.p95_ms) == (4, 11.5, 100)
    assert m.estimate(kind="decode", model="qwen", worker="gpu-b", token_budget=16) is None
    assert MeasuredCostModel.choose_lease_tokens(throughput_tokens_s=100, fixed_overhead_ms=20,
                                                 max_fixed_fraction=0.2) == 8
    assert MeasuredCostModel.choose_lease_tokens(throughput_tokens_s=100, fixed_overhead_ms=0, min_tokens=4) == 4


def test_planner_never_worsens_with_a_slow_worker():
    pair = plan_homogeneous_batch(16, {"B580": 120, "RX570": 270})
    trio = plan_homogeneous_batch(16, {"B580": 120, "RX570": 270, "M4": 500})
    short = plan_homogeneous_batch(4, {"B580": 10, "RX570": 20, "M4": 200})
    assert trio.predicted_makespan_ms <= pair.predicted_makespan_ms
    assert trio.assignments == {"B580": 10, "RX570": 4, "M4": 2}
    assert short.assignments == {"B580": 3, "RX570": 1, "M4": 0}
    even = plan_homogeneous_batch(16, {f"gpu{i}": 100.0 for i in range(8)})
    assert set(even.assignments.values()) == {2}
    with pytest.raises(ValueError):
        plan_homogeneous_batch(4, {})


def test_batch_reserves_work_by_measured_cost():
    with HiveBroker(pull_poll_s=0.02) as broker:
        agents, threads = _start_agents(broker, [(n, ("generate",), ("qwen",), lambda p: p)
                                                  for n in ("B580", "RX570", "M4")])
        for name, ms in (("B580", 10), ("RX570", 20), ("M4", 200)):
            for _ in range(3):
                broker.cost_model.observe(kind="decode", model="qwen", worker=name, token_budget=4, duration_ms=ms)
        futs = broker.submit_batch([{"n": n} for n in range(4)], model="qwen", required_caps=("generate",),
                                   kind="decode", token_budget=4)
        planned = {n: sum(f.planned_worker_id == n for f in futs) for n in ("B580", "RX570", "M4")}
        assert planned == {"B580": 3, "RX570": 1, "M4": 0}
        assert [f.result(timeout=3) for f in futs] == [{"n": n} for n in range(4)]
        with pytest.raises(RuntimeError, match="missing measured profiles"):
            broker.submit_batch([{"n": 0}], model="qwen", required_caps=("generate",), kind="other", token_budget=4)
        _stop(agents, threads)


# ---- the per-GPU agent layout as gloo ranks ------------------------------------------------------
def _fake_generate(payload):
    """Stands in for a GPU's greedy generation: deterministic in the request."""
    ids = payload["ids"]
    toks = [(sum(ids) * 31 + 7 * i) % 1000 for i in range(payload["max_new_tokens"])]
    return {"tokens": toks, "token_sha256": hashlib.sha256(json.dumps(toks, separators=(",", ":")).encode()).hexdigest()}


def _rank_main(rank, world, port, out):
    import datetime
    import os

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    broker = None
    addr = torch.zeros(1, dtype=torch.int64)
    if rank == 0:
        broker = HiveBroker(pull_poll_s=0.02).start()
        addr[0] = broker.address[1]
    dist.broadcast(addr, 0)
    served = []

    def execute(p):
        served.append(p["request"])
        return _fake_generate(p)

    agent = HiveAgent("127.0.0.1", int(addr.item()), f"gpu{rank}", caps=("generate", "throughput.generate"),
                      models=("qwen2-1.5b",), execute=execute)
    th = threading.Thread(target=agent.run, daemon=True)
    th.start()
    if rank == 0:
        assert _wait(lambda: len(broker.workers()) == world, 20)
        reqs = [{"ids": list(range(i, i + 5)), "max_new_tokens": 4, "request": i} for i in range(16)]
        for _ in range(40):          # warm-up until both workers are measured
            for f in broker.submit_batch(reqs[:2], model="qwen2-1.5b", require_profiles=False, token_budget=4):
                f.result(timeout=20)
            if all(broker.cost_model.estimate(kind="throughput.generate", model="qwen2-1.5b", worker=f"gpu{r}",
                                              token_budget=4) for r in range(world)):
                break
        futs = broker.submit_batch(reqs, model="qwen2-1.5b", token_budget=4)
        results = [f.result(timeout=20) for f in futs]
        planned = sorted(f.planned_worker_id for f in futs)
        broker.close()
        out.put(("results", [r["token_sha256"] for r in results],
                 [_fake_generate(r)["token_sha256"] for r in reqs], planned))
    th.join(timeout=20)
    out.put(("served", rank, len(served), th.is_alive()))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_agents_partition_the_burst():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    msgs = [out.get(timeout=120) for _ in range(3)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res = next(m for m in msgs if m[0] == "results")
    assert res[1] == res[2]                                  # every request's tokens as computed directly
    assert len(res[3]) == 16 and set(res[3]) == {"gpu0", "gpu1"}   # split by measured service time
    served = sorted(m[1:] for m in msgs if m[0] == "served")
    assert all(n >= 1 and not alive for _, n, alive in served)


# ---- the lease queue behind the broker ------------------------------------------------------------
def test_queue_orders_by_priority_then_submission():
    from seedplane_b200.hive.pool import LeaseQueue, WorkerInfo, WorkTile, _Ticket
    q = LeaseQueue()
    mk = lambda rid, prio, model="m": _Ticket(rid, WorkTile(kind="k", model=model, payload={"r": rid}, priority=prio),
                                                time.monotonic() + 60, rid)
    q.put([mk(1, 0), mk(2, 5), mk(3, 0, model="other"), mk(4, 5)])
    w = WorkerInfo("w", frozenset(), frozenset({"m"}), 0.0)
    assert [q.take(w, 0.0).request_id for _ in range(3)] == [2, 4, 1]
    assert q.take(w, 0.01) is None                  # request 3 is for a model w does not serve
    q.close(RuntimeError("closed"))


def test_reserved_work_is_released_when_its_worker_leaves():
    with HiveBroker(pull_poll_s=0.02) as broker:
        agents, threads = _start_agents(broker, [(n, ("generate",), ("qwen",), lambda p: p) for n in ("fast", "slow")])
        for name, ms in (("fast", 5), ("slow", 500)):
            for _ in range(3):
                broker.cost_model.observe(kind="decode", model="qwen", worker=name, token_budget=4, duration_ms=ms)
        _stop(agents[:1], threads[:1])              # the fast worker leaves before the batch
        assert _wait(lambda: set(broker.workers()) == {"slow"})
        futs = broker.submit_batch([{"n": n} for n in range(3)], model="qwen", kind="decode", token_budget=4)
        assert [f.result(timeout=3) for f in futs] == [{"n": 0}, {"n": 1}, {"n": 2}]
        assert {f.worker_id for f in futs} == {"slow"}
        _stop(agents[1:], threads[1:])


def test_local_agent_pulls_without_tcp_and_feeds_the_cost_model():
    with HiveBroker(pull_poll_s=0.02) as broker:
        ag = broker.local_agent("gpu0", caps=("generate",), models=("m",), execute=lambda p: {"twice": 2 * p["x"]})
        t = threading.Thread(target=ag.run, daemon=True)
        t.start()
        assert _wait(lambda: "gpu0" in broker.workers())
        futs = [broker.submit({"x": i}, model="m") for i in range(4)]
        assert [f.result(timeout=3) for f in futs] == [{"twice": 2 * i} for i in range(4)]
        est = broker.cost_model.estimate(kind="throughput.generate", model="m", worker="gpu0", token_budget=0)
        assert est is not None and est.samples == 4
        ag.stop()
        t.join(timeout=3)
        assert not t.is_alive() and "gpu0" not in broker.workers()


def test_unleased_work_expires():
    with HiveBroker(pull_poll_s=0.02) as broker:
        fut = broker.submit({"x": 1}, model="nobody-serves-this", timeout=0.05)
        ag = broker.local_agent("gpu0", caps=("generate",), models=("m",), execute=lambda p: p)
        t = threading.Thread(target=ag.run, daemon=True)
        t.start()
        with pytest.raises(TimeoutError):
            fut.result(timeout=3)
        ag.stop()
        t.join(timeout=3)


def test_grouped_leases_send_each_workers_share_as_one_batch():
    """submit_batch(group_per_worker=True): each planned worker gets ONE lease carrying its share as
    {"batch": [...]}; the agent answers {"batch": [...]} and every request's future resolves to its
    own element; the broker records the batch size the agent reports."""
    seen = {}

    def make(name):
        def execute(p):
            items = p["batch"]
            seen.setdefault(name, []).append(len(items))
            return {"batch": [{"twice": 2 * it["x"]} for it in items]}
        return execute

    with HiveBroker(pull_poll_s=0.02) as broker:
        agents, threads = _start_agents(broker, [(n, ("generate",), ("qwen",), make(n)) for n in ("gpu0", "gpu1")])
        for name in ("gpu0", "gpu1"):
            for _ in range(3):
                broker.cost_model.observe(kind="decode", model="qwen", worker=name, token_budget=4, duration_ms=10)
        futs = broker.submit_batch([{"x": n} for n in range(10)], model="qwen", required_caps=("generate",),
                                   kind="decode", token_budget=4, group_per_worker=True)
        assert [f.result(timeout=3) for f in futs] == [{"twice": 2 * n} for n in range(10)]
        assert sorted(sum(seen.values(), [])) == [5, 5]
        assert {f.planned_worker_id for f in futs} == {"gpu0", "gpu1"}
        est = broker.cost_model.estimate(kind="decode.batch", model="qwen", worker="gpu0", token_budget=4,
                                         batch_size=5)
        assert est is None or est.samples >= 1
        _stop(agents, threads)
    # a malformed batch answer fails every member of that lease
    with HiveBroker(pull_poll_s=0.02) as broker:
        agents, threads = _start_agents(broker, [("bad", ("generate",), ("other",), lambda p: {"batch": []})])
        futs = broker.submit_batch([{"x": 1}, {"x": 2}], model="other", required_caps=("generate",),
                                   require_profiles=False, group_per_worker=True)
        for f in futs:
            with pytest.raises(RuntimeError, match="does not match"):
                f.result(timeout=3)
        _stop(agents, threads)
