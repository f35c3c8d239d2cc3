"""HIVE broker and pull agents (`seedplane/hive/pool.py:18-478` of the reference), same protocol.

Broker: a ready queue of work tiles. Each agent holds one persistent TCP session: optional HMAC
challenge, HELLO (worker id, caps, models), READY, then PULL -> WORK (one leased tile) | WAIT |
STOP, and RESULT for the lease it holds. A tile goes to the first compatible agent that pulls it
(its caps include the tile's required caps and it serves the tile's model), unless a batch plan
reserved it for another worker. The broker times each lease end to end (hand-out to result) into
its `MeasuredCostModel`; `submit_batch` splits interchangeable tiles by those measurements
(`plan_homogeneous_batch`). A lost session fails the tile it held; expired tiles fail with
`TimeoutError`. Without an `authkey` the broker only binds a loopback address.
"""
from __future__ import annotations

import hashlib
import hmac
import ipaddress
import secrets
import socket
import threading
import time
from concurrent.futures import Future
from dataclasses import dataclass, field
from typing import Callable, Optional

from .cost import MeasuredCostModel
from .protocol import Frame, Message, json_payload, parse_json, recv_frame, send_frame
from .scheduler import plan_homogeneous_batch


@dataclass(frozen=True)
class WorkTile:
    """One unit of ready work. `dependencies` is lineage metadata: the submitter waits for them."""
    kind: str
    model: str
    payload: dict
    required_caps: frozenset = frozenset()
    dependencies: tuple = ()
    sequence_range: Optional[tuple] = None
    hidden_range: Optional[tuple] = None
    token_budget: int = 0
    branch_id: int = 0
    predicted_cost: dict = field(default_factory=dict)
    deadline_s: float = 300.0
    priority: int = 0
    movable: bool = False
    stealable: bool = False

    def __post_init__(self):
        if not self.kind or not self.model or not isinstance(self.payload, dict):
            raise ValueError("WorkTile needs kind, model, and an object payload")
        if self.token_budget < 0 or self.deadline_s <= 0:
            raise ValueError("WorkTile token budget must be non-negative and deadline positive")
        for name in ("sequence_range", "hidden_range"):
            r = getattr(self, name)
            if r is not None and (len(r) != 2 or r[0] < 0 or r[1] <= r[0]):
                raise ValueError(f"invalid WorkTile {name}")
        object.__setattr__(self, "required_caps", frozenset(self.required_caps))
        object.__setattr__(self, "dependencies", tuple(self.dependencies))

    def envelope(self, ttl_s: float) -> dict:
        return {"kind": self.kind, "model": self.model, "payload": self.payload,
                "dependencies": self.dependencies, "sequence_range": self.sequence_range,
                "hidden_range": self.hidden_range, "token_budget": self.token_budget, "branch_id": self.branch_id,
                "predicted_cost": self.predicted_cost, "movable": self.movable, "stealable": self.stealable,
                "lease_ttl_s": max(0.0, ttl_s)}


@dataclass
class _Item:
    request_id: int
    tile: WorkTile
    deadline: float
    future: Future
    order: int
    lease: int = 0
    worker: Optional[str] = None
    reserved_for: Optional[str] = None
    leased_at: Optional[float] = None


class WorkFuture:
    """The caller's handle on a submitted tile."""

    def __init__(self, item: _Item):
        self._item = item
        self.request_id = item.request_id

    @property
    def worker_id(self):
        return self._item.worker

    @property
    def planned_worker_id(self):
        return self._item.reserved_for

    def result(self, timeout=None):
        return self._item.future.result(timeout)

    def done(self):
        return self._item.future.done()

    def add_done_callback(self, fn):
        self._item.future.add_done_callback(fn)


def _fail(item: _Item, exc: BaseException):
    if not item.future.done():
        item.future.set_exception(exc)


class HiveBroker:
    def __init__(self, host="127.0.0.1", port=0, authkey=None, pull_poll_s=0.25):
        self.host, self.port = host, int(port)
        self.authkey = authkey.encode() if isinstance(authkey, str) else authkey
        if not self._loopback(host) and not self.authkey:
            raise ValueError("non-loopback HIVE broker requires an explicit authkey")
        if pull_poll_s <= 0:
            raise ValueError("pull_poll_s must be positive")
        self.pull_poll_s = float(pull_poll_s)
        self.cost_model = MeasuredCostModel()
        self._cv = threading.Condition(threading.RLock())
        self._queue = []
        self._workers = {}
        self._conns = set()
        self._threads = []
        self._ids = 0
        self._leases = 0
        self._closing = False
        self._sock = None
        self._acceptor = None

    @staticmethod
    def _loopback(host) -> bool:
        try:
            return ipaddress.ip_address(host).is_loopback
        except ValueError:
            return str(host).lower() == "localhost"

    @property
    def address(self):
        if self._sock is None:
            raise RuntimeError("broker is not started")
        return self._sock.getsockname()[:2]

    def start(self):
        if self._sock is not None:
            raise RuntimeError("broker already started")
        s = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        s.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        s.bind((self.host, self.port))
        s.listen(64)
        s.settimeout(0.25)
        self._sock = s
        self.host, self.port = s.getsockname()[:2]
        self._acceptor = threading.Thread(target=self._accept_loop, name="hive-accept", daemon=True)
        self._acceptor.start()
        return self

    # ---- submission ------------------------------------------------------------------------
    def _enqueue(self, tile: WorkTile, reserved_for=None) -> WorkFuture:
        self._ids += 1
        item = _Item(self._ids, tile, time.monotonic() + tile.deadline_s, Future(), self._ids,
                     reserved_for=reserved_for)
        self._queue.append(item)
        return WorkFuture(item)

    def _sort(self):
        self._queue.sort(key=lambda it: (-it.tile.priority, it.order))

    def submit(self, payload, *, model, required_caps=("generate",), priority=0, timeout=300,
               kind="throughput.generate", dependencies=(), sequence_range=None, hidden_range=None,
               token_budget=0, branch_id=0, predicted_cost=None, movable=False, stealable=False) -> WorkFuture:
        if timeout <= 0:
            raise ValueError("timeout must be positive")
        tile = WorkTile(kind=kind, model=model, payload=dict(payload), required_caps=frozenset(required_caps),
                        dependencies=tuple(dependencies), sequence_range=sequence_range, hidden_range=hidden_range,
                        token_budget=token_budget, branch_id=branch_id, predicted_cost=dict(predicted_cost or {}),
                        deadline_s=timeout, priority=priority, movable=movable, stealable=stealable)
        with self._cv:
            if self._closing or self._sock is None:
                raise RuntimeError("broker is not running")
            fut = self._enqueue(tile, self._fastest_profiled(tile))
            self._sort()
            self._cv.notify_all()
            return fut

    def submit_batch(self, payloads, *, model, required_caps=("generate",), priority=0, timeout=300,
                     kind="throughput.generate", token_budget=0, predicted_cost=None, require_profiles=True):
        """Interchangeable independent tiles, split over the measured workers to minimise the
        predicted makespan (a slow worker may get none). A generation request is never split."""
        payloads = list(payloads)
        if not payloads:
            return []
        if timeout <= 0 or any(not isinstance(p, dict) for p in payloads):
            raise ValueError("batch needs object payloads and a positive timeout")
        tiles = [WorkTile(kind=kind, model=model, payload=dict(p), required_caps=frozenset(required_caps),
                          token_budget=token_budget, predicted_cost=dict(predicted_cost or {}), deadline_s=timeout,
                          priority=priority) for p in payloads]
        with self._cv:
            if self._closing or self._sock is None:
                raise RuntimeError("broker is not running")
            eligible = [w for w, info in self._workers.items() if self._serves(info, tiles[0])]
            profiles = {}
            for w in eligible:
                est = self.cost_model.estimate(kind=kind, model=model, worker=w, token_budget=token_budget)
                if est is not None:
                    profiles[w] = est.p50_ms
            if require_profiles and (not eligible or len(profiles) != len(eligible)):
                raise RuntimeError("cannot plan safe HIVE batch; missing measured profiles: "
                                   f"{sorted(set(eligible) - set(profiles))}")
            order = []
            if profiles:
                plan = plan_homogeneous_batch(len(tiles), profiles)
                for w in sorted(plan.assignments, key=lambda w: (profiles[w], w)):
                    order += [w] * plan.assignments[w]
            futs = [self._enqueue(t, order[i] if order else None) for i, t in enumerate(tiles)]
            self._sort()
            self._cv.notify_all()
            return futs

    @staticmethod
    def _serves(info, tile: WorkTile) -> bool:
        return tile.model in info["models"] and tile.required_caps <= info["caps"]

    def _fastest_profiled(self, tile: WorkTile):
        ests = {}
        for w, info in self._workers.items():
            if self._serves(info, tile):
                e = self.cost_model.estimate(kind=tile.kind, model=tile.model, worker=w,
                                             token_budget=tile.token_budget)
                if e is None:
                    return None
                ests[w] = e.p50_ms
        return min(ests, key=lambda w: (ests[w], w)) if ests else None

    def workers(self):
        with self._cv:
            return {w: {"caps": sorted(i["caps"]), "models": sorted(i["models"]), "connected_at": i["connected_at"]}
                    for w, i in self._workers.items()}

    # ---- sessions --------------------------------------------------------------------------
    def _accept_loop(self):
        while not self._closing:
            try:
                conn, _ = self._sock.accept()
            except socket.timeout:
                continue
            except OSError:
                return
            conn.settimeout(30)
            t = threading.Thread(target=self._session, args=(conn,), daemon=True)
            with self._cv:
                self._conns.add(conn)
                self._threads.append(t)
            t.start()

    def _authenticate(self, conn):
        if not self.authkey:
            return
        challenge = secrets.token_bytes(32)
        send_frame(conn, Frame(Message.AUTH_CHALLENGE, payload=challenge))
        reply = recv_frame(conn)
        want = hmac.new(self.authkey, challenge, hashlib.sha256).digest()
        if reply.kind != Message.AUTH or not hmac.compare_digest(reply.payload, want):
            raise PermissionError("HIVE agent authentication failed")

    def _lease(self, worker) -> Optional[_Item]:
        """The first compatible tile (not reserved for another worker), waiting at most one poll period."""
        until = time.monotonic() + self.pull_poll_s
        with self._cv:
            while not self._closing:
                now = time.monotonic()
                live = []
                for it in self._queue:
                    if it.deadline <= now:
                        _fail(it, TimeoutError(f"HIVE work {it.request_id} expired in queue"))
                    else:
                        live.append(it)
                self._queue = live
                for k, it in enumerate(self._queue):
                    if self._serves(worker, it.tile) and it.reserved_for in (None, worker["id"]):
                        del self._queue[k]
                        self._leases += 1
                        it.lease, it.worker, it.leased_at = self._leases, worker["id"], time.monotonic()
                        return it
                left = until - time.monotonic()
                if left <= 0:
                    return None
                self._cv.wait(left)
            return None

    def _session(self, conn):
        wid, held = None, None
        try:
            self._authenticate(conn)
            hello = recv_frame(conn)
            if hello.kind != Message.HELLO:
                raise ValueError("first authenticated HIVE message must be HELLO")
            meta = parse_json(hello.payload)
            wid = str(meta.get("worker_id", "")).strip()
            if not wid:
                raise ValueError("agent HELLO missing worker_id")
            worker = {"id": wid, "caps": frozenset(map(str, meta.get("caps", []))),
                      "models": frozenset(map(str, meta.get("models", []))), "connected_at": time.time()}
            with self._cv:
                if wid in self._workers:
                    wid = None
                    raise ValueError("duplicate connected worker_id")
                self._workers[worker["id"]] = worker
                self._cv.notify_all()
            conn.settimeout(None)
            send_frame(conn, Frame(Message.READY, payload=json_payload({"protocol": 1})))
            while not self._closing:
                pull = recv_frame(conn)
                if pull.kind == Message.STOP:
                    break
                if pull.kind != Message.PULL:
                    raise ValueError(f"expected PULL, received {pull.kind.name}")
                held = self._lease(worker)
                if held is None:
                    send_frame(conn, Frame(Message.STOP if self._closing else Message.WAIT))
                    if self._closing:
                        break
                    continue
                send_frame(conn, Frame(Message.WORK, held.request_id, held.lease,
                                       json_payload(held.tile.envelope(held.deadline - time.monotonic()))))
                res = recv_frame(conn)
                if res.kind != Message.RESULT or res.request_id != held.request_id or res.sequence != held.lease:
                    raise ValueError("HIVE result does not match active work lease")
                data = parse_json(res.payload)
                if held.deadline <= time.monotonic():
                    _fail(held, TimeoutError(f"HIVE work {held.request_id} lease expired"))
                elif data.get("ok"):
                    m = data.get("metrics", {})
                    self.cost_model.observe(kind=held.tile.kind, model=held.tile.model, worker=wid,
                                            token_budget=held.tile.token_budget,
                                            duration_ms=max(1e-6, (time.monotonic() - held.leased_at) * 1000.0),
                                            batch_size=int(m.get("batch_size", 1)), load=float(m.get("load", 0.0)))
                    if not held.future.done():
                        held.future.set_result(data.get("result"))
                else:
                    _fail(held, RuntimeError(str(data.get("error", "agent execution failed"))))
                held = None
        except (OSError, ConnectionError, TimeoutError, ValueError, PermissionError) as exc:
            if held is not None:
                _fail(held, ConnectionError(f"worker {wid} lost lease: {exc}"))
        finally:
            with self._cv:
                if wid:
                    self._workers.pop(wid, None)
                self._conns.discard(conn)
                self._cv.notify_all()
            try:
                conn.close()
            except OSError:
                pass

    def close(self):
        with self._cv:
            if self._closing:
                return
            self._closing = True
            for it in self._queue:
                _fail(it, RuntimeError("HIVE broker closed before work was leased"))
            self._queue.clear()
            self._cv.notify_all()
            conns = list(self._conns)
        if self._sock is not None:
            self._sock.close()
        for c in conns:
            try:
                send_frame(c, Frame(Message.STOP))
            except OSError:
                pass
        if self._acceptor is not None:
            self._acceptor.join(timeout=1)
        for t in list(self._threads):
            t.join(timeout=1)
        for c in conns:
            try:
                c.shutdown(socket.SHUT_RDWR)
            except OSError:
                pass
            c.close()

    def __enter__(self):
        return self.start()

    def __exit__(self, *exc):
        self.close()


class HiveAgent:
    """A persistent pull agent; `execute(payload) -> result` owns the local model (one per GPU)."""

    def __init__(self, host, port, worker_id, *, caps, models, execute: Callable, authkey=None, connect_timeout=10):
        self.host, self.port = host, int(port)
        self.worker_id = str(worker_id)
        self.caps = sorted(set(map(str, caps)))
        self.models = sorted(set(map(str, models)))
        self.execute = execute
        self.authkey = authkey.encode() if isinstance(authkey, str) else authkey
        self.connect_timeout = connect_timeout
        self._stop = threading.Event()
        self.sock = None
        self.completed = 0

    def stop(self):
        self._stop.set()

    def run(self):
        self.sock = socket.create_connection((self.host, self.port), timeout=self.connect_timeout)
        self.sock.settimeout(None)
        try:
            if self.authkey:
                ch = recv_frame(self.sock)
                if ch.kind != Message.AUTH_CHALLENGE:
                    raise ValueError("expected HIVE authentication challenge")
                send_frame(self.sock, Frame(Message.AUTH, payload=hmac.new(self.authkey, ch.payload,
                                                                           hashlib.sha256).digest()))
            send_frame(self.sock, Frame(Message.HELLO, payload=json_payload(
                {"worker_id": self.worker_id, "caps": self.caps, "models": self.models})))
            if recv_frame(self.sock).kind != Message.READY:
                raise RuntimeError("HIVE broker did not accept agent HELLO")
            while not self._stop.is_set():
                send_frame(self.sock, Frame(Message.PULL))
                f = recv_frame(self.sock)
                if f.kind == Message.STOP:
                    break
                if f.kind == Message.WAIT:
                    continue
                if f.kind == Message.ERROR:
                    raise RuntimeError(parse_json(f.payload).get("error", "broker error"))
                if f.kind != Message.WORK:
                    raise ValueError(f"unexpected broker message {f.kind.name}")
                env = parse_json(f.payload)
                try:
                    t0 = time.perf_counter()
                    result = self.execute(env["payload"])
                    reply = {"ok": True, "result": result,
                             "metrics": {"duration_ms": (time.perf_counter() - t0) * 1000.0, "batch_size": 1}}
                except Exception as exc:          # a failed task fails its lease, not the agent
                    reply = {"ok": False, "error": f"{type(exc).__name__}: {exc}"}
                send_frame(self.sock, Frame(Message.RESULT, f.request_id, f.sequence, json_payload(reply)))
                self.completed += 1
        except (OSError, ConnectionError):
            if not self._stop.is_set():
                raise
        finally:
            if self.sock is not None:
                self.sock.close()
                self.sock = None
