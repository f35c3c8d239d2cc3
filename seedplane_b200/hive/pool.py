"""HIVE broker and pull agents: the public surface of the reference's `seedplane/hive/pool.py`
(`WorkTile`, `WorkFuture`, `HiveBroker`, `HiveAgent`) over its wire protocol, built around an
in-process lease queue.

Scheduling core: `LeaseQueue`, which knows nothing of sockets. A submitted tile becomes a ticket
in one heap keyed by (-priority, submission order): the heap of its work class (model, required
caps) when any compatible worker may take it, or the heap of one worker when a batch plan reserved
it for that worker. A worker takes the best head among its own heap and the class heaps it is
compatible with (its models hold the class's model, its caps the class's caps), so a take costs a
few heap operations instead of a scan of the queue. Deadlines sit in a third heap and expire
lazily, failing their futures with `TimeoutError`. When a worker leaves, its reserved tickets go
back to their class heaps.

Transport: `HiveBroker` adds a TCP listener; each agent connection is a `_Session` thread that
answers PULL with `LeaseQueue.take` (waiting at most `pull_poll_s`, then WAIT), sends WORK, and
settles the ticket from the RESULT. The broker times every lease from hand-out to result and feeds
its `MeasuredCostModel`, which `submit` and `submit_batch` use to place work. `LocalAgent` pulls
from the same queue in the broker's process, with no TCP, for executors that live beside the
broker. Without an `authkey` the broker binds loopback addresses only; with one, every connection
first answers an HMAC-SHA256 challenge.
"""
from __future__ import annotations

import hashlib
import heapq
import hmac
import ipaddress
import itertools
import secrets
import socket
import threading
import time
from concurrent.futures import Future
from dataclasses import dataclass, field
from typing import Callable, Dict, FrozenSet, Iterable, List, Optional, Tuple

from .cost import MeasuredCostModel
from .protocol import Frame, Message, json_payload, parse_json, recv_frame, send_frame
from .scheduler import plan_homogeneous_batch


@dataclass(frozen=True)
class WorkTile:
    """One unit of ready work. `dependencies` is lineage only: a submitter waits for them itself."""
    kind: str
    model: str
    payload: dict
    required_caps: FrozenSet[str] = frozenset()
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
        if not (self.kind and self.model) or not isinstance(self.payload, dict):
            raise ValueError("a WorkTile needs a kind, a model and a dict payload")
        if self.token_budget < 0:
            raise ValueError("a WorkTile's token budget cannot be negative")
        if not self.deadline_s > 0:
            raise ValueError("a WorkTile's deadline must be positive")
        for name in ("sequence_range", "hidden_range"):
            span = getattr(self, name)
            if span is not None:
                ok = len(span) == 2 and 0 <= span[0] < span[1]
                if not ok:
                    raise ValueError(f"WorkTile {name} must be (start, end) with 0 <= start < end")
        object.__setattr__(self, "required_caps", frozenset(map(str, self.required_caps)))
        object.__setattr__(self, "dependencies", tuple(self.dependencies))

    @property
    def work_class(self) -> Tuple[str, FrozenSet[str]]:
        return self.model, self.required_caps

    def to_wire(self, ttl_s: float) -> dict:
        """The WORK message's JSON object."""
        d = {name: getattr(self, name) for name in ("kind", "model", "payload", "dependencies", "sequence_range",
                                                     "hidden_range", "token_budget", "branch_id", "predicted_cost",
                                                     "movable", "stealable")}
        d["lease_ttl_s"] = ttl_s if ttl_s > 0 else 0.0
        return d


@dataclass(frozen=True)
class WorkerInfo:
    """A connected worker as the queue sees it."""
    worker_id: str
    caps: FrozenSet[str]
    models: FrozenSet[str]
    connected_at: float

    def can_run(self, work_class) -> bool:
        model, caps = work_class
        return model in self.models and caps <= self.caps


_PENDING, _LEASED, _SETTLED = 0, 1, 2


@dataclass(eq=False)
class _Ticket:
    request_id: int
    tile: WorkTile
    expires: float
    order: int
    reserved_for: Optional[str] = None
    future: Future = field(default_factory=Future)
    state: int = _PENDING
    lease: int = 0
    worker: Optional[str] = None
    leased_at: float = 0.0

    def heap_entry(self):
        return (-self.tile.priority, self.order, self)

    def settle(self, result=None, error: Optional[BaseException] = None) -> None:
        self.state = _SETTLED
        if self.future.done():
            return
        if error is not None:
            self.future.set_exception(error)
        else:
            self.future.set_result(result)


class WorkFuture:
    """A caller's handle on one submitted tile."""

    def __init__(self, ticket: _Ticket):
        self._t = ticket
        self.request_id = ticket.request_id

    @property
    def worker_id(self) -> Optional[str]:
        """The worker that leased the tile (None while queued)."""
        return self._t.worker

    @property
    def planned_worker_id(self) -> Optional[str]:
        """The worker a plan reserved the tile for (None: any compatible worker)."""
        return self._t.reserved_for

    def result(self, timeout=None):
        return self._t.future.result(timeout)

    def done(self) -> bool:
        return self._t.future.done()

    def add_done_callback(self, fn) -> None:
        self._t.future.add_done_callback(fn)


class BatchMemberFuture(WorkFuture):
    """One request of a grouped lease (`submit_batch(..., group_per_worker=True)`): its result is
    element `index` of the group's `{"batch": [...]}` result."""

    def __init__(self, ticket: _Ticket, index: int):
        super().__init__(ticket)
        self.index = index

    def result(self, timeout=None):
        res = self._t.future.result(timeout)
        items = res.get("batch") if isinstance(res, dict) else None
        if not isinstance(items, list) or len(items) != len(self._t.tile.payload["batch"]):
            raise RuntimeError("the agent's batch result does not match the batch it was given")
        return items[self.index]


class LeaseQueue:
    """Ready tickets in heaps by work class and by reserved worker; see the module docstring."""

    def __init__(self):
        self._cv = threading.Condition()
        self._by_class: Dict[tuple, list] = {}
        self._by_worker: Dict[str, list] = {}
        self._expiry: list = []
        self._lease_ids = itertools.count(1)
        self._closed: Optional[BaseException] = None

    def put(self, tickets: Iterable[_Ticket]) -> None:
        with self._cv:
            if self._closed is not None:
                raise RuntimeError("the HIVE queue is closed")
            for t in tickets:
                self._push(t)
                heapq.heappush(self._expiry, (t.expires, t.order, t))
            self._cv.notify_all()

    def _push(self, t: _Ticket) -> None:
        lane = self._by_worker if t.reserved_for is not None else self._by_class
        key = t.reserved_for if t.reserved_for is not None else t.tile.work_class
        heapq.heappush(lane.setdefault(key, []), t.heap_entry())

    def _expire(self, now: float) -> None:
        while self._expiry and self._expiry[0][0] <= now:
            _, _, t = heapq.heappop(self._expiry)
            if t.state == _PENDING:
                t.settle(error=TimeoutError(f"HIVE work {t.request_id} expired before any worker leased it"))

    @staticmethod
    def _head(heap: list) -> Optional[_Ticket]:
        while heap and heap[0][2].state != _PENDING:
            heapq.heappop(heap)
        return heap[0][2] if heap else None

    def _best_for(self, w: WorkerInfo) -> Optional[_Ticket]:
        mine = self._by_worker.get(w.worker_id)
        while mine:
            t = self._head(mine)
            if t is None or w.can_run(t.tile.work_class):
                break
            heapq.heappop(mine)             # reserved for w, which can no longer run it: unreserve
            t.reserved_for = None
            self._push(t)
        best, best_heap = None, None
        for heap in [mine] + [h for cls, h in self._by_class.items() if w.can_run(cls)]:
            t = self._head(heap) if heap else None
            if t is not None and (best is None or (-t.tile.priority, t.order) < (-best.tile.priority, best.order)):
                best, best_heap = t, heap
        if best is not None:
            heapq.heappop(best_heap)
        return best

    def take(self, w: WorkerInfo, wait_s: float) -> Optional[_Ticket]:
        """The best ticket `w` may run, waiting up to `wait_s` for one; None on timeout or close."""
        give_up = time.monotonic() + wait_s
        with self._cv:
            while self._closed is None:
                now = time.monotonic()
                self._expire(now)
                t = self._best_for(w)
                if t is not None:
                    t.state, t.worker, t.leased_at = _LEASED, w.worker_id, now
                    t.lease = next(self._lease_ids)
                    return t
                if now >= give_up:
                    return None
                self._cv.wait(give_up - now)
            return None

    def release_reserved(self, worker_id: str) -> None:
        """Work reserved for a worker that left goes back to its class heap."""
        with self._cv:
            for _, _, t in self._by_worker.pop(worker_id, []):
                if t.state == _PENDING:
                    t.reserved_for = None
                    self._push(t)
            self._cv.notify_all()

    def close(self, reason: BaseException) -> None:
        with self._cv:
            if self._closed is not None:
                return
            self._closed = reason
            for _, _, t in self._expiry:
                if t.state == _PENDING:
                    t.settle(error=reason)
            self._expiry.clear()
            self._by_class.clear()
            self._by_worker.clear()
            self._cv.notify_all()


def _is_loopback(host) -> bool:
    if str(host).lower() == "localhost":
        return True
    try:
        return ipaddress.ip_address(host).is_loopback
    except ValueError:
        return False


def _hmac(key: bytes, challenge: bytes) -> bytes:
    return hmac.new(key, challenge, hashlib.sha256).digest()


class HiveBroker:
    """The coordinator: a `LeaseQueue`, the connected workers, their measured costs, a listener."""

    def __init__(self, host="127.0.0.1", port=0, authkey=None, pull_poll_s=0.25):
        self.authkey = authkey.encode() if isinstance(authkey, str) else authkey
        if not self.authkey and not _is_loopback(host):
            raise ValueError(f"a HIVE broker on {host!r} (not loopback) needs an authkey")
        if not pull_poll_s > 0:
            raise ValueError("pull_poll_s must be positive")
        self.host, self.port = host, int(port)
        self.pull_poll_s = float(pull_poll_s)
        self.cost_model = MeasuredCostModel()
        self._queue = LeaseQueue()
        self._reg_lock = threading.Lock()
        self._registry: Dict[str, WorkerInfo] = {}
        self._sessions: set = set()
        self._request_ids = itertools.count(1)
        self._listener: Optional[socket.socket] = None
        self._acceptor: Optional[threading.Thread] = None
        self._stopping = threading.Event()

    # ---- life cycle --------------------------------------------------------------------------
    @property
    def address(self) -> Tuple[str, int]:
        if self._listener is None:
            raise RuntimeError("the HIVE broker has not been started")
        return self._listener.getsockname()[:2]

    def start(self) -> "HiveBroker":
        if self._listener is not None:
            raise RuntimeError("the HIVE broker is already running")
        ls = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        ls.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        ls.bind((self.host, self.port))
        ls.listen(64)
        ls.settimeout(0.25)
        self._listener = ls
        self.host, self.port = ls.getsockname()[:2]
        self._acceptor = threading.Thread(target=self._accept, name="hive-listener", daemon=True)
        self._acceptor.start()
        return self

    def close(self) -> None:
        if self._stopping.is_set():
            return
        self._stopping.set()
        self._queue.close(RuntimeError("the HIVE broker closed before this work was leased"))
        if self._listener is not None:
            self._listener.close()
        with self._reg_lock:
            sessions = list(self._sessions)
        for s in sessions:
            s.say_stop()
        if self._acceptor is not None:
            self._acceptor.join(timeout=1)
        for s in sessions:
            s.join(timeout=1)
        for s in sessions:
            s.shut()

    def __enter__(self):
        return self.start()

    def __exit__(self, *exc):
        self.close()

    def _check_running(self):
        if self._listener is None or self._stopping.is_set():
            raise RuntimeError("the HIVE broker is not running")

    # ---- workers -----------------------------------------------------------------------------
    def workers(self) -> Dict[str, dict]:
        with self._reg_lock:
            return {w: {"caps": sorted(i.caps), "models": sorted(i.models), "connected_at": i.connected_at}
                    for w, i in self._registry.items()}

    def _join(self, info: WorkerInfo) -> None:
        with self._reg_lock:
            if info.worker_id in self._registry:
                raise ValueError(f"a worker named {info.worker_id!r} is already connected")
            self._registry[info.worker_id] = info

    def _leave(self, worker_id: str) -> None:
        with self._reg_lock:
            self._registry.pop(worker_id, None)
        self._queue.release_reserved(worker_id)

    def _service_ms(self, tile: WorkTile, workers: Iterable[str]) -> Dict[str, Optional[float]]:
        out = {}
        for w in workers:
            est = self.cost_model.estimate(kind=tile.kind, model=tile.model, worker=w, token_budget=tile.token_budget)
            out[w] = None if est is None else est.p50_ms
        return out

    def _capable(self, tile: WorkTile) -> List[str]:
        with self._reg_lock:
            return [w for w, info in self._registry.items() if info.can_run(tile.work_class)]

    # ---- submission --------------------------------------------------------------------------
    def _ticket(self, tile: WorkTile, reserved_for: Optional[str]) -> _Ticket:
        rid = next(self._request_ids)
        return _Ticket(rid, tile, time.monotonic() + tile.deadline_s, rid, reserved_for)

    def submit(self, payload, *, model, required_caps=("generate",), priority=0, timeout=300,
               kind="throughput.generate", dependencies=(), sequence_range=None, hidden_range=None,
               token_budget=0, branch_id=0, predicted_cost=None, movable=False, stealable=False) -> WorkFuture:
        """Queue one ready tile. When every capable worker has a measured service time, the tile is
        reserved for the fastest of them (ties: by name); otherwise any capable worker takes it."""
        if not timeout > 0:
            raise ValueError("timeout must be positive")
        tile = WorkTile(kind=kind, model=model, payload=dict(payload), required_caps=frozenset(required_caps),
                        dependencies=tuple(dependencies), sequence_range=sequence_range, hidden_range=hidden_range,
                        token_budget=token_budget, branch_id=branch_id, predicted_cost=dict(predicted_cost or {}),
                        deadline_s=timeout, priority=priority, movable=movable, stealable=stealable)
        self._check_running()
        ms = self._service_ms(tile, self._capable(tile))
        fastest = None
        if ms and all(v is not None for v in ms.values()):
            fastest = min(ms, key=lambda w: (ms[w], w))
        t = self._ticket(tile, fastest)
        self._queue.put([t])
        return WorkFuture(t)

    def submit_batch(self, payloads, *, model, required_caps=("generate",), priority=0, timeout=300,
                     kind="throughput.generate", token_budget=0, predicted_cost=None,
                     require_profiles=True, group_per_worker=False) -> List[WorkFuture]:
        """Queue interchangeable, independent tiles split over the capable workers so that the
        predicted makespan (by measured median service times) is least; a slow worker may get
        none. With `require_profiles`, every capable worker must have been measured. Requests are
        never split.

        `group_per_worker`: each worker's share goes out as ONE lease whose payload is
        `{"batch": [payload, ...]}` (kind `<kind>.batch`), for agents that run a batch of requests
        together (runtime request batching, one set of decode steps for all of them); the agent
        answers `{"batch": [result, ...]}` in the same order and reports the batch size in its
        metrics. The returned futures are still one per request, in payload order."""
        payloads = list(payloads)
        if not payloads:
            return []
        if not timeout > 0:
            raise ValueError("timeout must be positive")
        if not all(isinstance(p, dict) for p in payloads):
            raise ValueError("every batch payload must be a dict")
        tiles = [WorkTile(kind=kind, model=model, payload=dict(p), required_caps=frozenset(required_caps),
                          token_budget=token_budget, predicted_cost=dict(predicted_cost or {}), deadline_s=timeout,
                          priority=priority) for p in payloads]
        self._check_running()
        ms = self._service_ms(tiles[0], self._capable(tiles[0]))
        measured = {w: v for w, v in ms.items() if v is not None}
        if require_profiles and (not ms or len(measured) < len(ms)):
            unmeasured = sorted(w for w, v in ms.items() if v is None)
            raise RuntimeError(f"batch planning needs measured service times; missing measured profiles for "
                               f"{unmeasured if ms else 'any capable worker'}")
        owners: List[Optional[str]] = [None] * len(tiles)
        if measured:
            plan = plan_homogeneous_batch(len(tiles), measured)
            fastest_first = sorted(plan.assignments, key=lambda w: (measured[w], w))
            owners = [w for w in fastest_first for _ in range(plan.assignments[w])]
        if group_per_worker:
            futures: List[WorkFuture] = []
            tickets = []
            for owner, idx in _runs(owners):
                group = WorkTile(kind=kind + ".batch", model=model, payload={"batch": [payloads[i] for i in idx]},
                                 required_caps=frozenset(required_caps), token_budget=token_budget,
                                 predicted_cost=dict(predicted_cost or {}), deadline_s=timeout, priority=priority)
                t = self._ticket(group, owner)
                tickets.append(t)
                futures += [BatchMemberFuture(t, j) for j in range(len(idx))]
            self._queue.put(tickets)
            return futures
        tickets = [self._ticket(tile, owner) for tile, owner in zip(tiles, owners)]
        self._queue.put(tickets)
        return [WorkFuture(t) for t in tickets]

    # ---- leases --------------------------------------------------------------------------------
    def _lease(self, info: WorkerInfo) -> Optional[_Ticket]:
        return self._queue.take(info, self.pull_poll_s)

    def _settle(self, t: _Ticket, worker_id: str, reply: dict) -> None:
        """A lease's result: late results fail the ticket; ok ones are timed into the cost model."""
        now = time.monotonic()
        if now >= t.expires:
            t.settle(error=TimeoutError(f"HIVE work {t.request_id}: the lease expired before its result"))
            return
        if not reply.get("ok"):
            t.settle(error=RuntimeError(str(reply.get("error", "the agent failed to execute the work"))))
            return
        metrics = reply.get("metrics") or {}
        # hand-out to result: transport, (de)serialisation and execution, as the broker sees it
        self.cost_model.observe(kind=t.tile.kind, model=t.tile.model, worker=worker_id,
                                token_budget=t.tile.token_budget, duration_ms=max(1e-6, (now - t.leased_at) * 1e3),
                                batch_size=int(metrics.get("batch_size", 1)), load=float(metrics.get("load", 0.0)))
        t.settle(result=reply.get("result"))

    def local_agent(self, worker_id, *, caps, models, execute: Callable) -> "LocalAgent":
        """An agent in this process that pulls from the queue directly (no TCP)."""
        return LocalAgent(self, worker_id, caps=caps, models=models, execute=execute)

    # ---- connections ---------------------------------------------------------------------------
    def _accept(self) -> None:
        while not self._stopping.is_set():
            try:
                conn, _ = self._listener.accept()
            except socket.timeout:
                continue
            except OSError:
                return
            s = _Session(self, conn)
            with self._reg_lock:
                self._sessions.add(s)
            s.start()

    def _session_ended(self, s: "_Session") -> None:
        with self._reg_lock:
            self._sessions.discard(s)


class _Session(threading.Thread):
    """One agent connection on the broker side: handshake, then PULL / WORK / RESULT turns."""

    def __init__(self, broker: HiveBroker, conn: socket.socket):
        super().__init__(name="hive-session", daemon=True)
        self.broker, self.conn = broker, conn
        self.info: Optional[WorkerInfo] = None
        self.held: Optional[_Ticket] = None
        self._send_lock = threading.Lock()    # close() sends STOP from another thread

    def _send(self, frame: Frame) -> None:
        with self._send_lock:
            send_frame(self.conn, frame)

    def say_stop(self) -> None:
        try:
            self._send(Frame(Message.STOP))
        except OSError:
            pass

    def shut(self) -> None:
        try:
            self.conn.shutdown(socket.SHUT_RDWR)
        except OSError:
            pass

    def _handshake(self) -> WorkerInfo:
        self.conn.settimeout(30)
        key = self.broker.authkey
        if key:
            challenge = secrets.token_bytes(32)
            self._send(Frame(Message.AUTH_CHALLENGE, payload=challenge))
            answer = recv_frame(self.conn)
            if answer.kind != Message.AUTH or not hmac.compare_digest(answer.payload, _hmac(key, challenge)):
                raise PermissionError("the agent failed the HIVE authentication challenge")
        hello = recv_frame(self.conn)
        if hello.kind != Message.HELLO:
            raise ValueError(f"an agent must open with HELLO, not {hello.kind.name}")
        meta = parse_json(hello.payload)
        wid = str(meta.get("worker_id", "")).strip()
        if not wid:
            raise ValueError("the agent's HELLO carries no worker_id")
        info = WorkerInfo(wid, frozenset(map(str, meta.get("caps", []))), frozenset(map(str, meta.get("models", []))),
                          time.time())
        self.broker._join(info)
        self.conn.settimeout(None)
        self._send(Frame(Message.READY, payload=json_payload({"protocol": 1})))
        return info

    def _turn(self) -> bool:
        """One PULL: False once the session should end."""
        msg = recv_frame(self.conn)
        if msg.kind == Message.STOP:
            return False
        if msg.kind != Message.PULL:
            raise ValueError(f"the agent sent {msg.kind.name} where PULL was expected")
        t = self.broker._lease(self.info)
        if t is None:
            stopping = self.broker._stopping.is_set()
            self._send(Frame(Message.STOP if stopping else Message.WAIT))
            return not stopping
        self.held = t
        self._send(Frame(Message.WORK, t.request_id, t.lease,
                                    json_payload(t.tile.to_wire(t.expires - time.monotonic()))))
        res = recv_frame(self.conn)
        if res.kind != Message.RESULT or (res.request_id, res.sequence) != (t.request_id, t.lease):
            raise ValueError("the agent's RESULT does not answer the lease it holds")
        self.broker._settle(t, self.info.worker_id, parse_json(res.payload))
        self.held = None
        return True

    def run(self) -> None:
        try:
            self.info = self._handshake()
            while not self.broker._stopping.is_set() and self._turn():
                pass
        except (OSError, ConnectionError, TimeoutError, ValueError, PermissionError) as exc:
            if self.held is not None:
                who = self.info.worker_id if self.info else "?"
                self.held.settle(error=ConnectionError(f"HIVE worker {who} dropped its lease: {exc}"))
        finally:
            if self.info is not None:
                self.broker._leave(self.info.worker_id)
            self.broker._session_ended(self)
            try:
                self.conn.close()
            except OSError:
                pass


def _runs(owners: List[Optional[str]]):
    """(owner, indices) of each maximal run of equal owners (a batch plan lists every worker's share
    contiguously)."""
    out: List[Tuple[Optional[str], List[int]]] = []
    for i, w in enumerate(owners):
        if out and out[-1][0] == w:
            out[-1][1].append(i)
        else:
            out.append((w, [i]))
    return out


def _run_task(execute: Callable, payload) -> dict:
    """Run one payload; a failure becomes the lease's error and leaves the agent alive."""
    t0 = time.perf_counter()
    try:
        result = execute(payload)
    except Exception as exc:  # noqa: BLE001 - any task failure belongs to its lease
        return {"ok": False, "error": f"{type(exc).__name__}: {exc}"}
    batch = payload.get("batch") if isinstance(payload, dict) else None
    return {"ok": True, "result": result, "metrics": {"duration_ms": (time.perf_counter() - t0) * 1e3,
                                                      "batch_size": len(batch) if isinstance(batch, list) else 1}}


class LocalAgent:
    """A pull agent in the broker's own process: takes tickets from the queue without TCP."""

    def __init__(self, broker: HiveBroker, worker_id, *, caps, models, execute: Callable):
        self.broker = broker
        self.info = WorkerInfo(str(worker_id), frozenset(map(str, caps)), frozenset(map(str, models)), time.time())
        self.execute = execute
        self.completed = 0
        self._stop = threading.Event()

    def stop(self) -> None:
        self._stop.set()

    def run(self) -> None:
        self.broker._join(self.info)
        try:
            while not self._stop.is_set() and not self.broker._stopping.is_set():
                t = self.broker._lease(self.info)
                if t is None:
                    continue
                self.broker._settle(t, self.info.worker_id, _run_task(self.execute, t.tile.payload))
                self.completed += 1
        finally:
            self.broker._leave(self.info.worker_id)


class HiveAgent:
    """A persistent pull agent over TCP; `execute(payload) -> result` owns the local model (one
    agent per GPU here)."""

    def __init__(self, host, port, worker_id, *, caps, models, execute: Callable, authkey=None,
                 connect_timeout=10):
        self.host, self.port = host, int(port)
        self.worker_id = str(worker_id)
        self.caps = sorted(set(map(str, caps)))
        self.models = sorted(set(map(str, models)))
        self.execute = execute
        self.authkey = authkey.encode() if isinstance(authkey, str) else authkey
        self.connect_timeout = connect_timeout
        self.sock: Optional[socket.socket] = None
        self.completed = 0
        self._stop = threading.Event()

    def stop(self) -> None:
        self._stop.set()

    def _open(self) -> socket.socket:
        sock = socket.create_connection((self.host, self.port), timeout=self.connect_timeout)
        sock.settimeout(None)
        if self.authkey:
            challenge = recv_frame(sock)
            if challenge.kind != Message.AUTH_CHALLENGE:
                raise ValueError(f"the broker sent {challenge.kind.name}, not the authentication challenge")
            send_frame(sock, Frame(Message.AUTH, payload=_hmac(self.authkey, challenge.payload)))
        send_frame(sock, Frame(Message.HELLO, payload=json_payload(
            {"worker_id": self.worker_id, "caps": self.caps, "models": self.models})))
        if recv_frame(sock).kind != Message.READY:
            raise RuntimeError("the HIVE broker refused this agent's HELLO")
        return sock

    def _pull_once(self) -> bool:
        """One PULL and its answer: False once the broker says STOP."""
        send_frame(self.sock, Frame(Message.PULL))
        msg = recv_frame(self.sock)
        if msg.kind == Message.STOP:
            return False
        if msg.kind == Message.WAIT:
            return True
        if msg.kind == Message.ERROR:
            raise RuntimeError(parse_json(msg.payload).get("error", "the broker reported an error"))
        if msg.kind != Message.WORK:
            raise ValueError(f"the broker sent {msg.kind.name} in answer to PULL")
        reply = _run_task(self.execute, parse_json(msg.payload)["payload"])
        send_frame(self.sock, Frame(Message.RESULT, msg.request_id, msg.sequence, json_payload(reply)))
        self.completed += 1
        return True

    def run(self) -> None:
        self.sock = self._open()
        try:
            while not self._stop.is_set() and self._pull_once():
                pass
        except (OSError, ConnectionError):
            if not self._stop.is_set():
                raise
        finally:
            sock, self.sock = self.sock, None
            if sock is not None:
                sock.close()
