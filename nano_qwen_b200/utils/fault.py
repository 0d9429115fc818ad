"""Failure detection on the host: heartbeats, a step watchdog, the kernels'
error word, and host-side fault injection for tests.

The reference's only failure handling was the NCCL process-group timeout of 30
minutes (reference: distributed/comm.py:14, :33-35).  Here:

* ``HeartbeatMonitor``: each rank writes a timestamp into the c10d store
  between steps; ``check()`` raises ``PeerFailure`` naming every rank whose
  heartbeat is older than the timeout, so survivors learn of a dead or stuck
  peer before their next collective instead of blocking in it.
* ``StepWatchdog``: a host thread that calls a handler (default: log and raise
  in the main thread at the next ``check()``) when a step exceeds its budget.
* ``check_device_errors``: every spin-wait in this library's kernels is bounded
  (by ``%globaltimer``, with limits set at run time by ``set_wait_limits``); a
  wait that runs out records a code in a device error word and returns instead
  of hanging.  This reads the word and raises.
* ``FaultInjector``: ``NQ_FAULT="rank:step:kind"`` makes that rank raise
  (``raise``), exit (``exit``) or stop heart-beating (``silent``) at that step.
  Injection is host-only; nothing here faults or stalls a GPU.
"""

from __future__ import annotations

import os
import threading
import time
from typing import Callable, List, Optional


class PeerFailure(RuntimeError):
    def __init__(self, ranks: List[int], detail: str = ""):
        self.ranks = list(ranks)
        super().__init__(f"peer rank(s) {self.ranks} stopped responding{': ' + detail if detail else ''}")


class DeviceWaitTimeout(RuntimeError):
    pass


class HeartbeatMonitor:
    def __init__(self, store, rank: int, world: int, interval_s: float = 5.0,
                 timeout_s: float = 60.0, prefix: str = "nq_hb"):
        self.store = store
        self.rank = rank
        self.world = world
        self.interval_s = interval_s
        self.timeout_s = timeout_s
        self.prefix = prefix
        self._last_beat = 0.0
        self.silent = False

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self, force: bool = False) -> None:
        if self.silent:
            return
        now = time.time()
        if force or now - self._last_beat >= self.interval_s:
            self.store.set(self._key(self.rank), repr(now))
            self._last_beat = now

    def stale_ranks(self) -> List[int]:
        now = time.time()
        out = []
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                self.store.wait([self._key(r)], _td(0.05))
                ts = float(self.store.get(self._key(r)).decode())
            except Exception:
                out.append(r)  # never beat, or the store cannot be read
                continue
            if now - ts > self.timeout_s:
                out.append(r)
        return out

    def check(self) -> None:
        bad = self.stale_ranks()
        if bad:
            raise PeerFailure(bad, f"no heartbeat for > {self.timeout_s:.1f} s")

    def gate(self, step: int) -> None:
        """Step gate, called between steps before any collective of ``step``:
        announce this rank at ``step`` and wait (at most ``timeout_s``) until
        every peer has announced it too.  A rank that left, crashed or hangs
        in its previous step never announces, and the survivors get a
        ``PeerFailure`` naming it here, on the host, instead of blocking in
        their next collective or peer-memory wait."""
        if not self.silent:
            self.store.set(f"{self.prefix}/step/{step}/{self.rank}", "1")
            # every peer passed its gate of step - 2 before announcing step - 1,
            # which this rank saw at its previous gate: that key is no longer read
            if step >= 2:
                try:
                    self.store.delete_key(f"{self.prefix}/step/{step - 2}/{self.rank}")
                except Exception:
                    pass
        peers = [r for r in range(self.world) if r != self.rank]
        keys = [f"{self.prefix}/step/{step}/{r}" for r in peers]
        try:
            self.store.wait(keys, _td(self.timeout_s))
            return
        except Exception:
            pass
        try:
            missing = [r for r, k in zip(peers, keys) if not self.store.check([k])]
        except Exception as e:  # the store's host rank is gone too
            raise PeerFailure(peers, f"store unreachable at step {step}: {e}") from e
        if missing:
            raise PeerFailure(missing, f"did not reach step {step} within {self.timeout_s:.1f} s")


def _td(s: float):
    import datetime
    return datetime.timedelta(seconds=s)


class StepWatchdog:
    """``with wd.step(i): ...``; if the body takes longer than ``budget_s`` the
    handler runs on the watchdog thread (default: remember the overrun, and
    ``check()`` raises it on the main thread)."""

    def __init__(self, budget_s: float, handler: Optional[Callable[[int, float], None]] = None):
        self.budget_s = budget_s
        self.handler = handler
        self._deadline = None
        self._step = -1
        self._overrun: Optional[str] = None
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def _run(self):
        while not self._stop.wait(0.05):
            with self._lock:
                d, s = self._deadline, self._step
            if d is not None and time.time() > d:
                elapsed = self.budget_s + (time.time() - d)
                with self._lock:
                    self._deadline = None
                    self._overrun = f"step {s} exceeded {self.budget_s:.1f} s ({elapsed:.1f} s)"
                if self.handler is not None:
                    self.handler(s, elapsed)

    def step(self, i: int):
        wd = self

        class _Ctx:
            def __enter__(self_):
                with wd._lock:
                    wd._step = i
                    wd._deadline = time.time() + wd.budget_s

            def __exit__(self_, *a):
                with wd._lock:
                    wd._deadline = None
                return False

        return _Ctx()

    def check(self) -> None:
        with self._lock:
            msg, self._overrun = self._overrun, None
        if msg:
            raise TimeoutError(msg)

    def close(self):
        self._stop.set()
        self._thread.join(timeout=1.0)


# Codes written by the kernels (csrc/sm100.cuh, enum ErrCode).
_ERR_NAMES = {1: "TMA producer wait timed out", 2: "MMA issuer wait timed out",
              3: "epilogue wait timed out", 4: "drain of in-flight copies timed out",
              5: "softmax/compute wait timed out", 6: "peer flag wait timed out",
              7: "bad launch argument"}


def check_device_errors(clear: bool = True) -> None:
    """Raise if any kernel of this library recorded an error (bounded wait ran
    out, bad launch argument).  Synchronises with the device."""
    import torch
    if not torch.cuda.is_available():
        return
    from ..ops._ext import ext
    E = ext()
    code = int(E.error_flag_read())
    if code:
        if clear:
            E.error_flag_clear()
        raise DeviceWaitTimeout(f"device error word {code}: {_ERR_NAMES.get(code & 0xff, 'unknown')}")


def set_wait_limits(mbar_s: Optional[float] = None, peer_s: Optional[float] = None) -> None:
    """Change the bounded-wait limits of the current GPU's kernels (seconds;
    ``None`` keeps a value).  Defaults: 2 s for waits on a CTA's own pipeline
    (mbarriers), 20 s for flags written by another GPU.  A watchdog that wants
    a dead peer to surface sooner lowers the peer limit; the kernels read the
    values at run time, so no rebuild is needed."""
    from ..ops._ext import ext
    ext().wait_limits_set(int(mbar_s * 1e9) if mbar_s else 0, int(peer_s * 1e9) if peer_s else 0)


def get_wait_limits() -> tuple:
    """(mbarrier limit, peer-flag limit) of the current GPU, in seconds."""
    from ..ops._ext import ext
    m, p = ext().wait_limits_get()
    return m / 1e9, p / 1e9


class FaultInjector:
    """Host-side fault injection from ``NQ_FAULT="rank:step:kind"``."""

    def __init__(self, rank: int, spec: Optional[str] = None):
        self.rank = rank
        spec = spec if spec is not None else os.environ.get("NQ_FAULT", "")
        self.plan = None
        if spec:
            r, s, kind = spec.split(":")
            self.plan = (int(r), int(s), kind)

    def maybe_fail(self, step: int, heartbeat: Optional[HeartbeatMonitor] = None) -> None:
        if self.plan is None:
            return
        r, s, kind = self.plan
        if r != self.rank or step != s:
            return
        if kind == "raise":
            raise RuntimeError(f"injected fault on rank {r} at step {s}")
        if kind == "exit":
            os._exit(17)
        if kind == "silent" and heartbeat is not None:
            heartbeat.silent = True
