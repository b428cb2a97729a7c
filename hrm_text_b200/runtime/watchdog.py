"""Host-side failure detection: a per-step deadline watchdog and a store-based heartbeat.

The reference has neither (it relies on NCCL's default timeout and manual restarts). Here:

* ``StepWatchdog`` arms a deadline around each training step; if the step does not finish in
  time it calls ``on_timeout`` (default: log every thread's stack and interrupt the main
  thread with ``KeyboardInterrupt``), so a rank stuck in a collective or a device wait is
  reported instead of hanging silently.
* ``Heartbeat`` lets every rank publish ``(step, wall time)`` into the process group's
  key-value store from a background thread; ``stale_ranks`` tells any rank which peers have
  stopped beating, before it launches its next collective.

Device-side waits are bounded by the kernels themselves (they record an error word and
return); ``hrm_text_b200.utils.errors.check_device_errors`` surfaces those.
"""
from __future__ import annotations

import _thread
import faulthandler
import sys
import threading
import time
from typing import Callable, Optional


def _default_on_timeout(step: int, elapsed: float) -> None:
    print(f"[watchdog] step {step} exceeded its deadline ({elapsed:.1f} s); thread stacks:", file=sys.stderr,
          flush=True)
    faulthandler.dump_traceback(file=sys.stderr, all_threads=True)
    _thread.interrupt_main()


class StepWatchdog:
    """``with watchdog.step(i): ...`` — calls ``on_timeout(i, elapsed)`` once if the body runs
    longer than ``deadline_s``."""

    def __init__(self, deadline_s: float, on_timeout: Optional[Callable[[int, float], None]] = None,
                 poll_s: float = 0.05):
        self.deadline_s = float(deadline_s)
        self.on_timeout = on_timeout or _default_on_timeout
        self.poll_s = poll_s
        self._lock = threading.Lock()
        self._armed: Optional[tuple[int, float]] = None
        self._fired = False
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, name="hrm-step-watchdog", daemon=True)
        self._thread.start()
        self.timeouts = 0

    def _run(self) -> None:
        while not self._stop.wait(self.poll_s):
            with self._lock:
                armed, fired = self._armed, self._fired
            if armed is None or fired:
                continue
            step, t0 = armed
            elapsed = time.monotonic() - t0
            if elapsed > self.deadline_s:
                with self._lock:
                    self._fired = True
                self.timeouts += 1
                self.on_timeout(step, elapsed)

    def arm(self, step: int) -> None:
        with self._lock:
            self._armed = (step, time.monotonic())
            self._fired = False

    def disarm(self) -> None:
        with self._lock:
            self._armed = None

    def step(self, step: int):
        wd = self

        class _Ctx:
            def __enter__(self):
                wd.arm(step)
                return wd

            def __exit__(self, *exc):
                wd.disarm()
                return False

        return _Ctx()

    def close(self) -> None:
        self._stop.set()
        self._thread.join(timeout=1.0)


class Heartbeat:
    """Per-rank liveness through a ``torch.distributed`` store (``TCPStore`` / ``FileStore``).

    Each rank's background thread writes ``hb/<rank> = "<step> <unix time>"`` every
    ``interval_s``; ``stale_ranks(max_age_s)`` lists peers whose last beat is older than that
    (or missing)."""

    def __init__(self, store, rank: int, world: int, interval_s: float = 1.0, prefix: str = "hb"):
        self.store, self.rank, self.world = store, rank, world
        self.interval_s, self.prefix = interval_s, prefix
        self.step = 0
        self._stop = threading.Event()
        self._beat()
        self._thread = threading.Thread(target=self._run, name="hrm-heartbeat", daemon=True)
        self._thread.start()

    def _beat(self) -> None:
        self.store.set(f"{self.prefix}/{self.rank}", f"{self.step} {time.time():.3f}")

    def _run(self) -> None:
        while not self._stop.wait(self.interval_s):
            try:
                self._beat()
            except Exception:  # the store went away: the job is ending
                return

    def set_step(self, step: int) -> None:
        self.step = step

    def last_beat(self, rank: int) -> Optional[tuple[int, float]]:
        key = f"{self.prefix}/{rank}"
        try:
            if not self.store.check([key]):
                return None
            step, t = self.store.get(key).decode().split()
            return int(step), float(t)
        except Exception:
            return None

    def stale_ranks(self, max_age_s: float) -> list[int]:
        now = time.time()
        out = []
        for r in range(self.world):
            if r == self.rank:
                continue
            beat = self.last_beat(r)
            if beat is None or now - beat[1] > max_age_s:
                out.append(r)
        return out

    def stop(self) -> None:
        self._stop.set()
        self._thread.join(timeout=2.0)
