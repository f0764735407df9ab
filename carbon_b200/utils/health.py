"""Host-side failure detection: peer heartbeats through the rendezvous store and a step watchdog.

The reference has no recovery machinery; it bounds its waits (60 s symmetric-memory signal timeouts,
``rehome_transport.py:18``, ``dec/row_balance.py:23``) and runs a watchdog thread around launches that might hang
(``dec/prenorm_pair.py:41,425-437``).  Here every device wait is already bounded (the barrier kernel records a status
code and returns); the two classes below cover the host side:

* ``Heartbeat``: every rank bumps a counter under ``<prefix><rank>`` in the c10d store from a daemon thread.  Between
  steps, before the next launch, ``check()`` raises ``PeerFailure`` for a peer whose counter has not moved for
  ``max_age`` seconds (measured on this rank's monotonic clock, so host clocks need not agree), for a peer that
  announced it left, and when the store itself is unreachable (its host rank is gone).  A rank that dies therefore
  stops the others before they enter a collective that would wait for it.
* ``Watchdog``: ``with wd.step("decode"):`` arms a timer; a step that overruns it raises ``StepStalled`` in the main
  thread (the timer interrupts it) or, for steps run on another thread, when the step returns.  All threads' stacks
  are written to stderr when it fires.
"""
from __future__ import annotations

import faulthandler
import signal
import sys
import threading
import time
from contextlib import contextmanager
from typing import Dict, Optional

_LEFT = b"left"


class PeerFailure(RuntimeError):
    def __init__(self, rank: int, reason: str):
        super().__init__(f"rank {rank}: {reason}")
        self.rank = rank
        self.reason = reason


class StepStalled(RuntimeError):
    pass


class Heartbeat:
    def __init__(self, store, rank: int, world: int, interval: float = 0.5, max_age: float = 10.0,
                 prefix: str = "carbon/hb/"):
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.max_age, self.prefix = interval, max_age, prefix
        self._count = 0
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._seen: Dict[int, tuple] = {}        # peer -> (last value, monotonic time it last changed)

    def _key(self, r: int) -> str:
        return f"{self.prefix}{r}"

    def beat(self) -> None:
        with self._lock:
            self._count += 1
            self.store.set(self._key(self.rank), str(self._count))

    def _loop(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self.beat()
            except Exception:                     # store gone: the peers' check() reports it on their side
                return

    def start(self) -> "Heartbeat":
        self.beat()
        now = time.monotonic()
        self._seen = {r: (None, now) for r in range(self.world) if r != self.rank}
        self._thread = threading.Thread(target=self._loop, name=f"carbon-heartbeat-{self.rank}", daemon=True)
        self._thread.start()
        return self

    def check(self) -> None:
        """Raise ``PeerFailure`` if any peer left, went silent for ``max_age`` seconds, or the store is gone."""
        now = time.monotonic()
        for r, (last, t) in self._seen.items():
            try:
                with self._lock:
                    present = self.store.check([self._key(r)])
                    val = self.store.get(self._key(r)) if present else None
            except Exception as e:
                raise PeerFailure(r, f"store unreachable ({type(e).__name__})") from e
            if val == _LEFT:
                raise PeerFailure(r, "left the job")
            if val != last:
                self._seen[r] = (val, now)
            elif now - t > self.max_age:
                what = "never joined" if last is None else "heartbeat silent"
                raise PeerFailure(r, f"{what} for {now - t:.1f} s")

    def leave(self) -> None:
        """Announce a clean exit: the peers' next ``check()`` fails at once instead of after ``max_age``."""
        self.stop()
        with self._lock:
            self.store.set(self._key(self.rank), _LEFT.decode())

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5 * self.interval + 1)
            self._thread = None


class _Stall(BaseException):
    pass


_ACTIVE: Dict[str, bool] = {}          # the main thread's armed step: {"armed", "fired"}
_HANDLER = {"installed": False, "usable": False}


def _on_signal(signum, frame):
    st = _ACTIVE.get("step")
    if st is not None and st["armed"] and st["fired"]:
        st["armed"] = False                  # deliver once
        raise _Stall()


def _install_handler() -> bool:
    """SIGUSR1 interrupts a main thread that is blocked in a system call (a wait, a sleep, a socket read).  Installed
    once, only where nothing else handles SIGUSR1; a stray or late signal is ignored."""
    if not _HANDLER["installed"]:
        _HANDLER["installed"] = True
        if signal.getsignal(signal.SIGUSR1) in (signal.SIG_DFL, None):
            signal.signal(signal.SIGUSR1, _on_signal)
            _HANDLER["usable"] = True
    return _HANDLER["usable"]


class Watchdog:
    def __init__(self, timeout: float, dump_stacks: bool = True):
        self.timeout = timeout
        self.dump_stacks = dump_stacks
        self.stalls = 0

    @contextmanager
    def step(self, name: str = "step"):
        main = threading.current_thread() is threading.main_thread()
        interrupt = main and _install_handler()
        st = {"armed": True, "fired": False}
        done = threading.Event()
        if interrupt:
            _ACTIVE["step"] = st
        main_id = threading.main_thread().ident

        def fire():
            if done.wait(self.timeout) or not st["armed"]:
                return
            st["fired"] = True
            if self.dump_stacks:
                faulthandler.dump_traceback(file=sys.stderr, all_threads=True)
            if interrupt:
                signal.pthread_kill(main_id, signal.SIGUSR1)

        threading.Thread(target=fire, name="carbon-watchdog", daemon=True).start()
        try:
            yield
        except _Stall:
            self.stalls += 1
            raise StepStalled(f"{name} did not finish within {self.timeout} s") from None
        finally:
            st["armed"] = False
            done.set()
            if interrupt:
                _ACTIVE.pop("step", None)
        if st["fired"]:                      # overran, but was not interrupted (another thread, or at the limit)
            self.stalls += 1
            raise StepStalled(f"{name} did not finish within {self.timeout} s")
