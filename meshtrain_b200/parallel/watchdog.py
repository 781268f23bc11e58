"""Failure detection for device-engine pipelines (NCCL between the stages of one box).

NCCL point-to-point calls have no notion of a dead peer: a stage whose
neighbour has gone waits in its next receive until the process group's
timeout.  ``PeerWatch`` turns a failure anywhere in the pipeline into an error
on every rank within about one polling interval, on the host, through the
job's c10d store (the TCPStore of the rendezvous):

* a rank whose step raises calls ``report(reason)``: it writes the reason
  under the job's ``failed`` key, so the whole pipeline learns of it;
* a background thread on every rank refreshes the rank's ``alive`` counter
  and polls the ``failed`` key and the peers' counters every ``poll_s``;
  ``beat(step)`` additionally records the last completed step;
* when it sees a failure, or a peer whose counter has not moved for
  ``timeout_s`` (a process that died without reporting), it records the
  reason;
* the training loop calls ``check()`` before it launches a step, and the
  engine polls the reason while it waits for the device (it never blocks
  inside CUDA on work that may wait for a dead peer): either raises
  ``PeerFailure``.  The trainer then leaves its process groups as they are
  (``abandon_groups``): NCCL work still queued toward the dead peer ends with
  the process.

This is the device-engine counterpart of the reference's ERROR packet to both
neighbours and its bounded waits (runtime/pipeline.py:270-283, 443-449); the
worker reports the resulting exception through the same stage_error ->
STOP_JOB path as a TCP stage.
"""

from __future__ import annotations

import datetime
import threading
import time

import torch.distributed as dist


class PeerFailure(RuntimeError):
    """Another rank of the pipeline failed or stopped making progress."""


_ABANDONED = False


def groups_abandoned() -> bool:
    """True once a failed trainer has aborted and left its process groups: code that
    tears down torch.distributed on its way out must not destroy them (destroying
    waits for NCCL work queued toward the dead peer, which never completes)."""
    return _ABANDONED


def default_store():
    from torch.distributed import distributed_c10d

    return distributed_c10d._get_default_store()


class PeerWatch:
    def __init__(self, rank: int, world: int, *, store=None, timeout_s: float = 60.0, poll_s: float = 0.2,
                 prefix: str = "meshtrain/watch", groups: list | None = None, start: bool = True):
        self.rank, self.world = rank, world
        self.store = store if store is not None else default_store()
        self.timeout_s = timeout_s
        self.poll_s = poll_s
        self.prefix = prefix
        self.groups = list(groups or [])
        self.reason: str | None = None
        self.aborted = False
        self._halt = threading.Event()
        self._last_seen: dict[int, tuple[str, float]] = {}
        self._pulse = 0
        self.beat(-1)
        self._alive()
        self._thread = threading.Thread(target=self._watch, daemon=True, name="peer-watch")
        if start:
            self._thread.start()

    # -- keys -------------------------------------------------------------------
    @property
    def _failed_key(self) -> str:
        return f"{self.prefix}/failed"

    def _beat_key(self, rank: int) -> str:
        return f"{self.prefix}/beat/{rank}"

    def _alive_key(self, rank: int) -> str:
        return f"{self.prefix}/alive/{rank}"

    def _alive(self) -> None:
        self._pulse += 1
        self.store.set(self._alive_key(self.rank), str(self._pulse))

    # -- main-thread calls ------------------------------------------------------
    def beat(self, step: int) -> None:
        """Marks this rank alive and done with ``step``."""
        self.store.set(self._beat_key(self.rank), f"{step}:{time.time():.3f}")

    def report(self, reason: str) -> None:
        """Tells every rank that this one failed (first report wins)."""
        message = f"rank {self.rank}: {reason}"[:500]
        try:
            if not self.store.check([self._failed_key]):
                self.store.set(self._failed_key, message)
        except Exception:  # noqa: BLE001 - the store may be gone with the rendezvous host
            pass
        self.reason = self.reason or message

    def check(self) -> None:
        """Raises PeerFailure if a failure has been seen (call before launching a step).

        Looks up only the job's ``failed`` key (one store round trip); the peers'
        liveness counters are the watcher thread's business."""
        if self.reason is None:
            self._poll_failed()
        if self.reason is not None:
            raise PeerFailure(self.reason)

    def _poll_failed(self) -> None:
        try:
            if self.store.check([self._failed_key]):
                reported = self.store.get(self._failed_key).decode()
                if not reported.startswith(f"rank {self.rank}:"):
                    self._trip(reported)
        except Exception as exc:  # noqa: BLE001 - the store host died: so did the rendezvous rank
            self._trip(f"store unreachable: {type(exc).__name__}: {exc}")

    def peer_failure(self, wait_s: float = 1.0) -> str | None:
        """After this rank's own step failed: the reason if another rank reported first.

        A peer that fails usually reports just before its links close, so an
        error here ("connection closed", an aborted NCCL call) is most often
        the consequence; this waits up to ``wait_s`` for that report.
        """
        give_up = time.monotonic() + wait_s
        while True:
            if self.reason is None:
                self._poll_once()
            if self.reason is not None and not self.reason.startswith(f"rank {self.rank}:"):
                return self.reason
            if time.monotonic() >= give_up:
                return None
            time.sleep(min(0.05, self.poll_s))

    def startup_gate(self, failure: str | None, timeout_s: float) -> None:
        """Agreement through the store, before any rank launches a collective or a send/receive.

        Every rank posts ``ok`` or its startup failure (a failed allocation, a failed memory
        check).  A rank that failed returns at once and raises its own error; the others
        wait (at most ``timeout_s``) for every rank's word and raise ``PeerFailure`` if any
        rank failed or never arrived.  No NCCL work is in flight on either side then, so
        every rank can tear its process groups down normally and the worker can join the
        next placement attempt (startup-OOM replanning) in the same process.
        """
        ready = [f"{self.prefix}/ready/{r}" for r in range(self.world)]
        self.store.set(ready[self.rank], "ok" if failure is None else f"failed: {failure}"[:500])
        if failure is not None:
            return
        try:
            self.store.wait(ready, datetime.timedelta(seconds=timeout_s))
        except Exception as exc:  # noqa: BLE001 - a store timeout or a vanished store host
            raise PeerFailure(f"not every rank reached the startup gate within {timeout_s:.0f}s "
                              f"({type(exc).__name__})") from exc
        for r, key in enumerate(ready):
            word = self.store.get(key).decode()
            if word != "ok":
                raise PeerFailure(f"rank {r} {word}")

    def add_groups(self, groups) -> None:
        self.groups.extend(groups)

    # -- background ---------------------------------------------------------------
    def _poll_once(self) -> None:
        try:
            if self.store.check([self._failed_key]):
                reported = self.store.get(self._failed_key).decode()
                if not reported.startswith(f"rank {self.rank}:"):
                    self._trip(reported)
                return
            now = time.monotonic()
            for peer in range(self.world):
                if peer == self.rank:
                    continue
                key = self._alive_key(peer)
                pulse = self.store.get(key).decode() if self.store.check([key]) else "absent"
                seen = self._last_seen.get(peer)
                if seen is None or seen[0] != pulse:
                    self._last_seen[peer] = (pulse, now)
                elif now - seen[1] > self.timeout_s:
                    done = self.store.get(self._beat_key(peer)).decode() if self.store.check(
                        [self._beat_key(peer)]) else "none"
                    self._trip(f"rank {peer} stopped responding for {self.timeout_s:.0f}s "
                               f"(last completed step {done.split(':')[0]})")
                    return
        except Exception as exc:  # noqa: BLE001 - the store host died: so did the rendezvous rank
            self._trip(f"store unreachable: {type(exc).__name__}: {exc}")

    def _trip(self, reason: str) -> None:
        # Only records the reason: the trainer polls it while it waits on the device
        # (``PipelineEngine.wait_event``) and before each step, raises PeerFailure on
        # its own thread and aborts the communicators on its way out (``close``).
        if self.reason is None:
            self.reason = reason

    def abandon_groups(self) -> None:
        """Marks this process's groups as left behind after a failure: nothing destroys
        or aborts them.  NCCL work still queued toward the dead peer ends with the
        process (or with the process group's own timeout).  Aborting the
        communicators from the process was measured to block with sends and
        receives in flight on several communicators, and a blocked abort holds up
        the failure report."""
        global _ABANDONED
        _ABANDONED = True

    def abort_communicators(self, wait_s: float = 2.0) -> None:
        """Aborts this rank's communicators (best effort) so in-flight NCCL work ends.

        The aborts run on a daemon thread, joined for at most ``wait_s``: an abort
        that blocks (NCCL work in flight on several communicators) must not stop
        the caller, which reports the failure and leaves without waiting for the
        device.  Gloo groups cannot abort; their calls end by timeout.
        """
        global _ABANDONED
        if self.aborted:
            return
        self.aborted = True
        _ABANDONED = True
        targets = list(self.groups)
        if dist.is_initialized():
            targets.append(dist.group.WORLD)

        def run():
            for group in targets:
                try:
                    group.abort()
                except Exception:  # noqa: BLE001 - gloo groups, or already torn down
                    pass

        worker = threading.Thread(target=run, daemon=True, name="peer-watch-abort")
        worker.start()
        worker.join(timeout=wait_s)

    def _watch(self) -> None:
        while not self._halt.wait(self.poll_s):
            if self.reason is not None:
                return
            try:
                self._alive()
            except Exception:  # noqa: BLE001 - reported by the poll below
                pass
            self._poll_once()

    def close(self) -> None:
        self._halt.set()
        if self._thread.is_alive():
            self._thread.join(timeout=2 * self.poll_s + 1)
