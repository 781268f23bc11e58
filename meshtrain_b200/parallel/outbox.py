"""Outbound side of the host pipeline.

The compute thread hands each outgoing tensor to ``Outbox.submit_tensor``,
which only starts the device-to-host copy (the ordering point against later
kernels) and queues a *letter*: a record that knows how to turn itself into a
packet once the copy is done.  Each link has one ``Courier`` thread that takes
letters in FIFO order, finishes the copy, serialises without copying and
sends.  With ``async_mode=False`` the compute thread delivers the letter
itself.

Semantics (reference runtime/outbox.py:53-185): FIFO per link; a courier's
queue holds at most ``max_queue`` letters and a submit that cannot enqueue
within ``timeout_s`` raises ``OutboxError`` (back-pressure from a peer that
stopped draining); a failed send is re-raised on the next submit or flush and
reported on the events queue; ``notify=True`` posts ``("send_done", link,
step, mb)`` after delivery.  Spans: QUEUE_WAIT, D2H_COPY, SERIALIZE and
NETWORK_SEND on the stage's timeline.
"""

from __future__ import annotations

import threading
import time
from collections import deque
from dataclasses import dataclass, field
from typing import Callable

from meshtrain_b200.networking.packet import DTYPE_NAMES, MessageType, TensorPacket
from meshtrain_b200.networking.serialization import tensor_to_bytes
from meshtrain_b200.utils.timeline import Timeline


class OutboxError(RuntimeError):
    pass


@dataclass
class Letter:
    """One outgoing message: a ready packet, or a pending copy plus its header fields."""

    link: str
    queued_at: float
    notify: bool = False
    packet: TensorPacket | None = None
    finish_copy: Callable | None = None   # -> (host tensor, release callback or None)
    fields: dict = field(default_factory=dict)

    @property
    def step(self):
        return self.fields.get("step_id") if self.packet is None else self.packet.step_id

    @property
    def microbatch(self):
        return self.fields.get("microbatch_id") if self.packet is None else self.packet.microbatch_id


class Courier:
    """The sender thread of one link, with its bounded FIFO of letters."""

    def __init__(self, name: str, deliver: Callable[[Letter], None], capacity: int, on_error: Callable):
        self.name = name
        self.capacity = max(1, capacity)
        self._deliver = deliver
        self._on_error = on_error
        self._letters: deque[Letter] = deque()
        self._cv = threading.Condition()
        self._busy = False
        self._closing = False
        self.peak = 0
        self.dead = False
        self.thread = threading.Thread(target=self._run, daemon=True, name=f"send-{name}")
        self.thread.start()

    def post(self, letter: Letter, timeout: float) -> None:
        with self._cv:
            if not self._cv.wait_for(lambda: len(self._letters) < self.capacity or self.dead, timeout):
                raise OutboxError(f"outbound queue to {self.name} stayed full for {timeout}s (peer not draining)")
            self._letters.append(letter)
            self.peak = max(self.peak, len(self._letters))
            self._cv.notify_all()

    def depth(self) -> int:
        with self._cv:
            return len(self._letters)

    def wait_idle(self, deadline: float) -> bool:
        with self._cv:
            return self._cv.wait_for(lambda: self.dead or (not self._letters and not self._busy),
                                     max(0.0, deadline - time.monotonic()))

    def _run(self) -> None:
        while True:
            with self._cv:
                self._cv.wait_for(lambda: self._letters or self._closing)
                if not self._letters:
                    return
                letter = self._letters.popleft()
                self._busy = True
                self._cv.notify_all()
            try:
                self._deliver(letter)
            except BaseException as exc:  # noqa: BLE001 - handed to the stage loop
                with self._cv:
                    self.dead = True
                    self._busy = False
                    self._letters.clear()
                    self._cv.notify_all()
                self._on_error(self.name, exc)
                return
            with self._cv:
                self._busy = False
                self._cv.notify_all()

    def close(self, join_s: float = 2.0) -> None:
        with self._cv:
            self._closing = True
            self._cv.notify_all()
        # a courier stuck on a dead socket is a daemon thread: it ends when the link closes
        self.thread.join(timeout=join_s)


class Outbox:
    def __init__(self, links: dict, timeline: Timeline, *, async_mode: bool, max_queue: int = 16,
                 timeout_s: float = 60.0, events=None, compression: str | None = None):
        from meshtrain_b200.networking.compression import policy

        self.compression = policy(compression)  # fp32 boundary tensors as 16-bit floats on the wire
        self.links = links
        self.timeline = timeline
        self.async_mode = async_mode
        self.timeout_s = timeout_s
        self.events = events
        self.bytes_sent = dict.fromkeys(links, 0)
        self.sent_messages = 0
        self._failure: BaseException | None = None
        self._couriers = {name: Courier(name, self._deliver, max_queue, self._failed) for name in links} \
            if async_mode else {}

    # ------------------------------------------------------------ submit
    def submit_tensor(self, link: str, tensor, message_type: MessageType, *, device, step: int, microbatch: int,
                      notify: bool = False, **fields) -> None:
        self._check()
        with self.timeline.span("D2H_COPY", step, microbatch, phase="begin"):
            finish = device.begin_d2h(tensor)
        fields = dict(fields, message_type=message_type, step_id=step, microbatch_id=microbatch)
        self._post(Letter(link, self.timeline.now(), notify, finish_copy=finish, fields=fields))

    def submit_packet(self, link: str, packet: TensorPacket) -> None:
        self._check()
        self._post(Letter(link, self.timeline.now(), packet=packet))

    def _post(self, letter: Letter) -> None:
        if self.async_mode:
            self._couriers[letter.link].post(letter, self.timeout_s)
        else:
            self._deliver(letter)

    # ------------------------------------------------------------ delivery
    def _packet_of(self, letter: Letter):
        if letter.packet is not None:
            return letter.packet, None
        tl, step, mb = self.timeline, letter.step, letter.microbatch
        with tl.span("D2H_COPY", step, mb, phase="finish"):
            host, release = letter.finish_copy()
        with tl.span("SERIALIZE", step, mb):
            if self.compression is not None:
                host = self.compression.wire(host)
            payload = tensor_to_bytes(host, copy=False)
        header = dict(letter.fields)
        mtype = header.pop("message_type")
        return TensorPacket(mtype, shape=tuple(host.shape), dtype=DTYPE_NAMES[host.dtype], payload=payload,
                            **header), release

    def _deliver(self, letter: Letter) -> None:
        tl = self.timeline
        if self.async_mode:
            tl.add("QUEUE_WAIT", letter.queued_at, tl.now(), letter.step, letter.microbatch, link=letter.link)
        packet, release = self._packet_of(letter)
        link = self.links[letter.link]
        sent_before = link.bytes_sent
        try:
            with tl.span("NETWORK_SEND", packet.step_id, packet.microbatch_id, link=letter.link,
                         bytes=len(packet.payload)):
                link.send_packet(packet)
        finally:
            if release is not None:
                release()
        self.bytes_sent[letter.link] += link.bytes_sent - sent_before
        self.sent_messages += 1
        if letter.notify and self.events is not None:
            self.events.put(("send_done", letter.link, packet.step_id, packet.microbatch_id))

    def _failed(self, link: str, exc: BaseException) -> None:
        if self._failure is None:
            self._failure = exc
        if self.events is not None:
            self.events.put(("send_error", link, exc))

    def _check(self) -> None:
        exc = self._failure
        if exc is not None:
            raise OutboxError(f"send failed: {type(exc).__name__}: {exc}") from exc

    # ------------------------------------------------------------ state
    @property
    def peak_depth(self) -> dict[str, int]:
        return {name: c.peak for name, c in self._couriers.items()} or dict.fromkeys(self.links, 0)

    def pending(self) -> dict[str, int]:
        return {name: c.depth() for name, c in self._couriers.items()}

    def flush(self, timeout: float | None = None) -> None:
        """Waits until every queued letter is delivered (or a send failed)."""
        deadline = time.monotonic() + (self.timeout_s if timeout is None else timeout)
        drained = all(c.wait_idle(deadline) for c in self._couriers.values())
        self._check()
        if not drained:
            raise OutboxError(f"outbound queues not drained after {timeout}s: {self.pending()}")

    def close(self) -> None:
        for courier in self._couriers.values():
            courier.close()
