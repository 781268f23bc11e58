"""Outbound path of the host pipeline: staging, serialisation and (async) sends.

    compute thread: submit -> device.begin_d2h (ordering point) -> bounded FIFO per link
    sender thread : finish D2H -> zero-copy serialise -> send -> send_done / send_error event

FIFO per link; bounded queues give back-pressure; a queue that stays full for
``timeout_s`` raises ``OutboxError``; ``async_mode=False`` sends on the
compute thread (reference runtime/outbox.py:53-185).
"""

from __future__ import annotations

import queue
import threading
from dataclasses import dataclass, field
from typing import Callable

from meshtrain_b200.networking.packet import DTYPE_NAMES, MessageType, TensorPacket
from meshtrain_b200.networking.serialization import tensor_to_bytes
from meshtrain_b200.networking.transport import Transport
from meshtrain_b200.utils.timeline import Timeline

_STOP = object()


class OutboxError(RuntimeError):
    pass


@dataclass
class _Item:
    link: str
    packet: TensorPacket | None
    finish: Callable | None
    submitted: float
    notify: bool
    fields: dict = field(default_factory=dict)


class Outbox:
    def __init__(self, links: dict[str, Transport], timeline: Timeline, *, async_mode: bool, max_queue: int = 16,
                 timeout_s: float = 60.0, events: "queue.Queue | None" = None):
        self.links = links
        self.timeline = timeline
        self.async_mode = async_mode
        self.timeout_s = timeout_s
        self.events = events
        self.bytes_sent = {n: 0 for n in links}
        self.peak_depth = {n: 0 for n in links}
        self.sent_messages = 0
        self._queues: dict[str, queue.Queue] = {}
        self._threads: list[threading.Thread] = []
        self._error: BaseException | None = None
        if async_mode:
            for name in links:
                q: queue.Queue = queue.Queue(maxsize=max(1, max_queue))
                self._queues[name] = q
                t = threading.Thread(target=self._sender, args=(name, q), daemon=True, name=f"send-{name}")
                t.start()
                self._threads.append(t)

    def submit_tensor(self, link: str, tensor, message_type: MessageType, *, device, step: int, microbatch: int,
                      notify: bool = False, **fields) -> None:
        self._raise_if_failed()
        with self.timeline.span("D2H_COPY", step, microbatch, phase="begin"):
            finish = device.begin_d2h(tensor)
        fields.update(message_type=message_type, step_id=step, microbatch_id=microbatch)
        self._enqueue(_Item(link, None, finish, self.timeline.now(), notify, fields))

    def submit_packet(self, link: str, packet: TensorPacket) -> None:
        self._raise_if_failed()
        self._enqueue(_Item(link, packet, None, self.timeline.now(), False))

    def _enqueue(self, item: _Item) -> None:
        if not self.async_mode:
            self._send(item)
            return
        q = self._queues[item.link]
        try:
            q.put(item, timeout=self.timeout_s)
        except queue.Full:
            raise OutboxError(f"outbound queue to {item.link} stayed full for {self.timeout_s}s "
                              "(peer not draining)") from None
        self.peak_depth[item.link] = max(self.peak_depth[item.link], q.qsize())

    def _send(self, item: _Item) -> None:
        tl = self.timeline
        f = item.fields
        step = f.get("step_id", item.packet.step_id if item.packet else None)
        mb = f.get("microbatch_id", item.packet.microbatch_id if item.packet else None)
        start = tl.now()
        if self.async_mode:
            tl.add("QUEUE_WAIT", item.submitted, start, step, mb, link=item.link)
        release = None
        if item.packet is not None:
            packet = item.packet
        else:
            with tl.span("D2H_COPY", step, mb, phase="finish"):
                cpu, release = item.finish()
            with tl.span("SERIALIZE", step, mb):
                payload = tensor_to_bytes(cpu, copy=False)
            f = dict(f)
            mtype = f.pop("message_type")
            packet = TensorPacket(mtype, shape=tuple(cpu.shape), dtype=DTYPE_NAMES[cpu.dtype], payload=payload, **f)
        link = self.links[item.link]
        before = link.bytes_sent
        try:
            with tl.span("NETWORK_SEND", step, mb, link=item.link, bytes=len(packet.payload)):
                link.send_packet(packet)
        finally:
            if release is not None:
                release()
        self.bytes_sent[item.link] += link.bytes_sent - before
        self.sent_messages += 1
        if item.notify and self.events is not None:
            self.events.put(("send_done", item.link, packet.step_id, packet.microbatch_id))

    def _sender(self, name: str, q: queue.Queue) -> None:
        while True:
            item = q.get()
            if item is _STOP:
                q.task_done()
                return
            try:
                self._send(item)
            except BaseException as exc:  # noqa: BLE001 - surfaced to the executor
                self._error = exc
                if self.events is not None:
                    self.events.put(("send_error", name, exc))
                q.task_done()
                return
            q.task_done()

    def _raise_if_failed(self) -> None:
        if self._error is not None:
            raise OutboxError(f"send failed: {type(self._error).__name__}: {self._error}") from self._error

    def pending(self) -> dict[str, int]:
        return {n: q.qsize() for n, q in self._queues.items()}

    def flush(self, timeout: float | None = None) -> None:
        if not self.async_mode:
            return
        timeout = self.timeout_s if timeout is None else timeout
        done = threading.Event()

        def waiter():
            for q in self._queues.values():
                q.join()
            done.set()

        threading.Thread(target=waiter, daemon=True).start()
        if not done.wait(timeout):
            self._raise_if_failed()
            raise OutboxError(f"outbound queues not drained after {timeout}s: {self.pending()}")
        self._raise_if_failed()

    def close(self) -> None:
        for q in self._queues.values():
            try:
                q.put_nowait(_STOP)
            except queue.Full:
                pass  # sender stuck on a dead socket: daemon thread, exits when the link closes
        for t in self._threads:
            t.join(timeout=2.0)
