"""Host runtime: one stage driven by its schedule over packet links.

``run_stage`` is the entry point (same contract as the reference's executor,
runtime/pipeline.py:157-461).  A ``StageRunner`` owns the stage's step loop:

* **Inbound.** One ``LinkReader`` thread per link receives packets (straight
  into pooled host buffers when it can), deserialises them and pushes them on
  one bounded queue; a full queue stops the readers, which stops TCP reads, so
  a slow stage throttles its neighbours.
* **Mailbox.** Accepted activations, gradients and targets of the current step
  wait in the ``Mailbox`` until the schedule reaches them; packets of the next
  step are held for it; any other step, a foreign job id, or a packet on the
  wrong link is a protocol error.  Host-to-device copies start on arrival.
* **Schedule.** The ``StepLedger`` (parallel/schedule.py) gives the next
  action and says when its inputs are present; the runner pumps the inbound
  queue until they are, for at most ``timeout_s`` without progress, then
  fails with a JSON dump of its state (PIPELINE_STALLED).
* **Outbound.** Forward outputs, input gradients (carrying the microbatch loss
  in ``meta``) and, on stage 0, the targets leave through the ``Outbox``;
  middle stages relay targets unchanged.
* **Step end.** One optimizer step per global step; a ``STEP_COMPLETE`` record
  with the timeline's compute / communication / overlap / idle split.
* **Failure.** Any error sends an ERROR packet to both neighbours, so the
  whole pipeline stops within milliseconds instead of timing out.
"""

from __future__ import annotations

import json
import queue
import threading
import time
from dataclasses import dataclass, field
from typing import Callable

import torch

from meshtrain_b200.networking.packet import MessageType, TensorPacket
from meshtrain_b200.networking.serialization import bytes_to_tensor
from meshtrain_b200.networking.transport import TransportClosed, TransportTimeout
from meshtrain_b200.parallel.autograd import BoundaryError, MicrobatchGraph
from meshtrain_b200.parallel.outbox import Outbox, OutboxError
from meshtrain_b200.parallel.schedule import Action, ActionKind, StepLedger
from meshtrain_b200.parallel.stage import Stage
from meshtrain_b200.telemetry import EventLogger
from meshtrain_b200.utils.timeline import Timeline

UPSTREAM = "upstream"
DOWNSTREAM = "downstream"


class PipelineError(RuntimeError):
    pass


@dataclass
class PipelineSettings:
    job_id: str
    steps: int
    batch_size: int
    num_microbatches: int = 1
    timeout_s: float = 60.0
    log_every: int = 10
    capture_gradients_at_step: int | None = None
    step_offset: int = 0
    log_microbatch_events: bool = False
    schedule: str = "gpipe"
    max_inflight_microbatches: int | None = None
    async_transport: bool = False
    max_outbound_queue: int | None = None
    trace: bool = True
    pinned_memory: bool = True
    buffer_pool: bool = True
    correctness_probe_steps: int = 0
    wire_compression: str | None = None  # "bf16" / "fp16": fp32 boundary tensors cross as 16-bit floats


@dataclass
class StageResult:
    stage_index: int
    worker: str
    losses: list[float] = field(default_factory=list)
    step_metrics: list[dict] = field(default_factory=list)
    gradients: dict[str, torch.Tensor] | None = None
    initial_params: dict[str, torch.Tensor] | None = None
    final_params: dict[str, torch.Tensor] | None = None
    error: str | None = None
    timeline: list[dict] | None = None


class LinkReader:
    """Receive thread of one link; posts ("packet", link, packet, tensor) or ("error", link, exc)."""

    POLL_S = 0.2

    def __init__(self, name: str, link, out: queue.Queue, timeline: Timeline, stop: threading.Event):
        self.name, self.link, self.out, self.timeline, self.stop = name, link, out, timeline, stop
        self.peak = 0
        self.thread = threading.Thread(target=self._loop, daemon=True, name=f"recv-{name}")
        self.thread.start()

    def _post(self, item) -> bool:
        while not self.stop.is_set():
            try:
                self.out.put(item, timeout=self.POLL_S)
            except queue.Full:
                continue  # the runner is behind: stop reading until it drains
            self.peak = max(self.peak, self.out.qsize())
            return True
        return False

    def _loop(self) -> None:
        tl = self.timeline
        while not self.stop.is_set():
            try:
                packet = self.link.recv_packet(timeout=self.POLL_S)
            except TransportTimeout:
                continue
            except Exception as exc:  # noqa: BLE001 - peer closed, malformed frame, ...
                if not self.stop.is_set():
                    self._post(("error", self.name, exc))
                return
            end = tl.now()
            tl.add("NETWORK_RECV", end - self.link.last_frame_s, end, packet.step_id, packet.microbatch_id,
                   link=self.name, bytes=len(packet.payload))
            tensor = getattr(packet, "recv_buffer", None)
            if tensor is None and packet.has_tensor:
                with tl.span("DESERIALIZE", packet.step_id, packet.microbatch_id):
                    tensor = bytes_to_tensor(packet.payload, packet.dtype, packet.shape)
            if not self._post(("packet", self.name, packet, tensor)):
                return


@dataclass
class Arrival:
    """A received tensor whose host-to-device copy is under way."""

    handle: object
    token: object
    meta: dict = field(default_factory=dict)


class Mailbox:
    """Inputs that arrived for the current step, and early packets of the next one."""

    def __init__(self) -> None:
        self.step = -1
        self.activations: dict[int, Arrival] = {}
        self.gradients: dict[int, Arrival] = {}
        self.targets: dict[int, torch.Tensor] = {}
        self.early: dict[int, list] = {}
        self.tokens: dict[int, list] = {}

    def open(self, step: int) -> list:
        """Starts ``step``; returns the packets that arrived for it ahead of time."""
        self.step = step
        self.activations.clear()
        self.gradients.clear()
        self.targets.clear()
        self.tokens.clear()
        return self.early.pop(step, [])

    def hold(self, step: int, item) -> None:
        self.early.setdefault(step, []).append(item)

    def contents(self) -> dict:
        return {"activations": sorted(self.activations), "gradients": sorted(self.gradients),
                "targets": sorted(self.targets)}


class _HostTensor:
    """Staging for a tensor that is already in host memory (targets sent from stage 0)."""

    @staticmethod
    def begin_d2h(tensor):
        t = tensor.detach()
        return lambda: (t, None)


class StageRunner:
    def __init__(self, stage: Stage, spec, settings: PipelineSettings, upstream, downstream, *, worker: str,
                 logger: EventLogger | None, metrics_callback: Callable[[dict], None] | None,
                 stop_event: threading.Event | None, capture_params: bool, timeline: Timeline | None):
        if (upstream is None) != stage.is_first or (downstream is None) != stage.is_last:
            raise PipelineError("stage links do not match stage position")
        if settings.batch_size % settings.num_microbatches:
            raise PipelineError("batch_size must be divisible by num_microbatches")
        self.stage, self.spec, self.cfg, self.worker = stage, spec, settings, worker
        self.M = settings.num_microbatches
        self.log = logger or EventLogger(worker, settings.job_id)
        self.metrics_callback = metrics_callback
        self.stop_event = stop_event
        self.capture_params = capture_params
        self.links = {name: link for name, link in ((UPSTREAM, upstream), (DOWNSTREAM, downstream)) if link}
        self.tl = timeline or Timeline(worker, stage.stage_index)
        self.dev = stage.device
        self.events: queue.Queue = queue.Queue(maxsize=4 * self.M + 16)
        self._reader_stop = threading.Event()
        self.readers: list[LinkReader] = []
        self.outbox = Outbox(self.links, self.tl, async_mode=settings.async_transport,
                             max_queue=settings.max_outbound_queue or 2 * self.M + 4, timeout_s=settings.timeout_s,
                             events=self.events, compression=settings.wire_compression)
        # with link compression, received boundary tensors return to the stage's compute dtype
        params = list(stage.module.parameters())
        self.compute_dtype = params[0].dtype if params and settings.wire_compression not in (None, "none") else None
        self.mail = Mailbox()
        self.ledger: StepLedger | None = None
        self.bytes_received = 0
        self.result = StageResult(stage.stage_index, worker)

    # ------------------------------------------------------------------ setup
    def _start_io(self) -> None:
        self.dev.configure_transfers(pinned=self.cfg.pinned_memory, pool=self.cfg.buffer_pool)
        receivable = {int(MessageType.FORWARD_ACTIVATION), int(MessageType.BACKWARD_GRADIENT)}
        dev = self.dev

        def allocate(mtype, dtype, shape):
            return dev.recv_buffer(shape, dtype) if mtype in receivable else None

        for name, link in self.links.items():
            link.payload_allocator = allocate
            self.readers.append(LinkReader(name, link, self.events, self.tl, self._reader_stop))

    # ------------------------------------------------------------------ inbound
    def _h2d(self, tensor, step: int, mb: int, meta=None) -> Arrival:
        if self.dev.backend == "cpu":
            handle, token = self.dev.begin_h2d(tensor)
        else:
            with self.tl.span("H2D_COPY", step, mb, phase="begin"):
                handle, token = self.dev.begin_h2d(tensor)
        return Arrival(handle, token, dict(meta or {}))

    def _claim(self, arrival: Arrival, step: int, mb: int):
        self.mail.tokens.setdefault(mb, []).append(arrival.token)
        if self.dev.backend == "cpu":
            tensor = self.dev.finish_h2d(arrival.handle)
        else:
            with self.tl.span("H2D_COPY", step, mb, phase="finish"):
                tensor = self.dev.finish_h2d(arrival.handle)
        if self.compute_dtype is not None and tensor.is_floating_point() and tensor.dtype != self.compute_dtype:
            tensor = tensor.to(self.compute_dtype)  # a compressed link delivered 16-bit floats
        return tensor

    def _deliver(self, link: str, packet: TensorPacket, tensor) -> None:
        """Files a packet of the current step and tells the ledger what became ready."""
        mb, kind, mail, ledger = packet.microbatch_id, packet.message_type, self.mail, self.ledger
        needs_target = self.stage.is_last and not self.stage.is_first
        if link == UPSTREAM and kind == MessageType.TARGET:
            mail.targets[mb] = tensor
            if mb in mail.activations:
                ledger.input_arrived(mb)
        elif link == UPSTREAM and kind == MessageType.FORWARD_ACTIVATION:
            if mb in mail.activations:
                raise BoundaryError(f"duplicate activation for step {packet.step_id} microbatch {mb}")
            mail.activations[mb] = self._h2d(tensor, packet.step_id, mb)
            if not needs_target or mb in mail.targets:
                ledger.input_arrived(mb)
        elif link == DOWNSTREAM and kind == MessageType.BACKWARD_GRADIENT:
            mail.gradients[mb] = self._h2d(tensor, packet.step_id, mb, packet.meta)
            ledger.gradient_arrived(mb)
        else:
            raise BoundaryError(f"unexpected {kind.name} from {link}")

    def _accept(self, link: str, packet: TensorPacket, tensor) -> None:
        if packet.message_type == MessageType.ERROR:
            raise PipelineError(f"{link} peer reported error: {packet.meta.get('error')}")
        if packet.job_id != self.cfg.job_id:
            raise BoundaryError(f"packet for job {packet.job_id!r} received in job {self.cfg.job_id!r}")
        self.bytes_received += len(packet.payload)
        if packet.message_type == MessageType.TARGET and not self.stage.is_last:
            self.outbox.submit_packet(DOWNSTREAM, packet)  # targets travel on to the last stage unchanged
        elif packet.step_id == self.mail.step:
            self._deliver(link, packet, tensor)
        elif packet.step_id == self.mail.step + 1:
            self.mail.hold(packet.step_id, (link, packet, tensor))
        else:
            raise BoundaryError(f"packet for step {packet.step_id} while in step {self.mail.step}")

    def _pump(self, timeout: float) -> bool:
        """Handles one inbound event; False when none came within ``timeout``."""
        if self.stop_event is not None and self.stop_event.is_set():
            raise PipelineError("job stopped")
        try:
            event = self.events.get(timeout=timeout)
        except queue.Empty:
            return False
        tag = event[0]
        if tag == "packet":
            self._accept(*event[1:])
        elif tag == "send_done":
            _, _link, step_id, mb = event
            if step_id == self.mail.step:
                self.ledger.forward_sent(mb)
        elif tag == "send_error":
            _, name, exc = event
            raise PipelineError(f"send to {name} peer failed: {type(exc).__name__}: {exc}") from exc
        else:  # a reader failed
            _, name, exc = event
            if isinstance(exc, TransportClosed):
                raise PipelineError(f"{name} peer disconnected: {exc}") from exc
            raise PipelineError(f"{name} link failed: {exc}") from exc
        return True

    def _stalled(self, reason: str) -> PipelineError:
        dump = {"reason": reason, "worker": self.worker, "stage": self.stage.stage_index,
                "state": self.ledger.snapshot() if self.ledger else None, "mailbox": self.mail.contents(),
                "future_steps": {s: len(v) for s, v in self.mail.early.items()},
                "saved_contexts": [list(k) for k in self.stage.contexts.pending()],
                "pending_sends": self.outbox.pending(), "inbound_queue": self.events.qsize()}
        self.log.log("PIPELINE_STALLED", None, None, dump=json.dumps(dump))
        return PipelineError(f"{reason}; state: {json.dumps(dump)}")

    def _await(self, action: Action, step: int) -> None:
        if self.ledger.ready(action):
            return
        t0 = self.tl.now()
        limit = self.cfg.timeout_s
        last_progress = time.monotonic()
        while not self.ledger.ready(action):
            if self._pump(min(limit, 0.5)):
                last_progress = time.monotonic()
            elif time.monotonic() - last_progress > limit:
                raise self._stalled(f"pipeline stalled: no progress within network timeout {limit}s "
                                    f"waiting for {action}")
        span = "WAIT_FORWARD" if action.kind is ActionKind.FORWARD else "WAIT_BACKWARD"
        self.tl.add(span, t0, self.tl.now(), step, action.microbatch)

    # ------------------------------------------------------------------ actions
    def _forward(self, step: int, mb: int, batch) -> None:
        stage, mail, cfg = self.stage, self.mail, self.cfg
        if stage.is_first:
            inp = batch[0][mb]
            if not stage.is_last:
                self.outbox.submit_tensor(DOWNSTREAM, batch[1][mb], MessageType.TARGET, device=_HostTensor,
                                          step=step, microbatch=mb, job_id=cfg.job_id, source_worker=self.worker)
        else:
            inp = self._claim(mail.activations.pop(mb), step, mb)
        graph = MicrobatchGraph(step, mb)
        with self.tl.span("FORWARD_COMPUTE", step, mb):
            out = stage.forward(inp, graph)
        self.peak_saved = max(self.peak_saved, stage.contexts.held_bytes())
        self.peak_graphs = max(self.peak_graphs, len(stage.contexts))
        if not stage.is_last:
            self.outbox.submit_tensor(DOWNSTREAM, out.detach(), MessageType.FORWARD_ACTIVATION, device=self.dev,
                                      step=step, microbatch=mb, notify=True, job_id=cfg.job_id,
                                      source_worker=self.worker)
        if cfg.log_microbatch_events:
            self.log.log("FORWARD_COMPLETE", step, mb, output=out.numel() * out.element_size(),
                         compute_s=graph.timings["forward"])

    def _backward(self, step: int, mb: int, batch) -> float:
        stage, mail, cfg = self.stage, self.mail, self.cfg
        if stage.is_last:
            target = batch[1][mb] if stage.is_first else mail.targets.pop(mb)
            with self.tl.span("BACKWARD_COMPUTE", step, mb):
                loss, grad_in, graph = stage.loss_backward(target, (step, mb), loss_scale=1.0 / self.M)
            meta = {"loss": float(loss)}
        else:
            arrival = mail.gradients.pop(mb)
            grad = self._claim(arrival, step, mb)
            meta = arrival.meta
            with self.tl.span("BACKWARD_COMPUTE", step, mb):
                grad_in, graph = stage.backward(grad, (step, mb))
        for token in mail.tokens.pop(mb, []):  # received buffers of this microbatch may be reused
            self.dev.after_use(token)
        if not stage.is_first:
            self.outbox.submit_tensor(UPSTREAM, grad_in, MessageType.BACKWARD_GRADIENT, device=self.dev, step=step,
                                      microbatch=mb, job_id=cfg.job_id, source_worker=self.worker, meta=meta)
        if cfg.log_microbatch_events:
            self.log.log("BACKWARD_COMPLETE", step, mb, compute_s=graph.timings["backward"])
        return float(meta.get("loss", 0.0))

    # ------------------------------------------------------------------ steps
    def _step(self, local_step: int) -> None:
        stage, cfg, tl, dev = self.stage, self.cfg, self.tl, self.dev
        step = cfg.step_offset + local_step
        t_start = tl.now()
        if stage.is_first:
            dev.reset_peak_memory()
        self.ledger = ledger = StepLedger(stage.stage_index, stage.num_stages, self.M, step, cfg.schedule,
                                          cfg.max_inflight_microbatches)
        received0, sent0 = self.bytes_received, sum(self.outbox.bytes_sent.values())
        for item in self.mail.open(step):
            self._deliver(*item)
        batch = None
        if stage.is_first:
            x, y = self.spec.make_batch(step, cfg.batch_size)
            batch = (x.chunk(self.M), y.chunk(self.M))
        loss_sum = 0.0
        self.peak_saved = self.peak_graphs = 0
        while not ledger.done:
            action = ledger.next_action()
            self._await(action, step)
            ledger.run(action)
            if action.kind is ActionKind.FORWARD:
                self._forward(step, action.microbatch, batch)
            else:
                loss_sum += self._backward(step, action.microbatch, batch)
            ledger.finish(action)
        if not ledger.all_complete():
            raise self._stalled("schedule finished with incomplete microbatches")
        if cfg.capture_gradients_at_step == step:
            self.result.gradients = stage.named_gradients()
        probe = local_step < cfg.correctness_probe_steps
        probe_record = None
        if probe:
            probe_record = {"grad_norms": {n: float(p.grad.detach().float().norm())
                                           for n, p in stage.module.named_parameters() if p.grad is not None}}
            params_before = stage.named_parameters_cpu() if local_step == 0 else None
        stage.refresh_tensor_store()
        memory = stage.memory_report()
        memory.update(tensor_store=stage.tensor_store.bytes_by_role(), saved_activations_peak=self.peak_saved,
                      saved_microbatches_peak=self.peak_graphs)
        with tl.span("OPTIMIZER_STEP", step):
            opt_s = stage.optimizer_step()
        stage.zero_grad()
        if probe and params_before is not None:
            after = stage.named_parameters_cpu()
            probe_record["param_delta_norms"] = {n: float((after[n] - params_before[n]).float().norm())
                                                 for n in params_before}
        t_end = tl.now()
        record = self._step_record(step, t_start, t_end, opt_s, loss_sum / self.M, received0, sent0, memory)
        if probe_record is not None:
            record["correctness"] = probe_record
        self.result.step_metrics.append(record)
        if stage.is_first:
            self.result.losses.append(record["loss"])
        if self.metrics_callback is not None:
            self.metrics_callback(record)
        if not cfg.trace:
            tl.drop_before(t_end)
        if local_step % cfg.log_every == 0 or local_step == cfg.steps - 1:
            fields = {"step_s": record["step_s"], "compute_s": record["compute_s"], "comm_s": record["comm_s"],
                      "exposed_s": record["exposed_communication_s"], "idle_s": record["idle_s"],
                      "sent_bytes": record["bytes_sent"]}
            if stage.is_first:
                fields = {"loss": record["loss"], **fields}
            self.log.log("STEP_COMPLETE", step, None, **fields)

    def _step_record(self, step, t_start, t_end, opt_s, mean_loss, received0, sent0, memory) -> dict:
        cfg, dev, stage = self.cfg, self.dev, self.stage
        step_s = t_end - t_start
        m = self.tl.step_metrics(step, (t_start, t_end))
        phase = m["phase_s"]
        dm = dev.memory_stats()
        record = {
            "event": "STEP_COMPLETE", "job": cfg.job_id, "worker": self.worker, "stage": stage.stage_index,
            "backend": dev.backend, "step": step, "schedule": cfg.schedule, "async_transport": cfg.async_transport,
            "step_s": step_s, "forward_s": phase.get("FORWARD_COMPUTE", 0.0),
            "backward_s": phase.get("BACKWARD_COMPUTE", 0.0), "optimizer_s": opt_s, "compute_s": m["compute_s"],
            "comm_s": m["communication_s"], "communication_s": m["communication_s"],
            "overlapped_s": m["overlapped_s"], "exposed_communication_s": m["exposed_communication_s"],
            "overlap_ratio": m["overlap_ratio"], "idle_s": m["idle_s"],
            "wait_forward_s": phase.get("WAIT_FORWARD", 0.0), "wait_backward_s": phase.get("WAIT_BACKWARD", 0.0),
            "bytes_sent": sum(self.outbox.bytes_sent.values()) - sent0,
            "bytes_received": self.bytes_received - received0,
            "lifecycle": {k: v for k, v in phase.items() if not k.startswith("WAIT")},
            "outbound_queue_peak": max(self.outbox.peak_depth.values(), default=0),
            "inbound_queue_peak": max((r.peak for r in self.readers), default=0),
            "peak_inflight_microbatches": self.ledger.peak_inflight, "buffer_pool": dev.host_pool.stats(),
            "utilization": m["compute_s"] / step_s if step_s else 0.0,
            "memory": {**memory, "device_allocated": dm.get("allocated", 0),
                       "device_peak": dm.get("peak_allocated", 0), "device_total": dm.get("total", 0)},
        }
        if stage.is_first:
            record["loss"] = mean_loss
            record["samples_per_s"] = cfg.batch_size / step_s if step_s else 0.0
            seq = getattr(self.spec, "seq_len", None)
            if seq:
                record["tokens_per_s"] = cfg.batch_size * seq / step_s if step_s else 0.0
        return record

    def _tell_neighbours(self, error: str) -> None:
        for link in self.links.values():
            try:
                link.send_packet(TensorPacket(MessageType.ERROR, job_id=self.cfg.job_id, source_worker=self.worker,
                                              meta={"error": f"{self.worker}: {error}"[:200]}))
            except Exception:  # noqa: BLE001 - the neighbour may be gone already
                pass

    def run(self) -> StageResult:
        if self.capture_params:
            self.result.initial_params = self.stage.named_parameters_cpu()
        try:
            self._start_io()
            for local_step in range(self.cfg.steps):
                self._step(local_step)
            self.outbox.flush()
        except Exception as exc:
            self.result.error = f"{type(exc).__name__}: {exc}"
            self.log.log("ERROR", None, None, error=self.result.error[:500])
            self._tell_neighbours(self.result.error)
            if isinstance(exc, OutboxError):
                raise PipelineError(str(exc)) from exc
            raise
        finally:
            self._reader_stop.set()
            for reader in self.readers:
                reader.thread.join(timeout=0.5)
            self.outbox.close()
        if self.capture_params:
            self.result.final_params = self.stage.named_parameters_cpu()
        if self.cfg.trace:
            self.result.timeline = self.tl.export()
        return self.result


def run_stage(stage: Stage, spec, settings: PipelineSettings, *, upstream=None, downstream=None,
              worker: str = "local", logger: EventLogger | None = None,
              metrics_callback: Callable[[dict], None] | None = None, stop_event: threading.Event | None = None,
              capture_params: bool = False, timeline: Timeline | None = None) -> StageResult:
    """Runs ``settings.steps`` global steps of one stage; returns its losses, metrics and captures."""
    runner = StageRunner(stage, spec, settings, upstream, downstream, worker=worker, logger=logger,
                         metrics_callback=metrics_callback, stop_event=stop_event, capture_params=capture_params,
                         timeline=timeline)
    return runner.run()
