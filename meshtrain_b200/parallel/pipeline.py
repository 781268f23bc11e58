"""Schedule-driven execution of one stage over packet links (host data plane).

Semantics follow the reference executor (reference runtime/pipeline.py:66-461):
per global step a ``StageStateMachine`` walks the GPipe / 1F1B action list;
inbound packets are routed by (step, microbatch), packets for step+1 are
buffered, anything else is a protocol error; received tensors start their
host-to-device copy as soon as they arrive; forward outputs and input
gradients leave through the ``Outbox``; one optimizer step per global step;
every wait is bounded and a stall raises with a JSON state dump; on failure an
ERROR packet goes to both neighbours.

Threads: the caller's compute thread, one reader thread per link (bounded
event queue = back-pressure) and, in async mode, one sender thread per link.
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
from meshtrain_b200.networking.transport import Transport, TransportClosed, TransportTimeout
from meshtrain_b200.parallel.autograd import BoundaryError, MicrobatchContext
from meshtrain_b200.parallel.outbox import Outbox, OutboxError
from meshtrain_b200.parallel.schedule import ActionKind, Event, StageStateMachine
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


class Inbox:
    """One reader thread per link feeding a bounded event queue."""

    def __init__(self, links: dict[str, Transport], timeline: Timeline, maxsize: int, poll_s: float = 0.2):
        self.queue: queue.Queue = queue.Queue(maxsize=maxsize)
        self.timeline = timeline
        self.peak_depth = 0
        self._stop = threading.Event()
        self._threads = []
        for name, link in links.items():
            t = threading.Thread(target=self._reader, args=(name, link, poll_s), daemon=True, name=f"recv-{name}")
            t.start()
            self._threads.append(t)

    def _put(self, item) -> bool:
        while not self._stop.is_set():
            try:
                self.queue.put(item, timeout=0.2)
                self.peak_depth = max(self.peak_depth, self.queue.qsize())
                return True
            except queue.Full:
                continue  # back-pressure: stop reading until the executor drains
        return False

    def _reader(self, name: str, link: Transport, poll_s: float) -> None:
        tl = self.timeline
        while not self._stop.is_set():
            try:
                pkt = link.recv_packet(timeout=poll_s)
            except TransportTimeout:
                continue
            except Exception as exc:  # noqa: BLE001 - closed peer, malformed frame...
                if not self._stop.is_set():
                    self._put(("error", name, exc))
                return
            end = tl.now()
            tl.add("NETWORK_RECV", end - getattr(link, "last_frame_s", 0.0), end, pkt.step_id, pkt.microbatch_id,
                   link=name, bytes=len(pkt.payload))
            tensor = getattr(pkt, "recv_buffer", None)
            if tensor is None and pkt.has_tensor:
                with tl.span("DESERIALIZE", pkt.step_id, pkt.microbatch_id):
                    tensor = bytes_to_tensor(pkt.payload, pkt.dtype, pkt.shape)
            if not self._put(("packet", name, pkt, tensor)):
                return

    def stop(self, join_s: float = 0.0) -> None:
        self._stop.set()
        for t in self._threads:
            t.join(timeout=join_s)


class _StepState:
    def __init__(self, step: int, sm: StageStateMachine):
        self.step = step
        self.sm = sm
        self.acts: dict[int, tuple] = {}
        self.targets: dict[int, torch.Tensor] = {}
        self.grads: dict[int, tuple] = {}
        self.tokens: dict[int, list] = {}


class _HostOnly:
    """Staging for tensors already in host memory (targets relayed downstream)."""

    @staticmethod
    def begin_d2h(tensor):
        t = tensor.detach()
        return lambda: (t, None)


def run_stage(stage: Stage, spec, settings: PipelineSettings, *, upstream: Transport | None,
              downstream: Transport | None, worker: str = "local", logger: EventLogger | None = None,
              metrics_callback: Callable[[dict], None] | None = None, stop_event: threading.Event | None = None,
              capture_params: bool = False, timeline: Timeline | None = None) -> StageResult:
    logger = logger or EventLogger(worker, settings.job_id)
    if (upstream is None) != stage.is_first or (downstream is None) != stage.is_last:
        raise PipelineError("stage links do not match stage position")
    M = settings.num_microbatches
    if settings.batch_size % M:
        raise PipelineError("batch_size must be divisible by num_microbatches")
    S, sidx = stage.num_stages, stage.stage_index
    links = {k: v for k, v in ((UPSTREAM, upstream), (DOWNSTREAM, downstream)) if v is not None}
    tl = timeline or Timeline(worker, sidx)
    inbox = Inbox(links, tl, maxsize=4 * M + 16) if links else None
    events = inbox.queue if inbox else queue.Queue()
    outbox = Outbox(links, tl, async_mode=settings.async_transport, max_queue=settings.max_outbound_queue or 2 * M + 4,
                    timeout_s=settings.timeout_s, events=events)
    result = StageResult(sidx, worker)
    if capture_params:
        result.initial_params = stage.named_parameters_cpu()
    dev = stage.device
    dev.configure_transfers(pinned=settings.pinned_memory, pool=settings.buffer_pool)
    recv_types = (int(MessageType.FORWARD_ACTIVATION), int(MessageType.BACKWARD_GRADIENT))
    for link in links.values():
        link.payload_allocator = (lambda mtype, dtype, shape:
                                  dev.recv_buffer(shape, dtype) if mtype in recv_types else None)
    future: dict[int, list] = {}
    cur: dict = {"st": None, "bytes_received": 0}

    def stall(reason: str) -> PipelineError:
        st: _StepState | None = cur["st"]
        dump = {"reason": reason, "worker": worker, "stage": sidx,
                "state": st.sm.snapshot() if st else None,
                "buffered": ({k: sorted(getattr(st, k)) for k in ("acts", "targets", "grads")} if st else None),
                "future_steps": {s: len(v) for s, v in future.items()},
                "saved_contexts": [list(k) for k in stage.contexts.pending()],
                "pending_sends": outbox.pending(), "inbound_queue": events.qsize()}
        logger.log("PIPELINE_STALLED", None, None, dump=json.dumps(dump))
        return PipelineError(f"{reason}; state: {json.dumps(dump)}")

    def h2d_begin(tensor, step, mb):
        if dev.backend == "cpu":
            return dev.begin_h2d(tensor)
        with tl.span("H2D_COPY", step, mb, phase="begin"):
            return dev.begin_h2d(tensor)

    def h2d_finish(entry, step, mb):
        handle, token = entry[0], entry[1]
        cur["st"].tokens.setdefault(mb, []).append(token)
        if dev.backend == "cpu":
            return dev.finish_h2d(handle)
        with tl.span("H2D_COPY", step, mb, phase="finish"):
            return dev.finish_h2d(handle)

    def route(link: str, pkt: TensorPacket, tensor) -> None:
        st: _StepState = cur["st"]
        mb, mtype = pkt.microbatch_id, pkt.message_type
        if mtype == MessageType.TARGET and link == UPSTREAM:
            st.targets[mb] = tensor
            if mb in st.acts:
                st.sm.on(Event.ACTIVATION_RECEIVED, mb)
        elif mtype == MessageType.FORWARD_ACTIVATION and link == UPSTREAM:
            if mb in st.acts:
                raise BoundaryError(f"duplicate activation for step {pkt.step_id} microbatch {mb}")
            st.acts[mb] = h2d_begin(tensor, pkt.step_id, mb)
            if not stage.is_last or mb in st.targets:
                st.sm.on(Event.ACTIVATION_RECEIVED, mb)
        elif mtype == MessageType.BACKWARD_GRADIENT and link == DOWNSTREAM:
            st.grads[mb] = (*h2d_begin(tensor, pkt.step_id, mb), dict(pkt.meta))
            st.sm.on(Event.GRADIENT_RECEIVED, mb)
        else:
            raise BoundaryError(f"unexpected {mtype.name} from {link}")

    def pump(timeout: float) -> bool:
        if stop_event is not None and stop_event.is_set():
            raise PipelineError("job stopped")
        try:
            item = events.get(timeout=timeout)
        except queue.Empty:
            return False
        kind = item[0]
        if kind == "error":
            _, name, exc = item
            if isinstance(exc, TransportClosed):
                raise PipelineError(f"{name} peer disconnected: {exc}") from exc
            raise PipelineError(f"{name} link failed: {exc}") from exc
        if kind == "send_error":
            _, name, exc = item
            raise PipelineError(f"send to {name} peer failed: {type(exc).__name__}: {exc}") from exc
        if kind == "send_done":
            _, _n, step_id, mb = item
            st = cur["st"]
            if st is not None and step_id == st.step:
                st.sm.on(Event.SEND_COMPLETED, mb)
            return True
        _, link, pkt, tensor = item
        if pkt.message_type == MessageType.ERROR:
            raise PipelineError(f"{link} peer reported error: {pkt.meta.get('error')}")
        if pkt.job_id != settings.job_id:
            raise BoundaryError(f"packet for job {pkt.job_id!r} received in job {settings.job_id!r}")
        cur["bytes_received"] += len(pkt.payload)
        if pkt.message_type == MessageType.TARGET and not stage.is_last:
            outbox.submit_packet(DOWNSTREAM, pkt)  # relay unchanged
            return True
        st = cur["st"]
        if pkt.step_id == st.step:
            route(link, pkt, tensor)
        elif pkt.step_id == st.step + 1:
            future.setdefault(pkt.step_id, []).append((link, pkt, tensor))
        else:
            raise BoundaryError(f"packet for step {pkt.step_id} while in step {st.step}")
        return True

    def wait_ready(action, step: int) -> None:
        sm = cur["st"].sm
        if sm.ready(action):
            return
        cat = "WAIT_FORWARD" if action.kind is ActionKind.FORWARD else "WAIT_BACKWARD"
        t0 = tl.now()
        last = time.monotonic()
        while not sm.ready(action):
            if pump(min(settings.timeout_s, 0.5)):
                last = time.monotonic()
            elif time.monotonic() - last > settings.timeout_s:
                raise stall(f"pipeline stalled: no progress within network timeout {settings.timeout_s}s "
                            f"waiting for {action}")
        tl.add(cat, t0, tl.now(), step, action.microbatch)

    def release(mb: int) -> None:
        for token in cur["st"].tokens.pop(mb, []):
            dev.after_use(token)

    try:
        for local_step in range(settings.steps):
            step = settings.step_offset + local_step
            t_start = tl.now()
            if stage.is_first:
                dev.reset_peak_memory()
            sm = StageStateMachine(sidx, S, M, step, settings.schedule, settings.max_inflight_microbatches)
            st = _StepState(step, sm)
            cur["st"] = st
            recv0, sent0 = cur["bytes_received"], sum(outbox.bytes_sent.values())
            for link, pkt, tensor in future.pop(step, []):
                route(link, pkt, tensor)
            if stage.is_first:
                x, y = spec.make_batch(step, settings.batch_size)
                xs, ys = x.chunk(M), y.chunk(M)
            loss_sum = 0.0
            peak_saved = peak_mbs = 0
            while not sm.done:
                action = sm.next_action()
                mb = action.microbatch
                wait_ready(action, step)
                if action.kind is ActionKind.FORWARD:
                    if stage.is_first:
                        inp = xs[mb]
                        if not stage.is_last:
                            outbox.submit_tensor(DOWNSTREAM, ys[mb], MessageType.TARGET, device=_HostOnly, step=step,
                                                 microbatch=mb, job_id=settings.job_id, source_worker=worker)
                    else:
                        inp = h2d_finish(st.acts.pop(mb), step, mb)
                    ctx = MicrobatchContext(step, mb)
                    sm.on(Event.FORWARD_STARTED, mb)
                    with tl.span("FORWARD_COMPUTE", step, mb):
                        out = stage.forward(inp, ctx)
                    sm.on(Event.FORWARD_FINISHED, mb)
                    peak_saved = max(peak_saved, stage.contexts.saved_bytes())
                    peak_mbs = max(peak_mbs, len(stage.contexts))
                    if not stage.is_last:
                        outbox.submit_tensor(DOWNSTREAM, out.detach(), MessageType.FORWARD_ACTIVATION, device=dev,
                                             step=step, microbatch=mb, notify=True, job_id=settings.job_id,
                                             source_worker=worker)
                    if settings.log_microbatch_events:
                        logger.log("FORWARD_COMPLETE", step, mb, output=out.numel() * out.element_size(),
                                   compute_s=ctx.timings["forward"])
                else:
                    sm.on(Event.BACKWARD_STARTED, mb)
                    if stage.is_last:
                        target = ys[mb] if stage.is_first else st.targets.pop(mb)
                        with tl.span("BACKWARD_COMPUTE", step, mb):
                            loss, grad_in, ctx = stage.loss_backward(target, (step, mb), loss_scale=1.0 / M)
                        meta = {"loss": float(loss)}
                    else:
                        entry = st.grads.pop(mb)
                        meta = entry[2]
                        grad = h2d_finish(entry, step, mb)
                        with tl.span("BACKWARD_COMPUTE", step, mb):
                            grad_in, ctx = stage.backward(grad, (step, mb))
                    sm.on(Event.BACKWARD_FINISHED, mb)
                    release(mb)
                    loss_sum += float(meta.get("loss", 0.0))
                    if not stage.is_first:
                        outbox.submit_tensor(UPSTREAM, grad_in, MessageType.BACKWARD_GRADIENT, device=dev, step=step,
                                             microbatch=mb, job_id=settings.job_id, source_worker=worker, meta=meta)
                    if settings.log_microbatch_events:
                        logger.log("BACKWARD_COMPLETE", step, mb, compute_s=ctx.timings["backward"])
                sm.advance()
            if not sm.all_complete():
                raise stall("schedule finished with incomplete microbatches")
            if settings.capture_gradients_at_step == step:
                result.gradients = stage.named_gradients()
            probe = local_step < settings.correctness_probe_steps
            if probe:
                grad_norms = {n: float(p.grad.detach().float().norm()) for n, p in stage.module.named_parameters()
                              if p.grad is not None}
                before = stage.named_parameters_cpu() if local_step == 0 else None
            stage.refresh_tensor_store()
            mem = stage.memory_report()
            mem["tensor_store"] = stage.tensor_store.bytes_by_role()
            mem["saved_activations_peak"] = peak_saved
            mem["saved_microbatches_peak"] = peak_mbs
            with tl.span("OPTIMIZER_STEP", step):
                opt_s = stage.optimizer_step()
            stage.zero_grad()
            t_end = tl.now()
            step_s = t_end - t_start
            m = tl.step_metrics(step, (t_start, t_end))
            ph = m["phase_s"]
            mean_loss = loss_sum / M
            dm = dev.memory_stats()
            record = {
                "event": "STEP_COMPLETE", "job": settings.job_id, "worker": worker, "stage": sidx,
                "backend": dev.backend, "step": step, "schedule": settings.schedule,
                "async_transport": settings.async_transport, "step_s": step_s,
                "forward_s": ph.get("FORWARD_COMPUTE", 0.0), "backward_s": ph.get("BACKWARD_COMPUTE", 0.0),
                "optimizer_s": opt_s, "compute_s": m["compute_s"], "comm_s": m["communication_s"],
                "communication_s": m["communication_s"], "overlapped_s": m["overlapped_s"],
                "exposed_communication_s": m["exposed_communication_s"], "overlap_ratio": m["overlap_ratio"],
                "idle_s": m["idle_s"], "wait_forward_s": ph.get("WAIT_FORWARD", 0.0),
                "wait_backward_s": ph.get("WAIT_BACKWARD", 0.0),
                "bytes_sent": sum(outbox.bytes_sent.values()) - sent0,
                "bytes_received": cur["bytes_received"] - recv0,
                "lifecycle": {k: v for k, v in ph.items() if not k.startswith("WAIT")},
                "outbound_queue_peak": max(outbox.peak_depth.values(), default=0),
                "inbound_queue_peak": inbox.peak_depth if inbox else 0,
                "peak_inflight_microbatches": sm.peak_inflight, "buffer_pool": dev.host_pool.stats(),
                "utilization": m["compute_s"] / step_s if step_s else 0.0,
                "memory": {**mem, "device_allocated": dm.get("allocated", 0),
                           "device_peak": dm.get("peak_allocated", 0), "device_total": dm.get("total", 0)},
            }
            if probe:
                corr = {"grad_norms": grad_norms}
                if before is not None:
                    after = stage.named_parameters_cpu()
                    corr["param_delta_norms"] = {n: float((after[n] - before[n]).float().norm()) for n in before}
                record["correctness"] = corr
            if stage.is_first:
                record["loss"] = mean_loss
                record["samples_per_s"] = settings.batch_size / step_s if step_s else 0.0
                seq = getattr(spec, "seq_len", None)
                if seq:
                    record["tokens_per_s"] = settings.batch_size * seq / step_s if step_s else 0.0
                result.losses.append(mean_loss)
            result.step_metrics.append(record)
            if metrics_callback is not None:
                metrics_callback(record)
            if not settings.trace:
                tl.drop_before(t_end)
            if local_step % settings.log_every == 0 or local_step == settings.steps - 1:
                fields = {"step_s": step_s, "compute_s": m["compute_s"], "comm_s": m["communication_s"],
                          "exposed_s": m["exposed_communication_s"], "idle_s": m["idle_s"],
                          "sent_bytes": record["bytes_sent"]}
                if stage.is_first:
                    fields = {"loss": mean_loss, **fields}
                logger.log("STEP_COMPLETE", step, None, **fields)
        outbox.flush()
    except Exception as exc:
        result.error = f"{type(exc).__name__}: {exc}"
        logger.log("ERROR", None, None, error=result.error[:500])
        for link in links.values():  # tell the neighbours so they fail fast
            try:
                link.send_packet(TensorPacket(MessageType.ERROR, job_id=settings.job_id, source_worker=worker,
                                              meta={"error": f"{worker}: {result.error}"[:200]}))
            except Exception:  # noqa: BLE001
                pass
        if isinstance(exc, OutboxError):
            raise PipelineError(str(exc)) from exc
        raise
    finally:
        if inbox is not None:
            inbox.stop(join_s=0.5)
        outbox.close()
    if capture_params:
        result.final_params = stage.named_parameters_cpu()
    if settings.trace:
        result.timeline = tl.export()
    return result
