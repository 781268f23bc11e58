"""Device-side pipeline engine for GPU stages (one process per GPU).

This is the B200 hot path.  Compared with the reference's per-stage executor
(reference runtime/pipeline.py:157-461, which blocks the host on the device
after every forward/backward, runtime/stage.py:118,141,160,172,184):

* no host synchronisation inside a step: actions are enqueued on the compute
  stream; stage-boundary tensors move by NCCL p2p on per-direction streams
  (``parallel/p2p.py``) and the compute stream waits on them only when needed;
* layers run their explicit fwd/bwd (``models/base.PipelineLayer``) on the
  hand-written kernels, with weight gradients accumulated in fp32 in the GEMM
  epilogue straight into one flat gradient buffer;
* all parameters of a stage live in flat buffers (fp32 master, fp32 grad,
  Adam moments, bf16 compute copy) so the optimizer is one fused launch;
* every action is bracketed by CUDA events; after the step one event sync
  yields device-timed step time, compute time, bubble and exposed p2p time.

Training semantics are the reference's: one optimizer step per global step,
loss scaled by 1/M, gradients accumulated over the M microbatches
(reference docs/pipeline-scheduling.md:3-15).
"""

from __future__ import annotations

import math
import os
import time
from dataclasses import dataclass, field

import torch
from torch import nn

from meshtrain_b200 import ops
from meshtrain_b200.models.base import ModelSpec
from meshtrain_b200.parallel.schedule import ActionKind, ChunkAction, ChunkLedger, StepLedger, stage_schedule

ALIGN = 64  # elements; keeps every parameter view 128-byte aligned for TMA


class FlatState:
    """All parameters of one stage in contiguous buffers.

    ``master`` fp32 (the optimizer's copy), ``compute`` the dtype the kernels
    read (bf16 views that the layers' parameters point into; the same buffer
    as ``master`` in fp32 runs), ``grad`` fp32 accumulators, ``exp_avg`` /
    ``exp_avg_sq`` Adam moments.  With ``offload`` the master copy and moments
    live in pinned host memory (see ``parallel/offload.py``).
    """

    def __init__(self, layers: list[nn.Module], device: torch.device, compute_dtype: torch.dtype,
                 offload: bool = False):
        self.device = device
        self.entries: list[tuple[int, str, nn.Parameter, int, int]] = []
        off = 0
        for li, layer in enumerate(layers):
            for name, p in layer.named_parameters():
                n = p.numel()
                self.entries.append((li, name, p, off, n))
                off += (n + ALIGN - 1) // ALIGN * ALIGN
        self.numel = max(off, ALIGN)
        self.offload = offload
        host_kw = dict(device="cpu", pin_memory=torch.cuda.is_available()) if offload else dict(device=device)
        self.master = torch.zeros(self.numel, dtype=torch.float32, **host_kw)
        for _li, _name, p, o, n in self.entries:
            self.master[o:o + n].copy_(p.detach().reshape(-1).to(torch.float32))
        if compute_dtype == torch.float32 and not offload:
            self.compute = self.master
        else:
            self.compute = torch.zeros(self.numel, dtype=compute_dtype, device=device)
            self.compute.copy_(self.master.to(device, non_blocking=False) if offload else self.master)
        for _li, _name, p, o, n in self.entries:
            p.data = self.compute[o:o + n].view(p.shape)
            p.requires_grad_(False)
        self.grad = torch.zeros(self.numel, dtype=torch.float32, device=device)
        self.grads: list[dict[str, torch.Tensor]] = [dict() for _ in layers]
        for li, name, p, o, n in self.entries:
            self.grads[li][name] = self.grad[o:o + n].view(p.shape)
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        if offload and torch.cuda.is_available():
            self.exp_avg = self.exp_avg.pin_memory()
            self.exp_avg_sq = self.exp_avg_sq.pin_memory()

    def bytes_by_role(self) -> dict[str, int]:
        e = 4 * self.numel
        return {"parameter": self.compute.numel() * self.compute.element_size(), "master": e, "gradient": e,
                "optimizer_state": 2 * e}

    def device_bytes(self) -> int:
        """Bytes these buffers hold on the stage's device (host-offloaded state and shared views excluded)."""
        seen, total = set(), 0
        for buf in (self.compute, self.master, self.grad, self.exp_avg, self.exp_avg_sq):
            if buf.device.type == self.device.type and buf.data_ptr() not in seen:
                seen.add(buf.data_ptr())
                total += buf.numel() * buf.element_size()
        return total

    def named_master(self, layer_offset: int = 0, global_layer=None) -> dict[str, torch.Tensor]:
        g = global_layer or (lambda i: i)
        return {f"model.layers.{g(li + layer_offset)}.{name}": self.master[o:o + n].view(p.shape)
                for li, name, p, o, n in self.entries}


@dataclass
class StepStats:
    step: int
    stage: int
    loss: float | None = None
    step_ms: float = 0.0
    forward_ms: float = 0.0
    backward_ms: float = 0.0
    optimizer_ms: float = 0.0
    compute_ms: float = 0.0
    wait_ms: float = 0.0
    exposed_p2p_ms: float = 0.0     # filled by PipelineTrainer.p2p_report from the senders' transfer times
    bubble_fraction: float = 0.0
    busy_ms: float = 0.0            # union of the compute stream's actions, the optimizer and side-stream work
    side_ms: float = 0.0            # weight-gradient GEMMs on the side stream
    recv_wait_ms: dict = field(default_factory=dict)   # "F<mb>" / "B<mb>": compute-stream stall on that receive
    send_ms: dict = field(default_factory=dict)        # "F<mb>" / "B<mb>": device time of this rank's send
    bytes_sent: int = 0
    bytes_received: int = 0
    peak_inflight: int = 0
    tokens: int = 0
    spans: list[dict] = field(default_factory=list)
    loss_ready: object = None       # CUDA event after the loss (last stage)
    pending: object = None          # events of a deferred-timing step, until finish_timing

    def to_record(self) -> dict:
        d = dict(self.__dict__)
        for key in ("spans", "recv_wait_ms", "send_ms", "loss_ready", "pending"):
            d.pop(key, None)
        return d


def interval_union_ms(intervals: list[tuple[float, float]]) -> float:
    """Total length of the union of [start, end) intervals."""
    total, reach = 0.0, float("-inf")
    for start, end in sorted(intervals):
        if end <= reach:
            continue
        total += end - max(start, reach)
        reach = end
    return total


class _Events:
    """Reusable CUDA event pool (creating events per action costs host time)."""

    def __init__(self):
        self.pool: list[torch.cuda.Event] = []
        self.i = 0

    def reset(self):
        self.i = 0

    def record(self, stream=None) -> torch.cuda.Event:
        if self.i == len(self.pool):
            self.pool.append(torch.cuda.Event(enable_timing=True))
        ev = self.pool[self.i]
        self.i += 1
        ev.record(stream)
        return ev


class SideStreamSpans:
    """Event brackets around the side-stream weight-gradient work of each action.

    ``side_work`` (called by the kernels layer before it enqueues a side-stream
    GEMM) opens a span with an event on the side stream; ``close`` at the end
    of the action records the closing event after the last GEMM it enqueued.
    Two events per action keep the bookkeeping off the critical path.
    """

    def __init__(self, events: "_Events"):
        self.events = events
        self.spans: list = []
        self._open = None
        self._stream = None

    def side_work(self, stream) -> None:
        if self._open is None:
            self._open, self._stream = self.events.record(stream), stream

    def close(self) -> None:
        if self._open is not None:
            self.spans.append((self._open, self.events.record(self._stream)))
            self._open = None


_RECOMPUTE_INPUT = "_recompute_input"


class PipelineEngine:
    """Runs one pipeline stage of a model on one GPU (or on CPU for tests)."""

    def __init__(self, spec: ModelSpec, *, layer_range: tuple[int, int] | None = None, stage: int, num_stages: int,
                 device: torch.device | str, num_microbatches: int, schedule: str = "1f1b",
                 max_inflight: int | None = None, optimizer: str = "adam", lr: float = 1e-3,
                 betas: tuple[float, float] = (0.9, 0.999), eps: float = 1e-8, weight_decay: float = 0.0,
                 links=None, init_on_device: bool = False,
                 record_spans: bool = True, offload=None, microbatch_size: int | None = None,
                 deferred_wgrad: bool = True, chunk_ranges: list[tuple[int, int]] | None = None,
                 recompute: set[int] | None = None):
        """``chunk_ranges``: the rank's model chunks for an interleaved 1F1B program (chunk c
        of this rank is virtual stage c * num_stages + stage); ``layer_range`` otherwise.
        ``recompute``: global units whose activations are recomputed in backward instead of
        kept (``parallel/recompute.py``)."""
        self.spec = spec
        self.deferred_wgrad = deferred_wgrad  # weight-gradient GEMMs on a side stream (CUDA)
        self.microbatch_size = microbatch_size  # middle stages see neither inputs nor targets
        self.device = torch.device(device)
        self.stage, self.num_stages = stage, num_stages
        self.is_first, self.is_last = stage == 0, stage == num_stages - 1
        ranges = [tuple(r) for r in chunk_ranges] if chunk_ranges else [tuple(layer_range)]
        self.chunk_ranges = ranges
        self.chunks = len(ranges)
        if self.chunks > 1 and schedule != "1f1b":
            raise ValueError("model chunks per rank need the 1f1b schedule (interleaved 1F1B)")
        self.start, self.end = ranges[0][0], ranges[-1][1]
        self.layer_ids = [i for a, b in ranges for i in range(a, b)]
        self.chunk_bounds = [0]
        for a, b in ranges:
            self.chunk_bounds.append(self.chunk_bounds[-1] + (b - a))
        self.M = num_microbatches
        self.schedule = schedule
        self.max_inflight = max_inflight
        if optimizer not in ("adam", "adamw", "sgd"):
            raise ValueError(f"unknown optimizer {optimizer!r}")
        self.opt_name = optimizer
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.links = links
        if num_stages > 1 and links is None:
            raise ValueError("a multi-stage engine needs StageLinks")
        init_dev = self.device if (init_on_device and self.device.type == "cuda") else None
        self.layers = [spec.build_layer(i, init_dev).to(self.device) for i in self.layer_ids]
        last_unit = spec.num_layers - 1  # the fused LM head runs its backward inside its forward
        self.recompute_local = {li for li, u in enumerate(self.layer_ids) if u in (recompute or ()) and u != last_unit}
        self.compute_dtype = spec.dtype
        self.flat = FlatState(self.layers, self.device, self.compute_dtype, offload=offload is not None)
        self.offload = offload
        if offload is not None:
            offload.attach(self.flat)
        self.loss_sum = torch.zeros((), dtype=torch.float32, device=self.device)
        self.opt_steps = 0
        self.cuda = self.device.type == "cuda"
        self.events = _Events() if self.cuda else None
        self._spare_pools: list[_Events] = []  # event pools of finished deferred-timing steps
        self.record_spans = record_spans
        self._has_fused_loss = hasattr(self.layers[-1], "fwd_loss")
        self.failure_check = None  # () -> reason or None: set by a trainer that watches its peers
        # NVTX ranges per action and for the optimizer (MESHTRAIN_NVTX=1), for Nsight timelines
        self.nvtx = os.environ.get("MESHTRAIN_NVTX") == "1"

    # ------------------------------------------------------------------ helpers
    def wait_event(self, event) -> None:
        """Waits on the host for ``event``; with a ``failure_check`` it polls instead of
        blocking inside CUDA, so a rank whose NCCL receive waits on a failed peer
        raises ``PeerFailure`` rather than blocking for good."""
        check = self.failure_check
        if check is None:
            event.synchronize()
            return
        while not event.query():
            reason = check()
            if reason is not None:
                from meshtrain_b200.parallel.watchdog import PeerFailure

                raise PeerFailure(reason)
            time.sleep(0.0002)

    def boundary_shape(self, mb_size: int) -> tuple[int, ...]:
        return self.spec.boundary_shape(mb_size)

    def _recv_buf(self, mb_size: int) -> torch.Tensor:
        return torch.empty(self.boundary_shape(mb_size), dtype=self.compute_dtype, device=self.device)

    def _forward_layers(self, x, saved_list, lo, hi):
        for li, sv in zip(range(lo, hi), saved_list):
            if li in self.recompute_local:
                # keep only the input; the backward runs this forward again (_rematerialise)
                x_in, x = x, self.layers[li].fwd(x, {})
                sv[_RECOMPUTE_INPUT] = x_in
            else:
                x = self.layers[li].fwd(x, sv)
        return x

    def _rematerialise(self, li: int, sv: dict) -> dict:
        """Saved tensors of a recomputed layer, from its kept input (forward run again)."""
        x_in = sv.pop(_RECOMPUTE_INPUT, None)
        if x_in is not None:
            self.layers[li].fwd(x_in, sv)
        return sv

    def first_virtual(self, chunk: int) -> bool:
        """Chunk ``chunk`` of this rank is the model's first piece (it reads the token ids)."""
        return self.is_first and chunk == 0

    def last_virtual(self, chunk: int) -> bool:
        """Chunk ``chunk`` of this rank is the model's last piece (it computes the loss)."""
        return self.is_last and chunk == self.chunks - 1

    def boundary(self, kind: str, chunk: int, sender: bool) -> int:
        """Index k of the virtual-stage boundary a message crosses (k -> k+1 forward,
        k+1 -> k backward); sender and receiver derive the same k."""
        vs = chunk * self.num_stages + self.stage
        if kind == "F":
            return vs if sender else vs - 1
        return vs - 1 if sender else vs

    def _last_forward_loss(self, h, y, saved_list):
        head = self.layers[-1]
        grads = self.flat.grads[-1]
        if self._has_fused_loss:
            head.fwd_loss(h, y, saved_list[-1], grads, self.loss_sum, 1.0 / self.M)
            return
        # generic path: explicit forward of the last layer, loss gradient by autograd
        out = head.fwd(h, saved_list[-1])
        out_l = out.detach().float().requires_grad_(True)
        with torch.enable_grad():
            loss = self.spec.loss_fn(out_l, y)
            (loss / self.M).backward()
        self.loss_sum += loss.detach().float()
        saved_list[-1]["dx"] = head.bwd(out_l.grad.to(out.dtype), saved_list[-1], grads)

    def optimizer_step(self) -> None:
        self.opt_steps += 1
        f = self.flat
        if self.offload is not None:
            self.offload.step(self)
            return
        lowp = None if f.compute is f.master else f.compute
        if self.opt_name == "sgd":
            f.master.add_(f.grad, alpha=-self.lr)
            if lowp is not None:
                lowp.copy_(f.master)
            return
        ops.adam_(f.master, f.grad, f.exp_avg, f.exp_avg_sq, lowp, lr=self.lr, beta1=self.betas[0],
                  beta2=self.betas[1], eps=self.eps, weight_decay=self.wd, decoupled=self.opt_name == "adamw",
                  step=self.opt_steps)

    # ------------------------------------------------------------------ step
    def train_step(self, step: int, inputs: torch.Tensor | None = None, targets: torch.Tensor | None = None,
                   timed: bool | str = True) -> StepStats:
        """One global step: M microbatches through the schedule, then the optimizer.

        ``inputs`` (first stage) / ``targets`` (last stage) are the global
        batch, on the host (pinned for an async copy) or on the device.
        ``timed``: True waits for the step and fills its device timing;
        "deferred" records the same events without waiting (the host runs on
        into the next step) and ``finish_timing(stats)`` fills them later.
        """
        M = self.M
        dev = self.device
        if self.is_first:
            if inputs is None:
                raise ValueError("the first stage needs inputs")
            xs = inputs.to(dev, non_blocking=True).chunk(M)
        if self.is_last:
            if targets is None:
                raise ValueError("the last stage needs targets")
            ys = targets.to(dev, non_blocking=True).chunk(M)
        if inputs is not None or targets is not None:
            batch = (inputs if inputs is not None else targets).shape[0]
        elif self.microbatch_size is not None:
            batch = self.microbatch_size * M
        else:
            raise ValueError("a middle stage needs the engine's microbatch_size")
        mb_size = batch // M
        if batch % M:
            raise ValueError("batch size must be divisible by the number of microbatches")
        v = self.chunks
        if v == 1:
            ledger = StepLedger(self.stage, self.num_stages, M, step, self.schedule, self.max_inflight)
            actions = [ChunkAction(a.kind, 0, a.microbatch) for a in ledger.actions]
            plain = {a: b for a, b in zip(actions, ledger.actions)}
            l_input = lambda c, m: ledger.input_arrived(m)  # noqa: E731
            l_grad = lambda c, m: ledger.gradient_arrived(m)  # noqa: E731
            l_sent = lambda c, m: ledger.forward_sent(m)  # noqa: E731
            l_run = lambda a: ledger.run(plain[a])  # noqa: E731
            l_finish = lambda a: ledger.finish(plain[a])  # noqa: E731
        else:
            ledger = ChunkLedger(self.stage, self.num_stages, M, step, v)
            actions = ledger.actions
            l_input, l_grad, l_sent = ledger.input_arrived, ledger.gradient_arrived, ledger.forward_sent
            l_run, l_finish = ledger.run, ledger.finish
        deferred = timed == "deferred"
        ev = self.events
        if ev is not None and deferred:  # this step's events stay untouched until finish_timing
            ev = self._spare_pools.pop() if self._spare_pools else _Events()
        if ev is not None:
            ev.reset()
            t0 = ev.record()
        self.flat.grad.zero_()
        self.loss_sum.zero_()
        if self.offload is not None:
            self.offload.prefetch(self)  # optimizer state for this step's update starts moving now
        links = self.links
        if links is not None:
            links.reset_stats()
        pending: dict[tuple[str, int, int], tuple] = {}
        S = self.num_stages

        def needs_remote(a):
            if a.kind is ActionKind.FORWARD:
                return not self.first_virtual(a.chunk)
            return not self.last_virtual(a.chunk)

        def post(a):
            key = (a.kind.value, a.chunk, a.microbatch)
            if key in pending or not needs_remote(a):
                return
            buf = self._recv_buf(mb_size)
            if a.kind is ActionKind.FORWARD:
                work = links.recv_activation(buf) if self.stage > 0 else links.recv_activation_ring(buf)
            else:
                work = links.recv_gradient(buf) if self.stage < S - 1 else links.recv_gradient_ring(buf)
            pending[key] = (work, buf)

        def msg_key(kind: str, mb: int, chunk: int, sender: bool) -> str:
            return f"{kind}{mb}" if v == 1 else f"{kind}{mb}/{self.boundary(kind, chunk, sender)}"

        saved: dict[tuple[int, int], list[dict]] = {}
        sends = []
        marks = []  # (message key, kind, ev_start, ev_ready, ev_end)
        if actions:
            post(actions[0])
        side = SideStreamSpans(ev) if ev is not None else None
        wgrad_ctx = ops.deferred_wgrad(self.deferred_wgrad and self.device.type == "cuda", timer=side)
        wgrad_ctx.__enter__()
        try:
            for i, a in enumerate(actions):
                if i + 1 < len(actions):
                    post(actions[i + 1])
                mb, c = a.microbatch, a.chunk
                lo, hi = self.chunk_bounds[c], self.chunk_bounds[c + 1]
                if self.nvtx:
                    torch.cuda.nvtx.range_push(f"stage{self.stage} {a}")
                e_start = ev.record() if ev else None
                buf = None
                if needs_remote(a):
                    work, buf = pending.pop((a.kind.value, c, mb))
                    work.wait()
                    (l_input if a.kind is ActionKind.FORWARD else l_grad)(c, mb)
                e_ready = ev.record() if ev else None
                l_run(a)
                last = self.last_virtual(c)
                hi_fwd = hi - 1 if last else hi
                if a.kind is ActionKind.FORWARD:
                    x = xs[mb] if self.first_virtual(c) else buf
                    sv = [dict() for _ in range(hi - lo)]
                    h = self._forward_layers(x, sv, lo, hi_fwd)
                    if last:
                        self._last_forward_loss(h, ys[mb], sv)
                    else:
                        key = msg_key("F", mb, c, True)
                        sends.append((key, links.send_activation(h) if self.stage < S - 1
                                      else links.send_activation_ring(h)))
                        l_sent(c, mb)  # ordering is kept by the NCCL stream
                    saved[(c, mb)] = sv
                else:
                    sv = saved.pop((c, mb))
                    dy = sv[-1].pop("dx") if last else buf
                    for li in reversed(range(lo, hi_fwd)):
                        layer_saved = self._rematerialise(li, sv[li - lo])
                        dy = self.layers[li].bwd(dy, layer_saved, self.flat.grads[li])
                        sv[li - lo] = None  # free this layer's activations before the next one's
                    del sv
                    if not self.first_virtual(c):
                        key = msg_key("B", mb, c, True)
                        sends.append((key, links.send_gradient(dy) if self.stage > 0
                                      else links.send_gradient_ring(dy)))
                l_finish(a)
                if side is not None:
                    side.close()
                e_end = ev.record() if ev else None
                if self.nvtx:
                    torch.cuda.nvtx.range_pop()
                marks.append((msg_key(a.kind.value, mb, c, False), a.kind.value, mb, e_start, e_ready, e_end))
        finally:
            wgrad_ctx.__exit__(None, None, None)  # the optimizer reads every weight gradient
        if not ledger.all_complete():
            raise RuntimeError(f"schedule finished with incomplete microbatches: {ledger.snapshot()}")
        for _key, w in sends:
            w.wait()
        e_opt0 = ev.record() if ev else None
        if self.nvtx:
            torch.cuda.nvtx.range_push(f"stage{self.stage} optimizer")
        self.optimizer_step()
        if self.nvtx:
            torch.cuda.nvtx.range_pop()
        e_opt1 = ev.record() if ev else None
        stats = StepStats(step=step, stage=self.stage, peak_inflight=ledger.peak_inflight, tokens=batch * (
            self.spec.seq_len if hasattr(self.spec, "seq_len") else 1))
        if links is not None:
            stats.bytes_sent = links.stats.bytes_sent
            stats.bytes_received = links.stats.bytes_received
        if self.is_last:
            stats.loss = self.loss_sum.clone()  # device scalar: sum over microbatches of the mean CE
            if self.cuda:
                stats.loss_ready = torch.cuda.Event()
                stats.loss_ready.record()
        if ev is not None and deferred:
            stats.pending = (ev, t0, marks, e_opt0, e_opt1, side.spans if side else [], sends)
        elif ev is not None and timed:
            self.wait_event(e_opt1)
            self._fill_timing(stats, t0, marks, e_opt0, e_opt1, side.spans if side else [], sends)
        return stats

    def finish_timing(self, stats: StepStats) -> StepStats:
        """Fills the device timing of a step run with ``timed="deferred"`` (waits for it)."""
        if stats.pending is None:
            return stats
        pool, t0, marks, e_opt0, e_opt1, side_spans, sends = stats.pending
        stats.pending = None
        self.wait_event(e_opt1)
        self._fill_timing(stats, t0, marks, e_opt0, e_opt1, side_spans, sends)
        self._spare_pools.append(pool)
        return stats

    def _fill_timing(self, st: StepStats, t0, marks, e_opt0, e_opt1, side_spans, sends) -> None:
        """Device-timed breakdown of the step from its CUDA events (all on this GPU).

        Busy time is the union of the compute stream's action spans, the
        optimizer and the side stream's weight-gradient GEMMs; the bubble is
        the rest of the step.  The stall of the compute stream before each
        receive is recorded per message, and each send's device time comes from
        NCCL's own timing (``TORCH_NCCL_ENABLE_TIMING``), so that the trainer
        can split stalls into transfer time and pipeline dependency.
        """
        from meshtrain_b200.parallel.p2p import work_duration_ms

        fwd = bwd = wait = 0.0
        busy = []
        spans = []
        for key, kind, mb, es, er, ee in marks:
            w = es.elapsed_time(er)
            c = er.elapsed_time(ee)
            wait += w
            if kind == "F":
                fwd += c
            else:
                bwd += c
            base = t0.elapsed_time(es)
            busy.append((base + w, base + w + c))
            if w > 0:
                st.recv_wait_ms[key] = w
            if self.record_spans:
                if w > 0.001:
                    spans.append({"cat": "WAIT_FORWARD" if kind == "F" else "WAIT_BACKWARD", "mb": mb,
                                  "start_ms": base, "end_ms": base + w})
                spans.append({"cat": "FORWARD_COMPUTE" if kind == "F" else "BACKWARD_COMPUTE", "mb": mb,
                              "start_ms": base + w, "end_ms": base + w + c})
        side = [(t0.elapsed_time(a), t0.elapsed_time(b)) for a, b in side_spans]
        opt = e_opt0.elapsed_time(e_opt1)
        total = t0.elapsed_time(e_opt1)
        b_opt = t0.elapsed_time(e_opt0)
        busy.append((b_opt, b_opt + opt))
        if self.record_spans:
            spans.append({"cat": "OPTIMIZER_STEP", "mb": None, "start_ms": b_opt, "end_ms": b_opt + opt})
            spans += [{"cat": "WGRAD_SIDE_STREAM", "mb": None, "start_ms": a, "end_ms": b} for a, b in side]
        for key, work in sends:
            ms = work_duration_ms(work)
            if ms is not None:
                st.send_ms[key] = ms
        st.forward_ms, st.backward_ms, st.optimizer_ms = fwd, bwd, opt
        st.compute_ms = fwd + bwd + opt
        st.side_ms = interval_union_ms(side)
        st.busy_ms = interval_union_ms(busy + side)
        st.wait_ms = wait
        st.step_ms = total
        st.bubble_fraction = max(0.0, 1.0 - st.busy_ms / total) if total > 0 else 0.0
        st.spans = spans

    # ------------------------------------------------------------------ state
    def sync_host_state(self) -> None:
        if self.offload is not None:
            self.offload.synchronize()

    def state_dict(self) -> dict:
        """Checkpoint tensors keyed by stable global IDs (model.layers.<g>.<name>[.optim.<k>])."""
        self.sync_host_state()
        out = {}
        f = self.flat
        for li, name, p, o, n in f.entries:
            gid = f"model.layers.{self.spec.global_layer(self.layer_ids[li])}.{name}"
            out[gid] = f.master[o:o + n].view(p.shape).detach().cpu().clone()
            out[gid + ".optim.exp_avg"] = f.exp_avg[o:o + n].view(p.shape).detach().cpu().clone()
            out[gid + ".optim.exp_avg_sq"] = f.exp_avg_sq[o:o + n].view(p.shape).detach().cpu().clone()
        out["optim.step"] = torch.tensor(self.opt_steps)
        return out

    def load_state_dict(self, sd: dict) -> None:
        f = self.flat
        for li, name, p, o, n in f.entries:
            gid = f"model.layers.{self.spec.global_layer(self.layer_ids[li])}.{name}"
            f.master[o:o + n].copy_(sd[gid].reshape(-1).to(f.master.dtype))
            if gid + ".optim.exp_avg" in sd:
                f.exp_avg[o:o + n].copy_(sd[gid + ".optim.exp_avg"].reshape(-1))
                f.exp_avg_sq[o:o + n].copy_(sd[gid + ".optim.exp_avg_sq"].reshape(-1))
        if f.compute is not f.master:
            f.compute.copy_(f.master.to(f.compute.device))
        self.opt_steps = int(sd.get("optim.step", torch.tensor(0)))

    def named_parameters_cpu(self) -> dict[str, torch.Tensor]:
        self.sync_host_state()
        g = self.spec.global_layer
        return {k: v.detach().cpu().clone()
                for k, v in self.flat.named_master(0, lambda li: g(self.layer_ids[li])).items()}

    def named_gradients_cpu(self) -> dict[str, torch.Tensor]:
        f = self.flat
        return {f"model.layers.{self.spec.global_layer(self.layer_ids[li])}.{name}": f.grad[o:o + n].view(p.shape).detach().cpu().clone()
                for li, name, p, o, n in f.entries}


def equal_split(num_layers: int, num_stages: int) -> list[tuple[int, int]]:
    """Contiguous, as-equal-as-possible layer ranges."""
    base, extra = divmod(num_layers, num_stages)
    out, s = [], 0
    for i in range(num_stages):
        n = base + (1 if i < extra else 0)
        out.append((s, s + n))
        s += n
    return out


def balanced_split(costs: list[float], num_stages: int) -> list[tuple[int, int]]:
    """Contiguous split minimising the largest per-stage cost (exact DP)."""
    n = len(costs)
    if num_stages > n:
        raise ValueError("more stages than layers")
    prefix = [0.0]
    for c in costs:
        prefix.append(prefix[-1] + c)
    INF = math.inf
    best = [[INF] * (n + 1) for _ in range(num_stages + 1)]
    cut = [[0] * (n + 1) for _ in range(num_stages + 1)]
    best[0][0] = 0.0
    for k in range(1, num_stages + 1):
        for j in range(k, n + 1):
            for i in range(k - 1, j):
                v = max(best[k - 1][i], prefix[j] - prefix[i])
                if v < best[k][j]:
                    best[k][j], cut[k][j] = v, i
    ranges, j = [], n
    for k in range(num_stages, 0, -1):
        i = cut[k][j]
        ranges.append((i, j))
        j = i
    return ranges[::-1]


def interleaved_split(costs: list[float], num_ranks: int, chunks: int) -> list[tuple[int, int]]:
    """Contiguous split into ``num_ranks * chunks`` pieces for an interleaved program,
    in which rank r runs pieces r, r + num_ranks, r + 2 num_ranks, ...

    Starts from the split that minimises the largest piece (``balanced_split``),
    then moves single cut points one unit at a time while that lowers the largest
    per-rank sum (ties: the largest piece).  The per-rank sum sets a rank's work
    per microbatch; a lone expensive piece (an LM head) is otherwise stacked on top
    of a full-size piece on its rank.
    """
    V = num_ranks * chunks
    n = len(costs)
    if V > n:
        raise ValueError("more pieces than layers")
    prefix = [0.0]
    for c in costs:
        prefix.append(prefix[-1] + c)
    cuts = [0] + [b for _a, b in balanced_split(costs, V)]

    def score(cs):
        pieces = [prefix[cs[i + 1]] - prefix[cs[i]] for i in range(V)]
        per_rank = [sum(pieces[r::num_ranks]) for r in range(num_ranks)]
        return max(per_rank), max(pieces)

    best = score(cuts)
    for _ in range(4 * n * V):
        improved = False
        for i in range(1, V):
            for d in (-1, 1):
                c = cuts[i] + d
                if not cuts[i - 1] < c < cuts[i + 1]:
                    continue
                trial = cuts[:i] + [c] + cuts[i + 1:]
                sc = score(trial)
                if sc < best:
                    cuts, best, improved = trial, sc, True
        if not improved:
            break
    return [(cuts[i], cuts[i + 1]) for i in range(V)]
