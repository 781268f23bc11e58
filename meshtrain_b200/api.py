"""Public training API for GPU pipelines (one process per GPU).

    from meshtrain_b200.api import PipelineTrainer
    trainer = PipelineTrainer({"type": "gpt", "layers": 24, ...}, num_microbatches=32)
    for step in range(steps):
        x, y = trainer.spec.make_batch(step, batch)            # host tensors (pinned is best)
        stats = trainer.step(step, x, y)                       # one global step
        if trainer.is_last: print(trainer.loss_value(stats))

Launch with ``torchrun --nproc-per-node N`` (or any launcher that sets
RANK / WORLD_SIZE / LOCAL_RANK / MASTER_ADDR / MASTER_PORT); rank r runs stage r.
A single process with no launcher runs all layers on one GPU (or on the CPU).

This is the in-box GPU counterpart of the reference's coordinator-driven
``meshtrain train`` (reference cli.py:380-415, runtime/pipeline.py:157):
same model specs, schedules and training semantics, with NCCL p2p links and
the device-side engine instead of TCP stage processes.
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist

from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.engine import PipelineEngine, StepStats, balanced_split, equal_split, interleaved_split


def dist_env() -> tuple[int, int, int]:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def init_distributed(backend: str | None = None, timeout_s: float | None = None) -> tuple[int, int, int]:
    """Initialise torch.distributed from the launcher's environment (no-op for one process).

    The process-group timeout (``MESHTRAIN_PG_TIMEOUT_S``, default 300 s) bounds
    every collective and point-to-point call; NCCL operation timing is switched
    on so that the engine can measure each send's device time.
    """
    rank, world, local = dist_env()
    if timeout_s is None:
        timeout_s = float(os.environ.get("MESHTRAIN_PG_TIMEOUT_S", "300"))
    os.environ.setdefault("TORCH_NCCL_ENABLE_TIMING", "1")
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29511")
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        kw = dict(backend=backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(**kw)
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, world, local


def _profiles(spec, microbatch_size: int, recompute: set[int] | None = None):
    """Layer profiles of ``spec`` (closed form for GPT / Llama), with recomputed units applied."""
    from meshtrain_b200.parallel.recompute import apply_to_profiles
    from meshtrain_b200.planner.graph import profiles_for

    layers = profiles_for(spec, microbatch_size)
    return apply_to_profiles(layers, recompute) if recompute else layers


def plan_device_pipeline(spec, num_stages: int, num_microbatches: int, microbatch_size: int, schedule: str,
                         optimizer: str, *, offload: bool = False, max_inflight: int | None = None,
                         memory_gb: float | None = None, recompute: set[int] | None = None,
                         offload_ring: dict | None = None):
    """Topology-aware placement of ``spec`` on ``num_stages`` GPUs of this box.

    Runs the planner (DP over contiguous splits, NVLink device links, the
    device engine's memory accounting) with one worker profile per local GPU;
    raises if no split fits the per-GPU memory budget.
    """
    from meshtrain_b200.planner.partition import PlannerOptions, b200_box, make_plan

    if memory_gb is None:
        memory_gb = (torch.cuda.get_device_properties(0).total_memory / 1024 ** 3
                     if torch.cuda.is_available() else 180.0)
    layers = _profiles(spec, microbatch_size, recompute)
    workers, network = b200_box(num_stages, memory_gb=memory_gb)
    eb = torch.empty((), dtype=spec.dtype).element_size()
    opts = PlannerOptions(optimizer=optimizer, num_microbatches=num_microbatches, schedule=schedule,
                          max_inflight=max_inflight, num_stages=num_stages, engine="device", param_dtype_bytes=eb,
                          dtype=str(spec.dtype).replace("torch.", ""), offload=offload, offload_ring=offload_ring)
    plan = make_plan("topology_aware", layers, workers, network, opts)
    if not plan.feasible:
        raise RuntimeError("no pipeline placement fits:\n" + plan.format())
    return plan


def check_interleaved_memory(spec, pieces: list[tuple[int, int]], world: int, chunks: int, num_microbatches: int,
                             microbatch_size: int, optimizer: str, *, offload: bool = False,
                             memory_gb: float | None = None, recompute: set[int] | None = None,
                             offload_ring: dict | None = None) -> list:
    """Startup memory estimate of an interleaved placement: one estimate per rank over its pieces.

    A rank holds ``chunks`` pieces (r, r + world, ...).  Its program keeps up to
    ``interleaved_warmup + 1`` chunk-forwards alive, each holding one chunk's saved
    activations, so the estimate counts that many times the largest chunk's
    activations.  Raises if a rank does not fit; returns the estimates.
    """
    from meshtrain_b200.planner.memory import estimate_interleaved_rank

    if memory_gb is None:
        memory_gb = (torch.cuda.get_device_properties(0).total_memory / 1024 ** 3
                     if torch.cuda.is_available() else 180.0)
    layers = _profiles(spec, microbatch_size, recompute)
    eb = torch.empty((), dtype=spec.dtype).element_size()
    out, failed = [], []
    for r in range(world):
        est = estimate_interleaved_rank(layers, pieces, r, world, chunks, num_microbatches,
                                        total=int(memory_gb * 1024 ** 3), optimizer=optimizer, param_dtype_bytes=eb,
                                        offload=offload, offload_ring=offload_ring)
        out.append(est)
        if not est.fits:
            failed.append(est.format(f"rank {r}"))
    if failed:
        raise RuntimeError("interleaved placement does not fit:\n" + "\n".join(failed))
    return out


def layer_costs(spec) -> list[float]:
    """Relative forward cost per layer (FLOPs per token), for partitioning."""
    from meshtrain_b200.planner.graph import analytic_layer_flops

    return analytic_layer_flops(spec)


def forecast_interleaving(costs: list[float], num_stages: int, num_microbatches: int,
                          chunk_options=(1, 2, 3, 4)) -> list[dict]:
    """Simulated step of each interleaving depth for a model's per-unit costs.

    For v model chunks per rank the units are split as the trainer splits them
    (``balanced_split`` for v = 1, ``interleaved_split`` otherwise) and the rank
    programs run against their dependencies with those piece costs (backward twice
    the forward).  Returns, per v: the bubble fraction, the makespan relative to
    v = 1, and the largest / mean per-rank work.  A model, not a measurement: it
    leaves out p2p latency and the smaller kernels of smaller pieces.
    """
    from meshtrain_b200.parallel.schedule import simulate, simulate_interleaved

    S, M = num_stages, num_microbatches
    rows, base = [], None
    for v in chunk_options:
        if v * S > len(costs) or (v > 1 and M % S):
            continue
        if v == 1:
            ranges = balanced_split(costs, S)
            pieces = [sum(costs[a:b]) for a, b in ranges]
            sim = simulate_interleaved(S, M, 1, piece_costs=pieces) if S > 1 else simulate("1f1b", 1, M)
        else:
            ranges = interleaved_split(costs, S, v)
            pieces = [sum(costs[a:b]) for a, b in ranges]
            sim = simulate_interleaved(S, M, v, piece_costs=pieces)
        per_rank = [sum(pieces[c * S + r] for c in range(v)) for r in range(S)]
        base = base or sim["makespan"]
        rows.append({"chunks": v, "bubble_fraction": sim["bubble_fraction"], "relative_step": sim["makespan"] / base,
                     "rank_imbalance": max(per_rank) / (sum(per_rank) / S)})
    return rows


class PipelineTrainer:
    def __init__(self, model: dict, *, num_microbatches: int, schedule: str = "1f1b", optimizer: str = "adam",
                 lr: float = 1e-3, weight_decay: float = 0.0, seed: int = 0, partition: str | list = "balanced",
                 max_inflight: int | None = None, device: str | None = None, init_on_device: bool = True,
                 offload=None, link_probe: bool = False, microbatch_size: int = 1, virtual_stages: int = 1,
                 recompute=None, offload_options: dict | None = None, memory_gb: float | None = None):
        """``partition``: "balanced" (FLOP-balanced DP), "topology_aware" (the planner, with memory
        budgets and NVLink links), "equal", or an explicit list of [start, end) layer ranges.

        ``virtual_stages`` v > 1 runs the interleaved 1F1B program: the model is cut into
        v * world contiguous pieces (FLOP-balanced, or ``partition`` as a list of that many
        ranges) and rank r holds pieces r, r + world, ... (needs ``num_microbatches`` to be a
        multiple of the world size).

        ``recompute``: activation recompute policy (``parallel/recompute.py``: "none", "all",
        "every:K", "largest:N" or a ``RecomputePolicy``); recomputed units keep only their
        input across the step, and the planner and memory estimate count them that way.

        ``offload``: None (optimizer state on the GPU), a ``HostOffload``, or "auto": the
        startup memory estimate (``memory_gb`` per GPU, default this GPU's) decides, and a
        ``HostOffload(**offload_options)`` is made only if the stages do not fit with their
        state resident (``parallel/placement.py``)."""
        self.rank, self.world, self.local_rank = init_distributed()
        self.spec = build_model_spec(model, seed=seed)
        n = self.spec.num_layers
        from meshtrain_b200.parallel.recompute import choose_units

        self.recompute = choose_units(recompute, _profiles(self.spec, microbatch_size)) if recompute else set()
        rc = self.recompute or None
        if isinstance(offload, str):
            from meshtrain_b200.parallel.offload import HostOffload
            from meshtrain_b200.parallel.placement import decide

            def fits_resident() -> bool:
                v_req = max(1, int(virtual_stages)) if self.world > 1 else 1
                try:
                    if v_req > 1 and num_microbatches % self.world == 0:
                        check_interleaved_memory(self.spec, interleaved_split(self._costs(), self.world, v_req),
                                                 self.world, v_req, num_microbatches, microbatch_size, optimizer,
                                                 memory_gb=memory_gb, recompute=rc)
                    else:
                        plan_device_pipeline(self.spec, self.world, num_microbatches, microbatch_size, schedule,
                                             optimizer, max_inflight=max_inflight, memory_gb=memory_gb,
                                             recompute=rc)
                except RuntimeError:
                    return False
                return True

            self.state_tier = decide(offload, fits_resident)
            offload = HostOffload(**(offload_options or {})) if self.state_tier.offload_state else None
        self.plan = None
        self.chunk_ranges = None
        self.memory_estimates = None
        self.virtual_stages = v = max(1, int(virtual_stages))
        if v > 1 and self.world == 1:
            v = self.virtual_stages = 1  # one rank: nothing to interleave
        if v > 1:
            if num_microbatches % self.world:
                raise ValueError(f"{v} virtual stages need num_microbatches ({num_microbatches}) to be a multiple "
                                 f"of the number of ranks ({self.world})")
            if isinstance(partition, list):
                pieces = [tuple(r) for r in partition]
            elif partition == "equal":
                pieces = equal_split(n, v * self.world)
            else:
                pieces = interleaved_split(self._costs(), self.world, v)
            if len(pieces) != v * self.world:
                raise ValueError(f"{len(pieces)} ranges for {v} x {self.world} virtual stages")
            self.chunk_ranges = [pieces[c * self.world + self.rank] for c in range(v)]
            ranges = [tuple(p) for p in pieces]
            if partition in ("topology_aware", "auto"):  # the startup memory estimate, per rank
                self.memory_estimates = check_interleaved_memory(
                    self.spec, ranges, self.world, v, num_microbatches, microbatch_size, optimizer,
                    offload=offload is not None, recompute=rc, memory_gb=memory_gb,
                    offload_ring=offload.ring_settings() if offload is not None else None)
        elif isinstance(partition, list):
            ranges = [tuple(r) for r in partition]
        elif partition == "equal":
            ranges = equal_split(n, self.world)
        elif partition in ("topology_aware", "auto"):
            self.plan = plan_device_pipeline(self.spec, self.world, num_microbatches, microbatch_size, schedule,
                                             optimizer, offload=offload is not None, max_inflight=max_inflight,
                                             recompute=rc, memory_gb=memory_gb,
                                             offload_ring=offload.ring_settings() if offload is not None else None)
            ranges = self.plan.ranges()
        elif partition == "balanced":
            ranges = balanced_split(self._costs(), self.world)
        else:
            raise ValueError(f"unknown partition {partition!r}")
        if v == 1 and len(ranges) != self.world:
            raise ValueError(f"{len(ranges)} stage ranges for {self.world} ranks")
        self.ranges = ranges
        self.stage = self.rank
        if device is None:
            device = f"cuda:{self.local_rank}" if torch.cuda.is_available() else "cpu"
        self.device = torch.device(device)
        links = None
        link_ms = None
        if self.world > 1:
            from meshtrain_b200.parallel.p2p import StageLinks

            links = StageLinks(self.stage, self.world, ring=v > 1)
            if self.device.type == "cuda":
                links.warmup(self.device)
                if link_probe:
                    link_ms = probe_link_ms(links, self.spec.boundary_shape(1), self.spec.dtype, self.device,
                                            scale=microbatch_size)
                    t = torch.tensor([link_ms or 0.0], dtype=torch.float64, device=self.device)
                    dist.all_reduce(t, op=dist.ReduceOp.MAX)
                    link_ms = float(t.item()) or None
        self.links = links
        self.link_ms = link_ms  # probed device time of one microbatch's boundary transfer (informational)
        self.watch = None
        if self.world > 1:
            from meshtrain_b200.parallel.watchdog import PeerWatch

            self.watch = PeerWatch(self.rank, self.world, groups=links.groups(),
                                   timeout_s=float(os.environ.get("MESHTRAIN_PEER_TIMEOUT_S", "60")))
            watch = self.watch
            self._failure_check = lambda: watch.reason  # noqa: E731
        self._engine_kw = dict(stage=self.stage, num_stages=self.world, device=self.device,
                               num_microbatches=num_microbatches, schedule=schedule, max_inflight=max_inflight,
                               optimizer=optimizer, lr=lr, weight_decay=weight_decay, links=links,
                               init_on_device=init_on_device, microbatch_size=microbatch_size, recompute=rc)
        self.engine = PipelineEngine(self.spec, layer_range=None if v > 1 else ranges[self.stage],
                                     chunk_ranges=self.chunk_ranges if v > 1 else None, offload=offload,
                                     **self._engine_kw)
        if self.watch is not None:
            self.engine.failure_check = self._failure_check

    def repartition(self, ranges: list[tuple[int, int]], scratch_root: str | None = None) -> None:
        """Moves to another split of the model between steps (every rank calls this).

        Each rank writes its weights and optimizer state (keyed by global tensor ID)
        to a scratch directory on this node, builds the engine of its new range(s) and
        reads back the tensors of its layers, whoever held them before.  ``ranges`` are
        the pieces in model order: one per rank, or (interleaved layouts) v per rank with
        piece k on rank k mod the number of ranks.  No host offload; the ranks share a
        filesystem (one box).
        """
        import shutil
        import tempfile
        import uuid

        from meshtrain_b200.checkpoint import load_stage_checkpoint, save_stage_checkpoint

        if self.engine.offload is not None:
            raise ValueError("repartition does not move host-offloaded optimizer state")
        v = self.virtual_stages
        ranges = [tuple(r) for r in ranges]
        starts, ends = [a for a, _ in ranges], [b for _, b in ranges]
        if (len(ranges) != self.world * v or starts != [0] + ends[:-1] or ends[-1] != self.spec.num_layers
                or any(a >= b for a, b in ranges)):
            raise ValueError(f"{ranges} is not a contiguous split of {self.spec.num_layers} units into {self.world}")
        if ranges == [tuple(r) for r in self.ranges]:
            return
        base = scratch_root or ("/dev/shm" if os.path.isdir("/dev/shm") else tempfile.gettempdir())
        name = [f"meshtrain-migrate-{uuid.uuid4().hex[:12]}"]
        if self.world > 1:
            dist.broadcast_object_list(name, src=0)  # one directory for every rank
        scratch = os.path.join(base, name[0])
        save_stage_checkpoint(scratch, self.engine, 0)
        self.barrier()
        self.engine = None  # free this rank's old buffers before the new ones are built
        if v > 1:
            self.chunk_ranges = [ranges[c * self.world + self.rank] for c in range(v)]
            self.engine = PipelineEngine(self.spec, layer_range=None, chunk_ranges=self.chunk_ranges, offload=None,
                                         **self._engine_kw)
        else:
            self.engine = PipelineEngine(self.spec, layer_range=ranges[self.stage], offload=None, **self._engine_kw)
        load_stage_checkpoint(scratch, self.engine, 0)
        if self.watch is not None:
            self.engine.failure_check = self._failure_check
        self.ranges = ranges
        self.barrier()
        if self.rank == 0:
            shutil.rmtree(scratch, ignore_errors=True)

    def rebalance(self, stats: list[StepStats], policy=None, busy_ms: float | None = None) -> list:
        """Gathers each rank's measured work per step and lets ``policy`` (default
        ``RebalanceByMeasurement``) propose a better split; carries it out and returns the
        moves ``[(unit, from, to)]`` (empty when the split stays).  ``busy_ms`` overrides
        this rank's measurement (CPU runs have no device timing)."""
        from meshtrain_b200.parallel.migration import RebalanceByMeasurement

        policy = policy or RebalanceByMeasurement()
        mine = busy_ms if busy_ms is not None else (
            sum(s.busy_ms for s in stats) / len(stats) if stats else 0.0)
        everyone = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(everyone, mine)
        else:
            everyone = [mine]
        metrics = {"ranges": self.ranges, "busy_ms": everyone, "unit_costs": self._costs(),
                   "chunks": self.virtual_stages}
        moves = policy.propose(stats[-1].step if stats else 0, metrics)
        if moves:
            self.repartition(policy.last_ranges)
        return moves

    def _costs(self) -> list[float]:
        """Per-unit cost for the FLOP-balanced splits; a recomputed unit runs its forward twice."""
        return [c * (4.0 / 3.0 if u in self.recompute else 1.0) for u, c in enumerate(layer_costs(self.spec))]

    @property
    def is_first(self) -> bool:
        return self.stage == 0

    @property
    def is_last(self) -> bool:
        return self.stage == self.world - 1

    def step(self, step: int, inputs: torch.Tensor | None, targets: torch.Tensor | None,
             timed: bool | str = True) -> StepStats:
        """One global step.  With several ranks a failure anywhere in the pipeline
        raises here (``PeerFailure`` on the ranks that did not fail) instead of
        leaving the survivors blocked in NCCL."""
        if self.watch is not None:
            self.watch.check()
        try:
            stats = self.engine.train_step(step, inputs if self.is_first else None,
                                           targets if self.is_last else None, timed=timed)
        except Exception as exc:
            if self.watch is not None:
                from meshtrain_b200.parallel.watchdog import PeerFailure

                peer = self.watch.peer_failure()
                if peer is not None:  # this rank failed because a peer did
                    raise PeerFailure(peer) from exc
                self.watch.report(f"step {step}: {type(exc).__name__}: {exc}")
            raise
        if self.watch is not None:
            self.watch.beat(step)
        return stats

    def finish_timing(self, stats: list[StepStats]) -> list[StepStats]:
        """Device timing of steps run with ``timed="deferred"`` (waits for them)."""
        for st in stats:
            self.engine.finish_timing(st)
        return stats

    def p2p_report(self, stats: list[StepStats]) -> dict:
        """Exposed p2p time and bubble of the given (timed) steps, measured on every rank.

        A rank's compute stream stalls before a receive until the message is
        there.  The stall is split into the message's transfer time (the
        sender's NCCL send time, measured on the sender's GPU) and the wait for
        the sender to produce it (pipeline dependency): exposed p2p of a
        receive is min(stall, transfer).  Every rank contributes its stalls and
        its send times (one object all-gather); the result holds the per-step
        mean of each rank and the max over ranks.  Also fills
        ``exposed_p2p_ms`` of this rank's ``stats``.
        """
        mine = [{"wait": s.recv_wait_ms, "send": s.send_ms, "bubble": s.bubble_fraction,
                 "parts": (s.step_ms, s.forward_ms, s.backward_ms, s.optimizer_ms, s.side_ms, s.wait_ms, s.busy_ms)}
                for s in stats]
        if self.world > 1:
            everyone: list = [None] * self.world
            dist.all_gather_object(everyone, mine)
        else:
            everyone = [mine]
        exposed = []
        for rank, steps in enumerate(everyone):
            per_step = []
            for i, rec in enumerate(steps):
                total = 0.0
                for key, stall in rec["wait"].items():
                    if "/" in key:  # "<F|B><mb>/<k>": boundary k between virtual stages k and k+1
                        k = int(key.split("/")[1])
                        sender = (k if key[0] == "F" else k + 1) % self.world
                    else:
                        sender = rank - 1 if key[0] == "F" else rank + 1
                    transfer = everyone[sender][i]["send"].get(key) if 0 <= sender < self.world else None
                    if transfer is not None:
                        total += min(stall, transfer)
                per_step.append(total)
            exposed.append(per_step)
        for st, ms in zip(stats, exposed[self.rank]):
            st.exposed_p2p_ms = ms
        n = max(1, len(stats))
        mean = lambda xs: sum(xs) / n  # noqa: E731
        return {"exposed_p2p_ms_per_step": max(mean(e) for e in exposed),
                "exposed_p2p_ms_by_rank": [round(mean(e), 4) for e in exposed],
                "bubble_fraction": max(mean([r["bubble"] for r in steps]) for steps in everyone),
                "bubble_by_rank": [round(mean([r["bubble"] for r in steps]), 4) for steps in everyone],
                "wait_ms_per_step": max(mean([sum(r["wait"].values()) for r in steps]) for steps in everyone),
                # per rank, mean over the steps: where the step's time goes on that stage
                "stage_ms": [{name: round(mean([r["parts"][i] for r in steps]), 3) for i, name in enumerate(
                    ("step", "forward", "backward", "optimizer", "side_stream", "recv_wait", "busy"))}
                    for steps in everyone]}

    def loss_value(self, stats: StepStats) -> float | None:
        """Mean loss of the step (device -> host read); None off the last stage."""
        if stats.loss is None:
            return None
        if stats.loss_ready is not None:
            self.engine.wait_event(stats.loss_ready)
        return float(stats.loss) / self.engine.M

    def barrier(self) -> None:
        if self.world > 1:
            dist.barrier(device_ids=[self.local_rank] if self.device.type == "cuda" else None)

    def allreduce_max(self, value: float) -> float:
        if self.world == 1:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self) -> None:
        failed = self.watch is not None and self.watch.reason is not None
        if self.watch is not None:
            self.watch.close()
        if self.world > 1 and dist.is_initialized():
            if failed:
                # The peers of a failed pipeline will not reach a barrier, and NCCL work
                # toward a dead peer never completes, so destroying the groups could block:
                # they are left to end with the process.
                self.watch.abandon_groups()
                return
            try:
                self.barrier()
            finally:
                dist.destroy_process_group()


def probe_link_ms(links, shape_one, dtype, device, scale: int = 1, iters: int = 5) -> float | None:
    """Device time of one boundary-sized p2p transfer between adjacent stages (a link probe)."""
    shape = (shape_one[0] * scale, *shape_one[1:])
    buf = torch.zeros(shape, dtype=dtype, device=device)
    times = []
    for _ in range(iters):
        for s in range(links.num_stages - 1):
            if links.stage == s:
                st = torch.cuda.Event(enable_timing=True)
                en = torch.cuda.Event(enable_timing=True)
                st.record()
                links.send_activation(buf).wait()
                en.record()
                en.synchronize()
                times.append(st.elapsed_time(en))
            elif links.stage == s + 1:
                links.recv_activation(buf).wait()
                torch.cuda.synchronize(device)
    links.reset_stats()
    return min(times) if times else None
