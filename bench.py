#!/usr/bin/env python
"""Pipeline-parallel training throughput: tokens/s at N stages on N GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--model gpt-0.48b]
    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N ...

Workload (default ``gpt-0.48b``): GPT decoder, d_model 1280, 24 layers, 20
heads, MLP 5120, vocab 50257, seq 2048, pre-LN, GELU, bf16; 32 microbatches
of 4 sequences per step (global batch 128 = 262,144 tokens), 1F1B, Adam;
uniform random tokens with shifted targets, random N(0, 0.02) init.  One
stage per GPU, split by the topology-aware planner; a stage boundary may fall
between a block's attention and MLP halves (``--units blocks`` keeps whole
blocks).  The same global
batch is used at every N (strong scaling).

Timing: W untimed warm-up steps, then K steps bracketed by barrier +
cuda.synchronize, CUDA events on each rank, max over ranks.  Bubble and
exposed p2p come from the timed steps' own events on every rank: the bubble
is the step time not covered by compute-stream actions, the optimizer or the
side-stream weight-gradient GEMMs; exposed p2p is, per received message, the
part of the compute stream's stall that the sender's measured NCCL send time
explains.  Weights and
activations (several GB per stage) far exceed the 126 MB L2, so no flush is
needed between steps.  ``e2e`` repeats K steps through the public
``PipelineTrainer.step`` API with the step's token ids / targets copied from
pinned host memory and the loss read back to the host every step.

``--impl reference`` runs the unmodified reference (installed under
baseline/_ref) through its own ``Stage`` + ``run_stage`` API on the same
model shape, one stage per GPU with its TCP transport between stages.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

HERE = os.path.dirname(os.path.abspath(__file__))

MODELS = {
    # name: (model dict, microbatches, microbatch size)
    "gpt-0.48b": (dict(type="gpt", layers=24, hidden_size=1280, heads=20, vocab_size=50257, seq_len=2048,
                       dtype="bfloat16", init_std=0.02, data="uniform"), 32, 4),
    "gpt-0.4b": (dict(type="gpt", layers=24, hidden_size=1024, heads=16, vocab_size=50257, seq_len=1024,
                      dtype="bfloat16", init_std=0.02, data="uniform"), 8, 4),
    "llama-8b": (dict(type="llama", layers=32, hidden_size=4096, heads=32, n_kv_heads=8, ffn_hidden=14336,
                      vocab_size=128256, seq_len=4096, rope_theta=500000.0, dtype="bfloat16", init_std=0.02,
                      data="uniform"), 64, 1),
    "gpt-tiny": (dict(type="gpt", layers=4, hidden_size=256, heads=4, vocab_size=1024, seq_len=256,
                      dtype="bfloat16", init_std=0.02, data="uniform"), 4, 2),
}
PUBLISHED_TOKENS_PER_S = None  # no tokens/s figure is published for the reference


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]):
        self.gpus = gpus
        self.proc = None
        self.out = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.out, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.flush()
        self.out.seek(0)
        sm, mx, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if idx not in self.gpus:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                pass
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.out.name)
        busy = [s for s in sm if s > 0.5 * (max(mx) if mx else 1)] or sm
        return {"sm_mhz": statistics.median(busy) if busy else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


def emit(rank: int, record: dict) -> None:
    if rank == 0:
        print(json.dumps(record), flush=True)


def bench_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from meshtrain_b200 import ops
    from meshtrain_b200.api import PipelineTrainer

    model, M, mbs = MODELS[args.model]
    if args.microbatches:
        M = args.microbatches
    if args.microbatch_size:
        mbs = args.microbatch_size
    batch = M * mbs
    offload = None
    if args.offload:
        from meshtrain_b200.parallel.offload import HostOffload

        offload = HostOffload(prefetch_ahead=1, chunk_mb=256, device_budget_gb=args.offload_budget_gb)
    units = dict(model, split_blocks=True) if args.units == "half-blocks" else model
    if args.virtual_stages is None:
        world_env = int(os.environ.get("WORLD_SIZE", "1"))
        args.virtual_stages = 2 if world_env > 1 and M % world_env == 0 else 1
    trainer = PipelineTrainer(units, num_microbatches=M, schedule=args.schedule, optimizer="adam", lr=1e-4,
                              microbatch_size=mbs, partition=args.partition, offload=offload,
                              virtual_stages=args.virtual_stages, recompute=args.recompute)
    rank, world = trainer.rank, trainer.world
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    spec = trainer.spec
    seq = spec.seq_len
    tokens_per_step = batch * seq
    total_steps = args.warmup + 2 * args.steps
    pin = torch.cuda.is_available()
    batches = []
    for s in range(total_steps):
        x, y = spec.make_batch(s, batch)
        batches.append((x.pin_memory() if pin else x, y.pin_memory() if pin else y))

    # warm-up
    for s in range(args.warmup):
        trainer.step(s, *batches[s], timed=False)
    torch.cuda.synchronize()
    status = ops.read_status(trainer.local_rank) if ops.extension_available() else 0
    torch.cuda.reset_peak_memory_stats(trainer.device)  # the timed steps' peak, reported below

    # device-timed region
    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    trainer.barrier()
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
    l0 = ops.launches()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    stats = []
    for s in range(args.warmup, args.warmup + args.steps):
        # the steps' own CUDA events give their bubble and per-message stalls; they are read
        # after the timed region, so the host never waits between steps
        stats.append(trainer.step(s, *batches[s], timed="deferred"))
    ev1.record()
    torch.cuda.synchronize()
    trainer.finish_timing(stats)
    launches = ops.launches() - l0
    peak_gb = trainer.allreduce_max(torch.cuda.max_memory_allocated(trainer.device) / 1024 ** 3)
    trainer.barrier()
    clocks = sampler.stop() if sampler else None
    dev_ms = ev0.elapsed_time(ev1)
    ms_max = trainer.allreduce_max(dev_ms)
    launches_max = int(trainer.allreduce_max(float(launches)))
    last_loss = trainer.loss_value(stats[-1]) if trainer.is_last else None

    # bubble and exposed p2p of the timed steps, measured on every rank (max over ranks)
    p2p = trainer.p2p_report(stats)
    bubble, exposed, wait = p2p["bubble_fraction"], p2p["exposed_p2p_ms_per_step"], p2p["wait_ms_per_step"]

    # end-to-end through the public API: H2D of inputs each step + loss D2H each step
    trainer.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_loss = None
    for s in range(args.warmup + args.steps, args.warmup + 2 * args.steps):
        st2 = trainer.step(s, *batches[s], timed=False)
        if trainer.is_last:
            e2e_loss = trainer.loss_value(st2)  # device -> host read of the step's loss
    torch.cuda.synchronize()
    e2e_s = trainer.allreduce_max(time.perf_counter() - t0)
    if trainer.is_last and last_loss is not None:
        loss_t = torch.tensor([last_loss, e2e_loss or 0.0], dtype=torch.float64, device=trainer.device)
    else:
        loss_t = torch.zeros(2, dtype=torch.float64, device=trainer.device)
    if world > 1:
        dist.all_reduce(loss_t, op=dist.ReduceOp.SUM)
    status |= ops.read_status(trainer.local_rank) if ops.extension_available() else 0
    status = int(trainer.allreduce_max(float(status)))

    ms_per_step = ms_max / args.steps
    value = tokens_per_step / (ms_per_step / 1e3)
    e2e_value = tokens_per_step * args.steps / e2e_s
    h2d = 0
    if trainer.is_first:
        h2d += batches[0][0].numel() * batches[0][0].element_size()
    h2d_t = trainer.allreduce_max(float(h2d))
    y_bytes = batches[0][1].numel() * batches[0][1].element_size()
    record = {
        "metric": "tokens/sec (device-timed, max over ranks)",
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": (value / PUBLISHED_TOKENS_PER_S) if PUBLISHED_TOKENS_PER_S else None,
        "dtype": "bf16",
        "data": "synthetic (uniform random tokens, shifted targets; random N(0,0.02) init)",
        "impl": "ours",
        "config": {
            "model": f"{args.model} (d{spec.d_model} L{spec.n_blocks} H{spec.n_heads} V{spec.vocab_size} S{seq})",
            "global_batch": batch, "seq_len": seq, "microbatches": M, "microbatch_size": mbs,
            "parallelism": f"pp{world}", "stage_layers": trainer.ranges,
            "schedule": (args.schedule if trainer.virtual_stages == 1 else
                         f"{args.schedule} interleaved, {trainer.virtual_stages} model chunks per GPU"),
            "partition": (args.partition if trainer.virtual_stages == 1 else
                          "pieces contiguous and FLOP-weighted, each rank's sum of pieces balanced"),
            "partition_units": args.units,
            "offload": "fp32 master + Adam moments in pinned host DRAM, streamed" if args.offload else None,
            **({"activation_recompute": f"{args.recompute} ({len(trainer.recompute)} units)"}
               if args.recompute != "none" else {}),
            "l2": "working set (weights + activations, GBs per stage) >> 126 MB L2; no flush needed",
        },
        "peak_device_memory_gib": round(peak_gb, 2),  # allocated by the timed steps, max over ranks
        "bubble_pct": round(100 * bubble, 2),
        "bubble_pct_by_stage": [round(100 * b, 2) for b in p2p["bubble_by_rank"]],
        "exposed_p2p_ms_per_step": round(exposed, 3),
        "exposed_p2p_ms_by_stage": p2p["exposed_p2p_ms_by_rank"],
        "wait_ms_per_step": round(wait, 3),
        "p2p_method": "per receive: min(compute-stream stall, sender's NCCL send time); mean over the timed steps",
        "stage_ms": p2p["stage_ms"],
        "loss": round(float(loss_t[0]), 5),
        "kernel_status": status,
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d_t + y_bytes),
                "d2h_bytes_per_step": 4, "loss": round(float(loss_t[1]), 5)},
        "gpu_launches": launches_max,
        "clocks": clocks,
    }
    if offload is not None:
        opt_ms = trainer.allreduce_max(sum(st.optimizer_ms for st in stats) / len(stats))
        moved = trainer.allreduce_max(float(offload.stats["h2d_bytes"]) / max(1, offload.stats["steps"]))
        record["offload"] = {
            "device_budget_gb": args.offload_budget_gb, "slots": offload.nslots, "chunks": len(offload.chunks),
            "resident_fraction": round(offload.resident_fraction(), 3),
            "h2d_gb_per_step": round(moved / 1e9, 3), "d2h_gb_per_step": round(moved / 1e9, 3),
            "optimizer_ms_per_step_max_rank": round(opt_ms, 2),
        }
    if spec.flops_per_token:
        record["model_tflops_per_gpu"] = round(spec.flops_per_token() * value / world / 1e12, 1)
    emit(rank, record)
    trainer.close()


def reference_stage_ranges(spec, world: int, microbatches: int, microbatch_size: int, dtype: str) -> list:
    """Stage layer ranges from the reference's own planner.

    The reference profiles its layers on the meta device (planner/graph.py
    ``profile_model``) and splits them with its ``compute`` strategy
    (planner/partition.py ``plan_compute``): contiguous ranges whose FLOP
    shares match the workers' measured FLOP/s, here N identical GPUs.  Only
    reference code runs; the workers are described to it as N equal CUDA
    devices of 180 GB.
    """
    if world == 1:
        return [(0, spec.num_layers)]
    from meshtrain.planner.graph import profile_model
    from meshtrain.planner.partition import PlannerOptions, WorkerProfile, make_plan

    layers = profile_model(spec, microbatch_size)
    workers = [WorkerProfile(worker_id=f"gpu{i}", name=f"gpu{i}", backend="cuda", memory_total=180 * 10 ** 9,
                             measured_flops=1.0e15) for i in range(world)]
    opts = PlannerOptions(optimizer="adam", num_microbatches=microbatches, dtype=dtype, num_stages=world,
                          schedule="1f1b")
    plan = make_plan("compute", layers, workers, opts=opts)
    return [(st.start, st.end) for st in plan.stages]


def bench_reference(args) -> None:
    """Unmodified reference (baseline/_ref) through its public Stage / run_stage API.

    Every rank builds its layer range with the reference's model spec, runs the
    reference's Stage (its torch modules and optimizer) and run_stage (its
    schedules, outbox and TCP transport over loopback between adjacent ranks).
    Only the launch glue (port exchange, barriers, CUDA-event timing) is ours.
    """
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    base = os.path.join(HERE, "baseline", "_ref")
    # `pip install --target baseline/_ref` puts the package at baseline/_ref/meshtrain;
    # a plain copy of the source tree has it at baseline/_ref/src/meshtrain.
    candidates = [base, os.path.join(base, "src")]
    ref = next((c for c in candidates if os.path.isfile(os.path.join(c, "meshtrain", "runtime", "pipeline.py"))),
               None)
    if ref is None:
        checked = " and ".join(os.path.join(c, "meshtrain") for c in candidates)
        emit(rank, {"impl": "reference", "unavailable": f"reference package not found (checked {checked})"})
        return
    sys.path.insert(0, ref)
    os.environ.setdefault("MESHTRAIN_QUIET", "1")
    import datetime

    import torch
    import torch.distributed as dist

    from meshtrain.models import build_model_spec as ref_build_spec
    from meshtrain.runtime.pipeline import PipelineSettings, run_stage
    from meshtrain.runtime.stage import Stage
    from meshtrain.worker.device import CUDADeviceAdapter

    model, M, mbs = MODELS[args.model]
    if args.microbatches:
        M = args.microbatches
    if args.microbatch_size:
        mbs = args.microbatch_size
    if model["type"] not in ("gpt", "tiny_transformer"):
        emit(rank, {"impl": "reference", "unavailable": f"reference has no {model['type']} model type"})
        return
    batch = M * mbs
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=900))
    # The reference's TCP receive path (networking/tcp.py:85, Tensor.numpy() on the
    # receive buffer) cannot carry bfloat16 payloads, so its stock multi-stage path
    # fails in bf16; with more than one stage it runs in float16 (same width and
    # tensor-core rate), the closest dtype its unmodified transport can carry.
    ref_dtype = model["dtype"] if world == 1 or model["dtype"] != "bfloat16" else "float16"
    cfg = {"type": "tiny_transformer", "layers": model["layers"], "hidden_size": model["hidden_size"],
           "heads": model["heads"], "vocab_size": model["vocab_size"], "seq_len": model["seq_len"],
           "dtype": ref_dtype}
    spec = ref_build_spec(cfg, seed=0)
    ranges = reference_stage_ranges(spec, world, M, mbs, ref_dtype)
    start, end = ranges[rank]
    if cuda:
        dev = CUDADeviceAdapter(local)
    else:  # CPU-only host (harness checks): the reference's own CPU adapter
        from meshtrain.worker.device import CPUDeviceAdapter

        dev = CPUDeviceAdapter()
    stage = Stage(spec.build_stage(start, end), stage_index=rank, num_stages=world, device=dev, optimizer="adam",
                  lr=1e-4, loss_fn=spec.loss_fn, name=f"ref{rank}", layer_offset=start)
    up = down = None
    if world > 1:
        from meshtrain.networking.tcp import TCPListener, connect

        store = dist.distributed_c10d._get_default_store()
        listener = None
        if rank > 0:
            listener = TCPListener("127.0.0.1", 0)
            store.set(f"refport{rank}", str(listener.port))
        if rank < world - 1:
            store.wait([f"refport{rank + 1}"], datetime.timedelta(seconds=300))
            port = int(store.get(f"refport{rank + 1}").decode())
            down = connect("127.0.0.1", port, timeout=300, hello={"job_id": "bench", "stage": rank})
        if listener is not None:
            up, _ = listener.accept(timeout=300)
            listener.close()

    def settings(steps, offset):
        return PipelineSettings(job_id="bench", steps=steps, batch_size=batch, num_microbatches=M, timeout_s=600,
                                log_every=10 ** 9, step_offset=offset, schedule=args.schedule, async_transport=True,
                                trace=False)

    def barrier():
        if world > 1:
            dist.barrier()

    run_stage(stage, spec, settings(args.warmup, 0), upstream=up, downstream=down, worker=f"ref{rank}")
    barrier()
    time.sleep(1.0)  # the previous run's link reader threads poll every 0.2 s before exiting
    barrier()
    if cuda:
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
    t0 = time.perf_counter()
    res = run_stage(stage, spec, settings(args.steps, args.warmup), upstream=up, downstream=down,
                    worker=f"ref{rank}")
    if cuda:
        ev1.record()
        torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    dev_ms = ev0.elapsed_time(ev1) if cuda else wall * 1e3
    # only stage 0 records the step's mean loss (reference runtime/pipeline.py:424-427)
    vals = torch.tensor([dev_ms, wall, res.losses[-1] if res.losses else -math.inf], dtype=torch.float64)
    if world > 1:
        mx = vals.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        vals = mx
    for link in (up, down):
        if link is not None:
            link.close()
    tokens = batch * model["seq_len"]
    ms_per_step = float(vals[0]) / args.steps
    record = {
        "impl": "reference",
        "metric": "tokens/sec (device-timed, max over ranks)",
        "value": round(tokens / (ms_per_step / 1e3), 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": {"bfloat16": "bf16", "float16": "fp16", "float32": "fp32"}[ref_dtype],
        "dtype_note": (None if ref_dtype == model["dtype"] else
                       "reference TCP transport cannot receive bfloat16 (networking/tcp.py:85); ran float16"),
        "data": "synthetic (reference arithmetic-sequence generator; PyTorch default init)",
        "config": {"model": f"{args.model} as reference tiny_transformer (d{model['hidden_size']} L{model['layers']} "
                            f"H{model['heads']} V{model['vocab_size']} S{model['seq_len']})",
                   "global_batch": batch, "seq_len": model["seq_len"], "microbatches": M,
                   "parallelism": f"pp{world}", "schedule": args.schedule, "stage_layers": ranges,
                   "partition": "reference planner, compute strategy" if world > 1 else "one stage",
                   "transport": "reference TCP over loopback" if world > 1 else "none (one stage)"},
        "e2e": {"value": round(tokens * args.steps / float(vals[1]), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": batch * model["seq_len"] * 8 * 2, "d2h_bytes_per_step": 4 * M},
        "loss": round(float(vals[2]), 5) if math.isfinite(float(vals[2])) else None,
    }
    if not math.isfinite(float(vals[2])):
        # torch.optim.Adam on float16 parameters keeps float16 moments; its eps (1e-8)
        # rounds to 0 in float16, so a parameter whose gradient is exactly 0 (an unused
        # embedding row) gets 0/0 in its first update and the loss turns NaN.  The
        # same kernels run at the same speed on NaN data, so the timing still stands.
        record["loss_note"] = "NaN: the reference's float16 Adam state (eps 1e-8 underflows to 0 in float16)"
    emit(rank, record)
    if world > 1:
        dist.destroy_process_group()


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", choices=sorted(MODELS), default="gpt-0.48b")
    ap.add_argument("--schedule", choices=["1f1b", "gpipe"], default="1f1b")
    ap.add_argument("--microbatches", type=int, default=None)
    ap.add_argument("--microbatch-size", type=int, default=None)
    ap.add_argument("--virtual-stages", type=int, default=None,
                    help="model chunks per GPU (interleaved 1F1B; 1 = plain 1F1B). Default: 2 when there is more "
                         "than one GPU and the microbatch count is a multiple of it (measured faster at 2, 4 and "
                         "8 GPUs), else 1")
    ap.add_argument("--offload", action="store_true", help="master weights + Adam moments in pinned host DRAM")
    ap.add_argument("--offload-budget-gb", type=float, default=16.0,
                    help="device memory for the offload slot ring (chunks prefetched during forward/backward)")
    ap.add_argument("--partition", choices=["topology_aware", "balanced", "equal"], default="topology_aware")
    ap.add_argument("--recompute", default="none",
                    help="activation recompute: none, all, every:K, largest:N (units keep only their input; "
                         "their forward runs again in backward)")
    ap.add_argument("--units", choices=["half-blocks", "blocks"], default="half-blocks",
                    help="partition units: a stage boundary may fall between a block's attention and MLP halves")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps; the timing is not a valid bench number", file=sys.stderr)
    if args.impl == "reference":
        bench_reference(args)
    else:
        bench_ours(args)


if __name__ == "__main__":
    sys.path.insert(0, HERE)
    main()
