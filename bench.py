#!/usr/bin/env python
"""Pipeline-parallel training throughput: tokens/s at N stages on N GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--model gpt-0.48b]
    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N ...

Workload (default ``gpt-0.48b``): GPT decoder, d_model 1280, 24 layers, 20
heads, MLP 5120, vocab 50257, seq 2048, pre-LN, GELU, bf16; 32 microbatches
of 4 sequences per step (global batch 128 = 262,144 tokens), 1F1B, Adam;
uniform random tokens with shifted targets, random N(0, 0.02) init.  One
stage per GPU, layers split by the cost-balanced planner.  The same global
batch is used at every N (strong scaling).

Timing: W untimed warm-up steps, then K steps bracketed by barrier +
cuda.synchronize, CUDA events on each rank, max over ranks.  Weights and
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
BASELINE_PUBLISHED = None  # no tokens/s figure is published for the reference


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
    trainer = PipelineTrainer(model, num_microbatches=M, schedule=args.schedule, optimizer="adam", lr=1e-4,
                              microbatch_size=mbs)
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
        stats.append(trainer.step(s, *batches[s], timed=False))
    ev1.record()
    torch.cuda.synchronize()
    launches = ops.launches() - l0
    trainer.barrier()
    clocks = sampler.stop() if sampler else None
    dev_ms = ev0.elapsed_time(ev1)
    ms_max = trainer.allreduce_max(dev_ms)
    launches_max = int(trainer.allreduce_max(float(launches)))
    last_loss = trainer.loss_value(stats[-1]) if trainer.is_last else None

    # per-step breakdown (bubble, exposed p2p) from one extra instrumented step
    st = trainer.step(total_steps - 1, *batches[-1], timed=True)
    bubble = trainer.allreduce_max(st.bubble_fraction)
    exposed = trainer.allreduce_max(st.exposed_p2p_ms)
    wait = trainer.allreduce_max(st.wait_ms)

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
        "vs_baseline": (value / BASELINE_PUBLISHED) if BASELINE_PUBLISHED else None,
        "dtype": "bf16",
        "data": "synthetic (uniform random tokens, shifted targets; random N(0,0.02) init)",
        "impl": "ours",
        "config": {
            "model": f"{args.model} (d{spec.d_model} L{spec.n_blocks} H{spec.n_heads} V{spec.vocab_size} S{seq})",
            "global_batch": batch, "seq_len": seq, "microbatches": M, "microbatch_size": mbs,
            "parallelism": f"pp{world}", "schedule": args.schedule, "stage_layers": trainer.ranges,
            "l2": "working set (weights + activations, GBs per stage) >> 126 MB L2; no flush needed",
        },
        "bubble_pct": round(100 * bubble, 2),
        "exposed_p2p_ms_per_step": round(exposed, 3),
        "wait_ms_per_step": round(wait, 3),
        "loss": round(float(loss_t[0]), 5),
        "kernel_status": status,
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d_t + y_bytes),
                "d2h_bytes_per_step": 4, "loss": round(float(loss_t[1]), 5)},
        "gpu_launches": launches_max,
        "clocks": clocks,
    }
    if spec.flops_per_token:
        record["model_tflops_per_gpu"] = round(spec.flops_per_token() * value / world / 1e12, 1)
    emit(rank, record)
    trainer.close()


def bench_reference(args) -> None:
    """Unmodified reference (baseline/_ref) through its public Stage/run_stage API."""
    ref = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "meshtrain")):
        emit(int(os.environ.get("RANK", "0")), {"impl": "reference",
                                               "unavailable": "reference not installed under baseline/_ref"})
        return
    sys.path.insert(0, ref)
    from meshtrain_b200 import reference_arm

    reference_arm.run(args, MODELS)


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
