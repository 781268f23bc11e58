"""Run a function on N local ranks (one spawned process each) with torch.distributed initialised.

Used by the CPU (``gloo``) multi-rank tests, ``meshtrain train --local`` for the
device engine, and experiments.  Each rank gets RANK / WORLD_SIZE / LOCAL_RANK /
MASTER_ADDR=127.0.0.1 / MASTER_PORT in its environment; the target's return
value (picklable) comes back in rank order.  A rank that raises fails the whole
call with its traceback; a rank that never reports ends the call at
``timeout_s``.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import pickle
import queue
import socket
import traceback


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, env, target, args, kwargs, results):
    os.environ.update(env)
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    try:
        # plain pickle: tensors travel by value, not as shared-memory handles that die with the rank
        results.put((rank, "ok", pickle.dumps(target(*args, **kwargs))))
    except BaseException as exc:  # noqa: BLE001 - reported to the parent
        results.put((rank, "error", f"{type(exc).__name__}: {exc}\n{traceback.format_exc()}"))
    finally:
        try:
            import torch.distributed as dist

            from meshtrain_b200.parallel.watchdog import groups_abandoned

            if dist.is_initialized() and not groups_abandoned():
                dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def spawn_ranks(target, world: int, *args, timeout_s: float = 300.0, env: dict | None = None, **kwargs) -> list:
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = free_port()
    base_env = {"PYTHONPATH": os.pathsep.join(filter(None, [os.path.dirname(os.path.dirname(os.path.dirname(
        os.path.abspath(__file__)))), os.environ.get("PYTHONPATH", "")]))}
    base_env.update(env or {})
    procs = [ctx.Process(target=_entry, args=(r, world, port, base_env, target, args, kwargs, results),
                         name=f"meshtrain-rank{r}") for r in range(world)]
    for p in procs:
        p.start()
    out: dict[int, object] = {}
    errors: dict[int, str] = {}
    try:
        while len(out) + len(errors) < world:
            try:
                rank, kind, payload = results.get(timeout=timeout_s)
            except queue.Empty:
                missing = sorted(set(range(world)) - set(out) - set(errors))
                raise TimeoutError(f"ranks {missing} reported nothing within {timeout_s}s") from None
            if kind == "ok":
                out[rank] = pickle.loads(payload)
            else:
                errors[rank] = payload
            if errors:
                break  # the other ranks will block on the failed one; stop waiting for them
    finally:
        for p in procs:
            p.join(timeout=5 if errors else 30)
            if p.is_alive():
                p.terminate()
                p.join(timeout=5)
    if errors:
        raise RuntimeError("rank failure:\n" + "\n".join(f"rank {r}: {e}" for r, e in sorted(errors.items())))
    return [out[r] for r in range(world)]
