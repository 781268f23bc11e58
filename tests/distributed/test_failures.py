"""Failures end cleanly: no hangs, errors that say what happened.

Everything here fails on the host: a silent or vanished peer, a stage that
raises, a rank that exits between steps.  Nothing faults or hangs a device.
"""

import threading
import time

import pytest

from meshtrain_b200.models import build_model_spec
from meshtrain_b200.networking.tcp import TCPListener, connect
from meshtrain_b200.parallel.pipeline import PipelineError, PipelineSettings, run_stage
from meshtrain_b200.parallel.spawn import spawn_ranks
from meshtrain_b200.parallel.stage import Stage
from meshtrain_b200.telemetry import EventLogger


class WirePair:
    """Both ends of one framed TCP connection on loopback (``ours`` for the stage under test)."""

    def __init__(self):
        listener = TCPListener("127.0.0.1", 0)
        accepted = []
        acceptor = threading.Thread(target=lambda: accepted.append(listener.accept(timeout=5)[0]))
        acceptor.start()
        self.ours = connect("127.0.0.1", listener.port, timeout=5, hello={"job_id": "f"})
        acceptor.join()
        listener.close()
        self.theirs = accepted[0]


MLP = build_model_spec({"type": "mlp"})


def _run_first_stage(downstream, timeout_s: float, steps: int = 1, stop_event=None):
    stage = Stage(MLP.build_stage(0, 3), stage_index=0, num_stages=2)
    run_stage(stage, MLP, PipelineSettings("f", steps=steps, batch_size=8, timeout_s=timeout_s),
              upstream=None, downstream=downstream, logger=EventLogger("w0", "f"), stop_event=stop_event)


# (scenario, how the neighbour misbehaves, stage timeout, expected message, seconds allowed)
SCENARIOS = [
    ("silent-peer", lambda wire, stop: None, 1.0, "stalled", 6.0),
    ("peer-disconnects", lambda wire, stop: threading.Timer(0.5, wire.theirs.close).start(), 30.0,
     "disconnected|failed", 6.0),
    ("stop-requested", lambda wire, stop: threading.Timer(0.3, stop.set).start(), 30.0, "stopped", 6.0),
]


@pytest.mark.parametrize("name,misbehave,timeout_s,message,allowed_s", SCENARIOS, ids=[s[0] for s in SCENARIOS])
def test_first_stage_ends_with_a_clear_error(name, misbehave, timeout_s, message, allowed_s):
    wire, stop = WirePair(), threading.Event()
    misbehave(wire, stop)
    began = time.monotonic()
    with pytest.raises(PipelineError, match=message) as failure:
        _run_first_stage(wire.ours, timeout_s, steps=5, stop_event=stop)
    assert time.monotonic() - began < allowed_s, f"{name}: no full-timeout wait"
    if name == "silent-peer":
        assert "state" in str(failure.value)  # the stall report dumps the stage's protocol state
    wire.theirs.close()


def test_a_failing_neighbour_stops_this_stage_through_its_error_packet():
    wire = WirePair()
    settings = PipelineSettings("f", steps=1, batch_size=8, timeout_s=30.0)
    seen = {}

    def misconfigured_last_stage():
        # layer 6 expects the MLP's narrow width and gets the wide activation: its forward raises
        stage = Stage(MLP.build_stage(6, 7), stage_index=1, num_stages=2, loss_fn=MLP.loss_fn)
        try:
            run_stage(stage, MLP, settings, upstream=wire.theirs, downstream=None, logger=EventLogger("w1", "f"))
        except Exception as exc:  # noqa: BLE001 - the failure this test provokes
            seen["error"] = exc

    neighbour = threading.Thread(target=misconfigured_last_stage)
    neighbour.start()
    with pytest.raises(PipelineError, match="peer reported error"):
        _run_first_stage(wire.ours, 30.0)
    neighbour.join(5)
    assert not neighbour.is_alive() and "error" in seen


def _engine_rank_that_leaves(steps_before_exit: int):
    """Device-engine ranks on gloo; the last rank leaves between steps, the others must error out."""
    import datetime
    import os

    import torch.distributed as dist

    from meshtrain_b200.api import PipelineTrainer

    rank = int(os.environ["RANK"])
    dist.init_process_group("gloo", rank=rank, world_size=int(os.environ["WORLD_SIZE"]),
                            timeout=datetime.timedelta(seconds=5))
    tr = PipelineTrainer({"type": "gpt", "layers": 2, "hidden_size": 64, "heads": 4, "vocab_size": 96,
                          "seq_len": 32}, num_microbatches=2, device="cpu", microbatch_size=2, partition="equal")
    done = 0
    try:
        for step in range(10):
            if rank == tr.world - 1 and step == steps_before_exit:
                return {"rank": rank, "left_after": done}
            x, y = tr.spec.make_batch(step, 4)
            tr.step(step, x, y)
            done += 1
    except Exception as exc:  # noqa: BLE001 - the survivor reports what it saw
        return {"rank": rank, "error": f"{type(exc).__name__}: {exc}"[:300], "done": done}
    return {"rank": rank, "done": done}


def test_rank_leaving_between_steps_surfaces_on_the_others():
    t0 = time.monotonic()
    out = spawn_ranks(_engine_rank_that_leaves, 2, 2, timeout_s=120)
    assert out[1] == {"rank": 1, "left_after": 2}
    assert "error" in out[0] and out[0]["done"] == 2, out[0]
    assert time.monotonic() - t0 < 90
