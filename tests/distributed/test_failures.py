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


def _link_pair():
    lis = TCPListener("127.0.0.1", 0)
    box = {}
    th = threading.Thread(target=lambda: box.update(s=lis.accept(timeout=5)))
    th.start()
    c = connect("127.0.0.1", lis.port, timeout=5, hello={"job_id": "f"})
    th.join()
    lis.close()
    return c, box["s"][0]


def _first_stage(spec):
    return Stage(spec.build_stage(0, 3), stage_index=0, num_stages=2)


def test_silent_peer_times_out_with_state_dump():
    spec = build_model_spec({"type": "mlp"})
    down, peer = _link_pair()
    t0 = time.monotonic()
    with pytest.raises(PipelineError, match="stalled") as ei:
        run_stage(_first_stage(spec), spec, PipelineSettings("f", steps=1, batch_size=8, timeout_s=1.0),
                  upstream=None, downstream=down, logger=EventLogger("w0", "f"))
    assert time.monotonic() - t0 < 6
    assert "state" in str(ei.value)
    peer.close()


def test_peer_disconnect_fails_fast():
    spec = build_model_spec({"type": "mlp"})
    down, peer = _link_pair()
    threading.Timer(0.5, peer.close).start()
    t0 = time.monotonic()
    with pytest.raises(PipelineError, match="disconnected|failed"):
        run_stage(_first_stage(spec), spec, PipelineSettings("f", steps=1, batch_size=8, timeout_s=30.0),
                  upstream=None, downstream=down, logger=EventLogger("w0", "f"))
    assert time.monotonic() - t0 < 6, "a disconnect must not wait for the full timeout"


def test_crashing_stage_reports_error_upstream():
    spec = build_model_spec({"type": "mlp"})
    down, up = _link_pair()
    settings = PipelineSettings("f", steps=1, batch_size=8, timeout_s=30.0)

    def bad_last_stage():
        stage = Stage(spec.build_stage(6, 7), stage_index=1, num_stages=2, loss_fn=spec.loss_fn)  # wrong width
        with pytest.raises(Exception):
            run_stage(stage, spec, settings, upstream=up, downstream=None, logger=EventLogger("w1", "f"))

    th = threading.Thread(target=bad_last_stage)
    th.start()
    with pytest.raises(PipelineError, match="peer reported error"):
        run_stage(_first_stage(spec), spec, settings, upstream=None, downstream=down, logger=EventLogger("w0", "f"))
    th.join(5)
    assert not th.is_alive()


def test_stop_event_ends_a_stage():
    spec = build_model_spec({"type": "mlp"})
    down, peer = _link_pair()
    stop = threading.Event()
    threading.Timer(0.3, stop.set).start()
    with pytest.raises(PipelineError, match="stopped"):
        run_stage(_first_stage(spec), spec, PipelineSettings("f", steps=5, batch_size=8, timeout_s=30.0),
                  upstream=None, downstream=down, logger=EventLogger("w0", "f"), stop_event=stop)
    peer.close()


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
