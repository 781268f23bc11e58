"""Wire compatibility with the reference: pipelines that mix the reference's own runtime (installed
under ``baseline/_ref``) and this package's host runtime, talking MSHT v1 framed packets over
loopback TCP, train exactly like one process, in both directions and under both schedules.

Both implementations build the same weights and batches for the same seeds (per-layer seeds, same
data generator), so a mixed pipeline is held to the single-process oracle.  The reference stage
runs in a process of its own, as the reference runs every stage (its runtime keeps per-process
state).  Skips where the reference is not installed."""

import multiprocessing as mp
import os
import socket

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF = os.path.join(ROOT, "baseline", "_ref")
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "meshtrain")),
                                reason="the reference is not installed under baseline/_ref")

MODELS = {"mlp": {"type": "mlp"},
          "transformer": {"type": "tiny_transformer", "layers": 2, "hidden_size": 64, "heads": 4, "vocab_size": 64,
                          "seq_len": 16}}
STEPS, BATCH, MICRO, LR = 3, 16, 4, 1e-3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _reference_stage(model: dict, first: bool, schedule: str, port: int, out) -> None:
    """One stage of the reference's runtime (child process): the first stage connects to our
    listener, the last stage listens for our first stage.  Puts its losses (first stage) or None."""
    import sys

    sys.path.append(REF)
    torch.set_num_threads(1)
    import meshtrain.models as ref_models
    import meshtrain.networking.tcp as ref_tcp
    import meshtrain.runtime.pipeline as ref_pipeline
    import meshtrain.runtime.stage as ref_stage
    import meshtrain.telemetry as ref_telemetry

    try:
        spec = ref_models.build_model_spec(dict(model))
        cut = spec.num_layers // 2
        settings = ref_pipeline.PipelineSettings("interop", steps=STEPS, batch_size=BATCH, num_microbatches=MICRO,
                                                 schedule=schedule)
        log = ref_telemetry.EventLogger("ref", "interop", verbose=False)
        if first:
            stage = ref_stage.Stage(spec.build_stage(0, cut), stage_index=0, num_stages=2, optimizer="adam", lr=LR)
            link = ref_tcp.connect("127.0.0.1", port, timeout=30, hello={"job_id": "interop"})
            result = ref_pipeline.run_stage(stage, spec, settings, upstream=None, downstream=link, logger=log)
            out.put(("ok", result.losses))
        else:
            listener = ref_tcp.TCPListener("127.0.0.1", port)
            stage = ref_stage.Stage(spec.build_stage(cut, spec.num_layers), stage_index=1, num_stages=2,
                                    optimizer="adam", lr=LR, loss_fn=spec.loss_fn, layer_offset=cut)
            link, _hello = listener.accept(timeout=30)
            ref_pipeline.run_stage(stage, spec, settings, upstream=link, downstream=None, logger=log)
            listener.close()
            out.put(("ok", None))
    except Exception as exc:  # noqa: BLE001 - handed to the test
        out.put(("error", f"{type(exc).__name__}: {exc}"))


@pytest.mark.parametrize("schedule", ["gpipe", "1f1b"])
@pytest.mark.parametrize("name", sorted(MODELS))
@pytest.mark.parametrize("reference_is_first", [True, False], ids=["reference-first", "reference-last"])
def test_mixed_pipeline_matches_one_process(reference_is_first, name, schedule):
    from meshtrain_b200.models import build_model_spec
    from meshtrain_b200.networking.tcp import TCPListener, connect
    from meshtrain_b200.parallel.local import reference_step
    from meshtrain_b200.parallel.pipeline import PipelineSettings, run_stage
    from meshtrain_b200.parallel.stage import Stage
    from meshtrain_b200.telemetry import EventLogger

    model = MODELS[name]
    threads = torch.get_num_threads()
    torch.set_num_threads(1)  # both stages and the oracle reduce in the same order
    try:
        spec = build_model_spec(dict(model))
        cut = spec.num_layers // 2
        settings = PipelineSettings("interop", steps=STEPS, batch_size=BATCH, num_microbatches=MICRO,
                                    schedule=schedule)
        port = _free_port()
        ctx = mp.get_context("spawn")
        out = ctx.Queue()
        listener = TCPListener("127.0.0.1", port) if reference_is_first else None
        child = ctx.Process(target=_reference_stage, args=(model, reference_is_first, schedule, port, out))
        child.start()
        log = EventLogger("ours", "interop")
        if reference_is_first:
            up, _hello = listener.accept(timeout=60)
            listener.close()
            ours = Stage(spec.build_stage(cut, spec.num_layers), stage_index=1, num_stages=2, optimizer="adam",
                         lr=LR, loss_fn=spec.loss_fn, layer_offset=cut)
            run_stage(ours, spec, settings, upstream=up, downstream=None, logger=log)
        else:
            down = connect("127.0.0.1", port, timeout=60, hello={"job_id": "interop"})
            ours = Stage(spec.build_stage(0, cut), stage_index=0, num_stages=2, optimizer="adam", lr=LR)
            mine = run_stage(ours, spec, settings, upstream=None, downstream=down, logger=log)
        status, payload = out.get(timeout=120)
        child.join(30)
        assert status == "ok", payload
        # the first stage records the loss that the last stage reports back over the wire
        losses = payload if reference_is_first else mine.losses
        oracle, _, _ = reference_step(dict(model), settings, optimizer="adam", lr=LR, steps=STEPS)
        assert len(losses) == STEPS and losses == pytest.approx(oracle, rel=2e-7)
    finally:
        torch.set_num_threads(threads)
