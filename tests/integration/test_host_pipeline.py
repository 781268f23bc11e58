"""The host pipeline runtime (stages as OS processes, framed packets over pipes
or loopback TCP) against the single-process oracle."""

import pytest
import torch

from meshtrain_b200.experiments.correctness import compare_gradients, format_gradient_report, run_gradient_equivalence
from meshtrain_b200.parallel.local import LocalStage, global_param_names, reference_step, run_local_pipeline
from meshtrain_b200.parallel.pipeline import PipelineSettings

MLP = {"type": "mlp"}
TT = {"type": "tiny_transformer", "layers": 4, "hidden_size": 64, "heads": 4, "vocab_size": 64, "seq_len": 16}
# The oracle and the stage processes both run single-threaded, so they reduce in
# the same order: errors are at the level of the C1 gate (2e-7), not float noise.
TOL = 2e-7


def _ok(rows, tol=TOL):
    print("\n" + format_gradient_report(rows))
    assert all(r.relative <= tol and r.max_abs <= 1e-6 for r in rows), format_gradient_report(rows)


def test_two_stages_match_single_process():
    rows, info = run_gradient_equivalence(MLP, [LocalStage((0, 3)), LocalStage((3, 7))], batch_size=32)
    assert {r.stage for r in rows} == {0, 1} and len(rows) == 8
    assert info["distributed_loss"] == pytest.approx(info["reference_loss"], rel=1e-6)
    _ok(rows)


@pytest.mark.parametrize("schedule", ["gpipe", "1f1b"])
def test_three_stages_microbatched_tcp(schedule):
    rows, _ = run_gradient_equivalence(MLP, [LocalStage((0, 2)), LocalStage((2, 5)), LocalStage((5, 7))],
                                       batch_size=32, num_microbatches=4, transport="tcp", schedule=schedule)
    _ok(rows)


def test_microbatch_accumulation_equals_full_batch():
    _, full, _ = reference_step(MLP, PipelineSettings("ref", steps=1, batch_size=32, num_microbatches=1))
    stages = [LocalStage((0, 4)), LocalStage((4, 7))]
    res = run_local_pipeline(MLP, stages, PipelineSettings("mb", steps=1, batch_size=32, num_microbatches=8,
                                                           capture_gradients_at_step=0))
    got = {}
    for r in res:
        got.update(global_param_names(stages, r.gradients, r.stage_index))
    # one batch of 32 against 8 microbatches of 4: a different summation order
    assert all(row.relative < 1e-5 for row in compare_gradients(full, got))


def test_transformer_three_stages():
    rows, _ = run_gradient_equivalence(TT, [LocalStage((0, 2)), LocalStage((2, 4)), LocalStage((4, 6))],
                                       batch_size=8, num_microbatches=2)
    _ok(rows)


def test_async_1f1b_training_tracks_single_process():
    stages = [LocalStage((0, 3)), LocalStage((3, 7))]
    settings = PipelineSettings("train", steps=30, batch_size=64, num_microbatches=4, log_every=10,
                                schedule="1f1b", async_transport=True, max_outbound_queue=2)
    res = run_local_pipeline(MLP, stages, settings, optimizer="adam", lr=1e-3, capture_params=True)
    losses = res[0].losses
    assert losses[-1] < losses[0]
    for r in res:
        assert all(not torch.equal(r.initial_params[k], r.final_params[k]) for k in r.initial_params)
    ref, _, ref_params = reference_step(MLP, settings, optimizer="adam", lr=1e-3, steps=30)
    assert losses == pytest.approx(ref, rel=2e-7, abs=1e-7)
    final = {}
    for r in res:
        final.update(global_param_names(stages, r.final_params, r.stage_index))
    for k, v in ref_params.items():
        assert torch.allclose(final[k], v, atol=1e-6, rtol=2e-7), k


def test_emulated_slow_link_still_correct():
    stages = [LocalStage((0, 3)), LocalStage((3, 7))]
    settings = PipelineSettings("slow", steps=2, batch_size=16, num_microbatches=2, capture_gradients_at_step=1)
    res = run_local_pipeline(MLP, stages, settings, transport="tcp", link_emulation=(50e6, 0.002))
    _, ref_grads, _ = reference_step(MLP, settings, steps=2)
    got = {}
    for r in res:
        got.update(global_param_names(stages, r.gradients, r.stage_index))
    assert all(row.relative < TOL for row in compare_gradients(ref_grads, got))
    m = res[0].step_metrics[-1]
    assert m["bytes_sent"] > 0


def test_compressed_links_halve_the_bytes():
    """``wire_compression="bf16"``: fp32 activations and gradients cross as bf16, the pipeline still
    trains (losses within bf16 rounding of the uncompressed run) and sends about half the bytes."""
    from meshtrain_b200.parallel.local import LocalStage, run_local_pipeline
    from meshtrain_b200.parallel.pipeline import PipelineSettings

    model = {"type": "tiny_transformer", "layers": 2, "hidden_size": 64, "heads": 4, "vocab_size": 64, "seq_len": 16}
    stages = [LocalStage((0, 2)), LocalStage((2, 4))]
    runs = {}
    for wire in (None, "bf16"):
        settings = PipelineSettings("wire", steps=4, batch_size=8, num_microbatches=4, schedule="1f1b",
                                    wire_compression=wire)
        res = run_local_pipeline(model, stages, settings, optimizer="adam", lr=1e-3, transport="tcp")
        sent = sum(m["bytes_sent"] for m in res[0].step_metrics)
        runs[wire] = (res[0].losses, sent)
    plain, packed = runs[None], runs["bf16"]
    assert packed[0] == pytest.approx(plain[0], rel=2e-2)
    assert packed[1] < 0.6 * plain[1]
