"""Device timing of engine steps on one GPU: waiting per step (timed=True) and
reading the events afterwards (timed="deferred") give the same breakdown shape,
and the deferred steps leave the host free to run ahead."""

import pytest
import torch

pytestmark = pytest.mark.gpu

MODEL = {"type": "gpt", "layers": 2, "hidden_size": 256, "heads": 4, "vocab_size": 1000, "seq_len": 256,
         "dtype": "bfloat16", "init_std": 0.02, "data": "uniform"}


def test_deferred_timing_matches_waiting():
    from meshtrain_b200 import ops
    from meshtrain_b200.models import build_model_spec
    from meshtrain_b200.parallel.engine import PipelineEngine

    ops.set_backend("custom")
    spec = build_model_spec(MODEL, seed=0)
    eng = PipelineEngine(spec, layer_range=(0, spec.num_layers), stage=0, num_stages=1, device="cuda:0",
                         num_microbatches=2)
    batches = [spec.make_batch(s, 4) for s in range(6)]
    for s in range(2):
        eng.train_step(s, *batches[s], timed=False)
    waited = [eng.train_step(s, *batches[s], timed=True) for s in range(2, 4)]
    deferred = [eng.train_step(s, *batches[s], timed="deferred") for s in range(4, 6)]
    assert all(st.pending is not None and st.step_ms == 0.0 for st in deferred)
    torch.cuda.synchronize()
    for st in deferred:
        eng.finish_timing(st)
        assert st.pending is None
    for st in waited + deferred:
        assert st.step_ms > 0 and 0.0 <= st.bubble_fraction < 1.0
        assert st.forward_ms > 0 and st.backward_ms > 0 and st.optimizer_ms > 0
    assert len(eng._spare_pools) == 2  # the deferred steps' event pools are reused
    mean = lambda xs: sum(xs) / len(xs)  # noqa: E731
    assert mean([s.step_ms for s in deferred]) == pytest.approx(mean([s.step_ms for s in waited]), rel=0.5)
    assert ops.read_status(0) == 0
