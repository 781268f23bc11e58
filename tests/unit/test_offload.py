"""Host offload of master weights + Adam moments gives the same training as resident state."""

import pytest
import torch

from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.engine import PipelineEngine
from meshtrain_b200.parallel.offload import HostOffload

GPT = {"type": "gpt", "layers": 2, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32,
       "dtype": "float32"}


def _train(offload, optimizer="adamw", steps=3):
    spec = build_model_spec(GPT, seed=1)
    eng = PipelineEngine(spec, layer_range=(0, spec.num_layers), stage=0, num_stages=1, device="cpu",
                         num_microbatches=2, optimizer=optimizer, lr=1e-3, weight_decay=0.01, offload=offload)
    losses = []
    for step in range(steps):
        x, y = spec.make_batch(step, 4)
        losses.append(float(eng.train_step(step, x, y).loss))
    return losses, eng.named_parameters_cpu(), eng


@pytest.mark.parametrize("optimizer", ["adamw", "adam", "sgd"])
@pytest.mark.parametrize("chunk_mb,ahead", [(0.01, 1), (0.003, 0), (64, 3)])
def test_offloaded_step_matches_resident(optimizer, chunk_mb, ahead):
    ref_losses, ref_params, _ = _train(None, optimizer)
    off = HostOffload(prefetch_ahead=ahead, chunk_mb=chunk_mb)
    losses, params, eng = _train(off, optimizer)
    assert losses == pytest.approx(ref_losses, rel=1e-6)
    for k, v in ref_params.items():
        assert torch.allclose(params[k], v, rtol=1e-6, atol=1e-7), k
    assert off.stats["steps"] == 3 and off.stats["h2d_bytes"] == off.stats["d2h_bytes"] == 3 * 12 * eng.flat.numel
    assert eng.flat.master.device.type == "cpu"


def test_staging_is_bounded_by_slots():
    off = HostOffload(prefetch_ahead=1, chunk_mb=0.01)
    _, _, eng = _train(off, steps=1)
    assert len(off.chunks) > off.nslots >= 2
    assert off.device_bytes() == off.nslots * 3 * off.chunk_elems * 4


@pytest.mark.parametrize("kw", [{}, {"chunk_mb": 1.0}, {"chunk_mb": 0.5, "device_budget_gb": 0.01},
                                {"chunk_mb": 2.0, "prefetch_ahead": 3}])
def test_slot_ring_estimate_matches_the_allocated_ring(kw):
    """The memory estimate's ``slot_ring_bytes`` equals what a ``HostOffload`` with the same settings
    allocates, both from its constructor arguments and from ``ring_settings()``."""
    from meshtrain_b200.parallel.offload import HostOffload, slot_ring_bytes

    class Flat:  # the attributes ``attach`` reads
        device = torch.device("cpu")
        numel = 3_000_000

    off = HostOffload(**kw)
    off.attach(Flat())
    assert slot_ring_bytes(Flat.numel, **kw) == off.device_bytes()
    assert slot_ring_bytes(Flat.numel, **off.ring_settings()) == off.device_bytes()
