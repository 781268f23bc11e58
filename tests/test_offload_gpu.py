"""Streamed host offload on the GPU: pinned host master/moments, double-buffered device slots,
fused Adam kernel per chunk; must track resident-state training bit for bit."""

import pytest
import torch

from meshtrain_b200 import ops
from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.engine import PipelineEngine
from meshtrain_b200.parallel.offload import HostOffload

pytestmark = pytest.mark.gpu

GPT = {"type": "gpt", "layers": 2, "hidden_size": 256, "heads": 4, "vocab_size": 1000, "seq_len": 256,
       "dtype": "bfloat16", "init_std": 0.02, "data": "uniform"}


def _run(offload):
    ops.set_backend("custom")
    spec = build_model_spec(GPT, seed=2)
    eng = PipelineEngine(spec, layer_range=(0, spec.num_layers), stage=0, num_stages=1, device="cuda",
                         num_microbatches=2, optimizer="adamw", lr=1e-3, weight_decay=0.01, offload=offload,
                         init_on_device=True)
    losses = []
    for step in range(3):
        x, y = spec.make_batch(step, 4)
        losses.append(float(eng.train_step(step, x.pin_memory(), y.pin_memory(), timed=False).loss))
    return losses, eng


def test_offload_matches_resident_on_gpu():
    ref_losses, ref = _run(None)
    off = HostOffload(prefetch_ahead=1, chunk_mb=1.0)
    losses, eng = _run(off)
    assert eng.flat.master.is_pinned() and eng.flat.exp_avg.is_pinned()
    assert len(off.chunks) > off.nslots
    assert losses == pytest.approx(ref_losses, rel=1e-6)
    a, b = ref.named_parameters_cpu(), eng.named_parameters_cpu()
    for k in a:
        assert torch.equal(a[k], b[k]), k
    assert torch.equal(ref.flat.compute.cpu(), eng.flat.compute.cpu())
    assert ops.read_status(torch.cuda.current_device()) == 0
