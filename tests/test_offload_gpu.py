"""Streamed host offload on the GPU: pinned host master/moments, double-buffered device slots,
fused Adam kernel per chunk; must track resident-state training."""

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
    # the backward kernels accumulate some gradients with fp32 atomics (order varies run to run),
    # so parameters agree to rounding, not bit for bit
    a, b = ref.named_parameters_cpu(), eng.named_parameters_cpu()
    for k in a:
        assert torch.allclose(a[k], b[k], rtol=1e-4, atol=1e-6), k
    assert torch.allclose(ref.flat.compute.float().cpu(), eng.flat.compute.float().cpu(), rtol=1e-2, atol=1e-5)
    assert ops.read_status(torch.cuda.current_device()) == 0


def test_chunked_adam_is_bitwise_equal_to_one_launch():
    """Same gradients in, same bits out: chunking the fused Adam over device slots changes nothing."""
    from meshtrain_b200.parallel.engine import FlatState

    torch.manual_seed(0)
    layers = [torch.nn.Linear(300, 500), torch.nn.Linear(500, 70)]
    layers2 = [torch.nn.Linear(300, 500), torch.nn.Linear(500, 70)]
    for a, b in zip(layers, layers2):  # before FlatState rebinds the parameters to bf16 views
        b.load_state_dict(a.state_dict())
    resident = FlatState([l.cuda() for l in layers], torch.device("cuda"), torch.bfloat16)
    offl = FlatState([l.cuda() for l in layers2], torch.device("cuda"), torch.bfloat16, offload=True)
    off = HostOffload(prefetch_ahead=1, chunk_mb=0.05)
    off.attach(offl)

    class Eng:
        opt_name, lr, betas, eps, wd = "adamw", 1e-3, (0.9, 0.999), 1e-8, 0.01

    for step in range(1, 4):
        g = torch.randn(resident.numel, device="cuda")
        resident.grad.copy_(g)
        offl.grad.copy_(g)
        Eng.opt_steps = step
        ops.adam_(resident.master, resident.grad, resident.exp_avg, resident.exp_avg_sq, resident.compute, lr=1e-3,
                  beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, decoupled=True, step=step)
        off.prefetch()
        off.step(Eng)
    off.synchronize()
    torch.cuda.synchronize()
    assert torch.equal(resident.master.cpu(), offl.master)
    assert torch.equal(resident.exp_avg_sq.cpu(), offl.exp_avg_sq)
    assert torch.equal(resident.compute, offl.compute)
