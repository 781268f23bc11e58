"""Activation recompute on the GPU kernels: a bf16 GPT and a bf16 Llama stage with every
block recomputed in backward give the loss and gradients of the stage that keeps its
activations (within bf16 rounding: split-K partial sums may add in another order when the
forward runs again), and hold less memory at the step's peak."""

import pytest
import torch

from meshtrain_b200 import ops
from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.recompute import choose_units
from meshtrain_b200.planner.graph import analytic_profile

pytestmark = pytest.mark.gpu

GPT = {"type": "gpt", "layers": 4, "hidden_size": 512, "heads": 8, "vocab_size": 2048, "seq_len": 512,
       "dtype": "bfloat16"}
LLAMA = {"type": "llama", "layers": 2, "hidden_size": 512, "heads": 4, "n_kv_heads": 2, "ffn_hidden": 1024,
         "vocab_size": 2048, "seq_len": 512, "dtype": "bfloat16"}


def _step(cfg, recompute):
    from meshtrain_b200.parallel.engine import PipelineEngine

    spec = build_model_spec(cfg, seed=7)
    units = choose_units(recompute, analytic_profile(spec, 4)) if recompute else None
    eng = PipelineEngine(spec, layer_range=(0, spec.num_layers), stage=0, num_stages=1, device="cuda:0",
                         num_microbatches=2, optimizer="sgd", lr=0.0, init_on_device=True, recompute=units)
    x, y = spec.make_batch(0, 8)
    x, y = x.cuda(), y.cuda()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    before = torch.cuda.memory_allocated()
    st = eng.train_step(0, x, y)
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - before
    grads = eng.named_gradients_cpu()
    assert ops.read_status(0) == 0
    return float(st.loss), grads, peak


@pytest.mark.parametrize("cfg", [GPT, LLAMA], ids=["gpt", "llama"])
def test_recompute_matches_kept_activations(cfg):
    ops.set_backend("custom")
    loss0, g0, peak0 = _step(cfg, None)
    loss1, g1, peak1 = _step(cfg, "all")
    assert loss1 == pytest.approx(loss0, rel=1e-3)
    for k, ref in g0.items():
        got = g1[k].float()
        ref = ref.float()
        rel = ((got - ref).norm() / (ref.norm() + 1e-12)).item()
        assert rel < 2e-2, (k, rel)
    assert peak1 < peak0
