"""Activation recompute in the device engine: the same gradients and training as keeping
every activation (CPU, fp32, one thread: bit for bit), with fewer bytes held per microbatch."""

import pytest
import torch

from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.recompute import (RecomputeEvery, RecomputeLargest, apply_to_profiles, choose_units,
                                               parse_policy)
from meshtrain_b200.parallel.spawn import spawn_ranks
from meshtrain_b200.planner.graph import analytic_profile

GPT = {"type": "gpt", "layers": 3, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32,
       "dtype": "float32"}
LLAMA = {"type": "llama", "layers": 2, "hidden_size": 64, "heads": 4, "n_kv_heads": 2, "ffn_hidden": 96,
         "vocab_size": 96, "seq_len": 32, "dtype": "float32"}


def _grads(cfg, recompute, split=False):
    from meshtrain_b200.parallel.engine import PipelineEngine

    torch.set_num_threads(1)
    spec = build_model_spec(dict(cfg, split_blocks=split), seed=5)
    units = choose_units(recompute, analytic_profile(spec, 2)) if recompute else None
    eng = PipelineEngine(spec, layer_range=(0, spec.num_layers), stage=0, num_stages=1, device="cpu",
                         num_microbatches=2, optimizer="sgd", lr=0.0, recompute=units)
    x, y = spec.make_batch(0, 4)
    st = eng.train_step(0, x, y)
    return float(st.loss), eng.named_gradients_cpu(), eng


@pytest.mark.parametrize("cfg", [GPT, LLAMA], ids=["gpt", "llama"])
@pytest.mark.parametrize("policy", ["all", "every:2", "largest:1"])
def test_recompute_gives_identical_gradients(cfg, policy):
    loss0, g0, _ = _grads(cfg, None)
    loss1, g1, eng = _grads(cfg, policy)
    assert eng.recompute_local, "the policy chose no unit"
    assert loss1 == loss0
    for k, v in g0.items():
        assert torch.equal(g1[k], v), k


def test_recompute_on_half_block_units():
    loss0, g0, _ = _grads(GPT, None, split=True)
    loss1, g1, eng = _grads(GPT, "all", split=True)
    assert len(eng.recompute_local) == 6 and loss1 == loss0
    assert all(torch.equal(g1[k], v) for k, v in g0.items())


def test_policies_and_profiles():
    spec = build_model_spec(dict(GPT, dtype="bfloat16", layers=4), seed=0)
    prof = analytic_profile(spec, 4)
    assert choose_units("all", prof) == {1, 2, 3, 4}  # never the embedding (0) or the head (5)
    assert choose_units("every:2", prof) == {2, 4}
    assert choose_units(RecomputeEvery(3), prof) == {3}
    assert choose_units("none", prof) == set()
    assert len(choose_units("largest:2", prof)) == 2
    assert RecomputeLargest(1, {1: 5, 2: 9}).should_recompute(2, 0)
    with pytest.raises(ValueError):
        parse_policy("sometimes")
    after = apply_to_profiles(prof, {1, 2})
    assert after[1].saved_bytes == prof[1].input_bytes < prof[1].saved_bytes
    assert after[1].recompute_bytes == prof[1].saved_bytes and after[3] == prof[3]
    assert after[1].flops == pytest.approx(prof[1].flops * 4 / 3)


def test_recompute_lowers_the_estimate():
    from meshtrain_b200.api import check_interleaved_memory, plan_device_pipeline

    spec = build_model_spec({"type": "llama", "layers": 8, "hidden_size": 4096, "heads": 32, "n_kv_heads": 8,
                             "ffn_hidden": 14336, "vocab_size": 128256, "seq_len": 4096, "dtype": "bfloat16"})
    prof = analytic_profile(spec, 1)
    units = choose_units("all", prof)
    keep = plan_device_pipeline(spec, 2, 16, 1, "1f1b", "adam", memory_gb=180.0)
    lean = plan_device_pipeline(spec, 2, 16, 1, "1f1b", "adam", memory_gb=180.0, recompute=units)
    assert lean.stages[0].memory.saved_activations < keep.stages[0].memory.saved_activations / 3
    pieces = [(0, 3), (3, 5), (5, 8), (8, 10)]
    a = check_interleaved_memory(spec, pieces, 2, 2, 16, 1, "adam", memory_gb=180.0)
    b = check_interleaved_memory(spec, pieces, 2, 2, 16, 1, "adam", memory_gb=180.0, recompute=units)
    assert b[0].required < a[0].required


def _train(model, steps, recompute=None, M=4, mbs=2):
    from meshtrain_b200.api import PipelineTrainer

    torch.set_num_threads(1)
    tr = PipelineTrainer(model, num_microbatches=M, optimizer="adam", lr=1e-3, device="cpu", microbatch_size=mbs,
                         recompute=recompute)
    losses = []
    for step in range(steps):
        x, y = tr.spec.make_batch(step, M * mbs)
        losses.append(tr.loss_value(tr.step(step, x, y)))
    params = tr.engine.named_parameters_cpu()
    tr.close()
    return losses, params


def test_gloo_ranks_with_recompute_match_one_rank_without():
    single = spawn_ranks(_train, 1, GPT, 3)[0]
    ranked = spawn_ranks(_train, 2, GPT, 3, recompute="all")
    assert ranked[-1][0] == pytest.approx(single[0], rel=1e-6)
    merged = {}
    for _, params in ranked:
        merged.update(params)
    for k, v in single[1].items():
        assert torch.allclose(merged[k], v, rtol=1e-5, atol=1e-7), k
