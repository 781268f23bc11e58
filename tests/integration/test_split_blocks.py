"""Half-block partition units (models/split.py): the same model, parameters and
training as whole blocks, with stage boundaries allowed inside a block."""

import pytest
import torch

from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.spawn import spawn_ranks

GPT = {"type": "gpt", "layers": 3, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32,
       "dtype": "float32"}
LLAMA = {"type": "llama", "layers": 2, "hidden_size": 64, "heads": 4, "n_kv_heads": 2, "ffn_hidden": 96,
         "vocab_size": 96, "seq_len": 32, "dtype": "float32"}


@pytest.mark.parametrize("cfg", [GPT, LLAMA], ids=["gpt", "llama"])
def test_units_and_parameters_match_whole_blocks(cfg):
    whole = build_model_spec(cfg, seed=5)
    split = build_model_spec(dict(cfg, split_blocks=True), seed=5)
    assert split.num_layers == whole.num_layers + whole.n_blocks
    ids_whole, ids_split = {}, {}
    for i in range(whole.num_layers):
        for n, p in whole.build_layer(i).named_parameters():
            ids_whole[f"model.layers.{i}.{n}"] = p
    for u in range(split.num_layers):
        for n, p in split.build_layer(u).named_parameters():
            key = f"model.layers.{split.global_layer(u)}.{n}"
            assert key not in ids_split, key  # every parameter owned by exactly one unit
            ids_split[key] = p
    assert ids_split.keys() == ids_whole.keys()
    for k, p in ids_whole.items():
        assert torch.equal(ids_split[k], p), k
    assert split.layer_name(1).endswith(".attn") and split.layer_name(2).endswith(".mlp")
    assert sum(split.layer_parameter_counts()) == whole.parameter_count()


@pytest.mark.parametrize("cfg", [GPT, LLAMA], ids=["gpt", "llama"])
def test_split_units_forward_backward_match(cfg):
    """Running the halves in sequence is the block: same loss and gradients on one stage."""
    from meshtrain_b200.parallel.engine import PipelineEngine

    out = {}
    for split in (False, True):
        spec = build_model_spec(dict(cfg, split_blocks=split), seed=3)
        eng = PipelineEngine(spec, layer_range=(0, spec.num_layers), stage=0, num_stages=1,
                             device=torch.device("cpu"), num_microbatches=2, optimizer="sgd", lr=0.0)
        x, y = spec.make_batch(0, 4)
        st = eng.train_step(0, x, y)
        out[split] = (float(st.loss.detach()), eng.named_gradients_cpu())
    assert out[True][0] == out[False][0]
    assert out[True][1].keys() == out[False][1].keys()
    for k, g in out[False][1].items():
        assert torch.equal(out[True][1][k], g), k


def _train(model, steps, partition, M=4, mbs=2):
    from meshtrain_b200.api import PipelineTrainer

    tr = PipelineTrainer(model, num_microbatches=M, optimizer="adam", lr=1e-3, device="cpu", schedule="1f1b",
                         microbatch_size=mbs, partition=partition)
    losses = []
    for step in range(steps):
        x, y = tr.spec.make_batch(step, M * mbs)
        losses.append(tr.loss_value(tr.step(step, x, y)))
    params = tr.engine.named_parameters_cpu()
    tr.close()
    return losses, params


def test_boundary_inside_a_block_matches_single_rank():
    """Stage 0 ends after block 1's attention half; stage 1 starts with its MLP half."""
    split = dict(GPT, split_blocks=True)
    single = spawn_ranks(_train, 1, GPT, 3, [[0, 5]])[0]
    ranked = spawn_ranks(_train, 2, split, 3, [[0, 4], [4, 8]])
    assert ranked[-1][0] == pytest.approx(single[0], rel=1e-5)
    merged = {}
    for _, params in ranked:
        assert not set(params) & set(merged)
        merged.update(params)
    assert set(merged) == set(single[1])
    for k, v in single[1].items():
        assert torch.allclose(merged[k], v, rtol=1e-4, atol=1e-6), k


def test_checkpoint_moves_between_split_and_whole(tmp_path):
    """A checkpoint written by half-block stages loads into whole-block stages and back."""
    from meshtrain_b200.checkpoint import load_stage_checkpoint, save_stage_checkpoint
    from meshtrain_b200.parallel.engine import PipelineEngine

    split_spec = build_model_spec(dict(GPT, split_blocks=True), seed=1)
    whole_spec = build_model_spec(GPT, seed=1)
    engines = [PipelineEngine(split_spec, layer_range=r, stage=s, num_stages=2, device=torch.device("cpu"),
                              num_microbatches=1, optimizer="adam", lr=1e-3, links=object())  # no step is run
               for s, r in enumerate([(0, 4), (4, 8)])]
    for e in engines:
        with torch.no_grad():
            e.flat.master.add_(0.5)
        e.opt_steps = 7
        save_stage_checkpoint(tmp_path, e, 3)
    whole = PipelineEngine(whole_spec, layer_range=(0, whole_spec.num_layers), stage=0, num_stages=1,
                           device=torch.device("cpu"), num_microbatches=1, optimizer="adam", lr=1e-3)
    assert load_stage_checkpoint(tmp_path, whole) == 3
    want = {}
    for e in engines:
        want.update(e.named_parameters_cpu())
    got = whole.named_parameters_cpu()
    assert got.keys() == want.keys()
    for k in want:
        assert torch.equal(got[k], want[k]), k


def test_half_block_units_balance_eight_stages():
    """At 8 stages the 0.48B GPT's largest stage is within 10 % of the average with half-block
    units, where whole blocks leave it about 20 % above."""
    from meshtrain_b200.api import layer_costs
    from meshtrain_b200.parallel.engine import balanced_split

    m = {"type": "gpt", "layers": 24, "hidden_size": 1280, "heads": 20, "vocab_size": 50257, "seq_len": 2048,
         "dtype": "bfloat16"}
    ratio = {}
    for split in (False, True):
        c = layer_costs(build_model_spec(dict(m, split_blocks=split)))
        r = balanced_split(c, 8)
        ratio[split] = max(sum(c[a:b]) for a, b in r) / (sum(c) / 8)
    assert ratio[True] < 1.1 < ratio[False]
