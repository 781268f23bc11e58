"""Live layer migration: a measured imbalance moves stage boundaries between steps, and
training continues exactly as if the new split had been used from the start."""

import pytest
import torch

from meshtrain_b200.parallel.migration import RebalanceByMeasurement, owner_of
from meshtrain_b200.parallel.spawn import spawn_ranks

GPT = {"type": "gpt", "layers": 4, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32,
       "dtype": "float32"}


def test_policy_moves_units_off_the_slow_stage():
    policy = RebalanceByMeasurement(min_gain=0.03)
    metrics = {"ranges": [(0, 3), (3, 6)], "busy_ms": [30.0, 10.0], "unit_costs": [1.0] * 6}
    moves = policy.propose(5, metrics)
    assert policy.last_ranges == [(0, 2), (2, 6)] and moves == [(2, "rank0", "rank1")]
    assert policy.predicted_gain > 0.3
    # measured as predicted: nothing moves
    assert policy.propose(6, {**metrics, "busy_ms": [20.0, 20.0]}) == []
    assert owner_of([(0, 2), (2, 5)]) == {0: 0, 1: 0, 2: 1, 3: 1, 4: 1}


def _train(model, steps, switch_at=None, new_ranges=None, partition=None, busy=None):
    from meshtrain_b200.api import PipelineTrainer

    torch.set_num_threads(1)
    tr = PipelineTrainer(model, num_microbatches=4, optimizer="adam", lr=1e-3, device="cpu", microbatch_size=2,
                         partition=partition or "equal")
    losses, moves = [], []
    for step in range(steps):
        if step == switch_at:
            if new_ranges is not None:
                tr.repartition(new_ranges)
            else:
                moves = tr.rebalance([], busy_ms=busy[tr.rank])
        x, y = tr.spec.make_batch(step, 8)
        losses.append(tr.loss_value(tr.step(step, x, y)))
    params = tr.engine.named_parameters_cpu()
    ranges = [tuple(r) for r in tr.ranges]
    tr.close()
    return losses, params, ranges, moves


def _merged(ranked):
    out = {}
    for _, params, _, _ in ranked:
        out.update(params)
    return out


def test_repartition_mid_run_matches_training_on_the_new_split():
    ref = spawn_ranks(_train, 2, GPT, 4, partition=[(0, 2), (2, 6)])
    moved = spawn_ranks(_train, 2, GPT, 4, switch_at=2, new_ranges=[(0, 2), (2, 6)])  # equal split is (0,3),(3,6)
    assert moved[0][2] == [(0, 2), (2, 6)]
    assert moved[-1][0] == pytest.approx(ref[-1][0], rel=1e-6)
    want, got = _merged(ref), _merged(moved)
    for k, v in want.items():
        assert torch.allclose(got[k], v, rtol=1e-5, atol=1e-7), k


def test_rebalance_from_measurements_moves_a_unit():
    out = spawn_ranks(_train, 2, GPT, 3, switch_at=1, busy=[30.0, 10.0])
    assert out[0][2] == [(0, 2), (2, 6)] and out[1][2] == [(0, 2), (2, 6)]
    assert out[0][3] == [(2, "rank0", "rank1")]
    assert all(loss is not None for loss in out[-1][0])


def test_local_training_with_rebalancing_enabled(tmp_path):
    """``pipeline.rebalance_after_steps`` in a config: CPU ranks have no device timing, so the split stays
    and training runs to the end."""
    import yaml

    from meshtrain_b200.cli import main

    cfg = {"job": {"name": "rb", "runs_dir": str(tmp_path / "runs")},
           "model": {"type": "gpt", "layers": 2, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32},
           "network": {"tensor_transport": "nccl", "timeout_s": 60},
           "pipeline": {"rebalance_after_steps": 2}, "placement": {"strategy": "equal", "num_stages": 2},
           "training": {"batch_size": 8, "microbatch_size": 2, "steps": 4, "optimizer": "adam", "learning_rate": 1e-3}}
    path = tmp_path / "rb.yaml"
    path.write_text(yaml.safe_dump(cfg))
    assert main(["train", str(path), "--local"]) == 0
    run = next((tmp_path / "runs").iterdir())
    assert (run / "timeline.json").exists() and (run / "metrics.jsonl").exists()


def test_policy_on_an_interleaved_layout():
    policy = RebalanceByMeasurement(min_gain=0.03)
    # two ranks, two pieces each: rank 0 holds pieces 0 and 2, rank 1 pieces 1 and 3
    metrics = {"ranges": [(0, 2), (2, 4), (4, 6), (6, 8)], "busy_ms": [30.0, 10.0], "unit_costs": [1.0] * 8,
               "chunks": 2}
    moves = policy.propose(3, metrics)
    # measured 3:1 -> rank 0's units cost 7.5 each, rank 1's 2.5; the new pieces give each rank 20
    assert moves and policy.predicted_gain == pytest.approx(1 / 3)
    assert policy.last_ranges == [(0, 1), (1, 2), (2, 5), (5, 8)]
    assert owner_of([(0, 2), (2, 4), (4, 6), (6, 8)], 2) == {0: 0, 1: 0, 2: 1, 3: 1, 4: 0, 5: 0, 6: 1, 7: 1}


GPT6 = dict(GPT, layers=6)


def _train_interleaved(model, steps, switch_at=None, new_pieces=None, pieces=None):
    from meshtrain_b200.api import PipelineTrainer

    torch.set_num_threads(1)
    tr = PipelineTrainer(model, num_microbatches=4, optimizer="adam", lr=1e-3, device="cpu", microbatch_size=2,
                         partition=pieces or "equal", virtual_stages=2)
    losses = []
    for step in range(steps):
        if step == switch_at:
            tr.repartition(new_pieces)
        x, y = tr.spec.make_batch(step, 8)
        losses.append(tr.loss_value(tr.step(step, x, y)))
    params = tr.engine.named_parameters_cpu()
    pieces_now = [tuple(r) for r in tr.ranges]
    tr.close()
    return losses, params, pieces_now, []


def test_interleaved_repartition_mid_run_matches_the_new_split_from_the_start():
    new = [(0, 1), (1, 4), (4, 6), (6, 8)]  # the equal split of 8 units is (0,2),(2,4),(4,6),(6,8)
    ref = spawn_ranks(_train_interleaved, 2, GPT6, 4, pieces=new)
    moved = spawn_ranks(_train_interleaved, 2, GPT6, 4, switch_at=2, new_pieces=new)
    assert moved[0][2] == new
    assert moved[-1][0] == pytest.approx(ref[-1][0], rel=1e-6)
    want, got = _merged(ref), _merged(moved)
    for k, v in want.items():
        assert torch.allclose(got[k], v, rtol=1e-5, atol=1e-7), k
