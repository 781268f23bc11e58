"""NCCL pipelines on 2 and 4 GPUs give the single-GPU result (same kernels, same order).

Each rank runs one stage of a small bf16 GPT through the hand-written kernels;
activations and their gradients cross between GPUs as NCCL send/recv.  Loss
trajectory and final fp32 master weights are compared with one GPU running
every layer.
"""

import pytest
import torch

from meshtrain_b200.parallel.spawn import spawn_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

MODEL = {"type": "gpt", "layers": 6, "hidden_size": 256, "heads": 4, "vocab_size": 1000, "seq_len": 256,
         "dtype": "bfloat16", "init_std": 0.02, "data": "uniform"}


def _train(steps, M, mbs, schedule, partition, model=None):
    from meshtrain_b200 import ops
    from meshtrain_b200.api import PipelineTrainer

    ops.set_backend("custom")
    # SGD: parameter differences stay proportional to gradient differences (Adam's
    # normalised update turns last-bit gradient noise on near-zero entries into
    # differences of up to lr per step, which says nothing about the pipeline)
    tr = PipelineTrainer(model or MODEL, num_microbatches=M, schedule=schedule, optimizer="sgd", lr=0.05,
                         microbatch_size=mbs, partition=partition)
    losses = []
    for step in range(steps):
        x, y = tr.spec.make_batch(step, M * mbs)
        st = tr.step(step, x.pin_memory(), y.pin_memory(), timed=True)
        losses.append(tr.loss_value(st))
        assert 0.0 <= st.bubble_fraction <= 1.0
    torch.cuda.synchronize()
    status = ops.read_status(torch.cuda.current_device())
    params = tr.engine.named_parameters_cpu()
    tr.close()
    return losses, params, status


@pytest.mark.parametrize("world,schedule", [(2, "1f1b"), (4, "1f1b"), (4, "gpipe")])
def test_nccl_pipeline_matches_one_gpu(world, schedule):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ranges = [[0, 2], [2, 4], [4, 6], [6, 8]][:world] if world == 4 else [[0, 4], [4, 8]]
    single = spawn_ranks(_train, 1, 4, 4, 2, schedule, [[0, 8]])[0]
    again = spawn_ranks(_train, 1, 4, 4, 2, schedule, [[0, 8]])[0]
    ranked = spawn_ranks(_train, world, 4, 4, 2, schedule, ranges)
    assert all(r[2] == 0 for r in ranked) and single[2] == 0 and again[2] == 0
    losses = ranked[-1][0]
    assert losses == pytest.approx(single[0], rel=1e-5), (losses, single[0])
    merged = {}
    for _, params, _ in ranked:
        merged.update(params)
    assert set(merged) == set(single[1])
    # Several backward kernels accumulate with fp32 atomics / bulk reduce-adds whose order
    # varies from run to run, so the pipeline must agree with one GPU as closely as one
    # GPU agrees with itself on a second run (with a small floor for runs that match).
    for k, v in single[1].items():
        noise = (again[1][k] - v).abs()
        d = (merged[k] - v).abs()
        floor = 1e-4 * v.abs().max().item() + 1e-7  # when the two one-GPU runs happen to agree bit for bit
        assert d.max().item() <= max(4 * noise.max().item(), floor), (k, d.max().item(), noise.max().item())
        assert d.mean().item() <= max(4 * noise.mean().item(), floor / 100), (k, d.mean().item(), noise.mean().item())


def test_boundary_inside_a_block_over_nccl():
    """Half-block units: stage 0 ends with block 2's attention half, stage 1 starts with its MLP half."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    split = dict(MODEL, split_blocks=True)
    single = spawn_ranks(_train, 1, 3, 4, 2, "1f1b", [[0, 8]])[0]
    again = spawn_ranks(_train, 1, 3, 4, 2, "1f1b", [[0, 8]])[0]
    ranked = spawn_ranks(_train, 2, 3, 4, 2, "1f1b", [[0, 6], [6, 14]], split)
    assert all(r[2] == 0 for r in ranked)
    assert ranked[-1][0] == pytest.approx(single[0], rel=1e-5), (ranked[-1][0], single[0])
    merged = {}
    for _, params, _ in ranked:
        assert not set(params) & set(merged)
        merged.update(params)
    assert set(merged) == set(single[1])
    for k, v in single[1].items():
        noise = (again[1][k] - v).abs()
        d = (merged[k] - v).abs()
        floor = 1e-4 * v.abs().max().item() + 1e-7  # when the two one-GPU runs happen to agree bit for bit
        assert d.max().item() <= max(4 * noise.max().item(), floor), (k, d.max().item(), noise.max().item())
