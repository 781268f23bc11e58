"""Stream ordering over NCCL under a forced delay on one GPU rank.

One rank of a 2-GPU bf16 pipeline spins its compute stream (``torch.cuda._sleep``)
before each forward, or before each receive buffer is allocated, so its sends
leave late or its receives are consumed late while the other rank runs ahead.
If a receive buffer were reused before it was read, or a sent tensor freed
before its transfer finished, the result would change by far more than the
run-to-run noise of the attention dQ reductions; it must match the undelayed
run.  Also run with two model chunks per rank (the wrap-around link).
"""

import pytest
import torch

from meshtrain_b200.parallel.spawn import spawn_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

MODEL = {"type": "gpt", "layers": 6, "hidden_size": 256, "heads": 4, "vocab_size": 1000, "seq_len": 256,
         "dtype": "bfloat16", "init_std": 0.02, "data": "uniform"}


def _train(steps, delay_rank, where, virtual_stages):
    from meshtrain_b200 import ops
    from meshtrain_b200.api import PipelineTrainer

    ops.set_backend("custom")
    tr = PipelineTrainer(MODEL, num_microbatches=4, optimizer="sgd", lr=0.05, microbatch_size=2,
                         virtual_stages=virtual_stages)
    if delay_rank == tr.rank:
        eng = tr.engine
        cycles = 2_000_000  # about a millisecond of the compute stream's time per call
        if where == "forward":
            real = eng._forward_layers

            def late_forward(*args, **kwargs):
                torch.cuda._sleep(cycles)
                return real(*args, **kwargs)
            eng._forward_layers = late_forward
        else:
            real_buf = eng._recv_buf

            def late_consumer(*args, **kwargs):
                torch.cuda._sleep(cycles)
                return real_buf(*args, **kwargs)
            eng._recv_buf = late_consumer
    losses = []
    for step in range(steps):
        x, y = tr.spec.make_batch(step, 8)
        losses.append(tr.loss_value(tr.step(step, x.pin_memory(), y.pin_memory())))
    torch.cuda.synchronize()
    status = ops.read_status(torch.cuda.current_device())
    params = tr.engine.named_parameters_cpu()
    tr.close()
    return losses, params, status


@pytest.mark.parametrize("delay_rank,where,chunks", [(0, "forward", 1), (1, "receive", 1), (1, "receive", 2)])
def test_late_rank_over_nccl_changes_nothing(delay_rank, where, chunks):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    plain = spawn_ranks(_train, 2, 3, None, where, chunks)
    late = spawn_ranks(_train, 2, 3, delay_rank, where, chunks)
    assert all(r[2] == 0 for r in plain + late)
    assert late[-1][0] == pytest.approx(plain[-1][0], rel=2e-3)
    for r in range(2):
        for k, v in plain[r][1].items():
            assert torch.allclose(late[r][1][k], v, rtol=2e-2, atol=2e-4), k
