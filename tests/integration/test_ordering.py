"""Determinism and stream-ordering checks of the device engine on CPU ranks.

* Two identical runs of a 2-rank fp32 pipeline give bit-identical losses and
  parameters (no reduction whose order depends on timing).
* A rank that runs late - a sleep before each of its forwards, or after each
  of its receives - changes nothing: messages are matched by order on their
  communicator, receive buffers are never reused before they are read, and a
  send's tensor stays alive until the transfer is done.
"""

import time

import pytest
import torch

from meshtrain_b200.parallel.spawn import spawn_ranks

GPT = {"type": "gpt", "layers": 4, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32,
       "dtype": "float32"}


def _run(steps: int, delay_rank: int | None = None, where: str = "forward", seconds: float = 0.02,
         virtual_stages: int = 1):
    from meshtrain_b200.api import PipelineTrainer

    # one intra-op thread: CPU scatter-adds (the embedding gradient) then sum in a fixed order
    torch.set_num_threads(1)
    tr = PipelineTrainer(GPT, num_microbatches=4, optimizer="adam", lr=1e-3, device="cpu", microbatch_size=2,
                         virtual_stages=virtual_stages)
    if delay_rank == tr.rank:
        eng = tr.engine
        if where == "forward":
            real = eng._forward_layers

            def late_forward(*args, **kwargs):
                time.sleep(seconds)  # the producer runs late: its peers wait on their receives
                return real(*args, **kwargs)
            eng._forward_layers = late_forward
        else:
            real_buf = eng._recv_buf

            def late_consumer(*args, **kwargs):
                time.sleep(seconds)  # receives are posted late and consumed late
                return real_buf(*args, **kwargs)
            eng._recv_buf = late_consumer
    losses = []
    for step in range(steps):
        x, y = tr.spec.make_batch(step, 8)
        losses.append(tr.loss_value(tr.step(step, x, y)))
    params = tr.engine.named_parameters_cpu()
    tr.close()
    return losses, params


def _same(a, b):
    (la, pa), (lb, pb) = a, b
    assert la == lb  # bit-identical, not approximately equal
    assert set(pa) == set(pb)
    for k in pa:
        assert torch.equal(pa[k], pb[k]), k


def test_two_runs_are_bit_identical():
    first = spawn_ranks(_run, 2, 3)
    second = spawn_ranks(_run, 2, 3)
    for r in range(2):
        _same(first[r], second[r])


@pytest.mark.parametrize("delay_rank,where", [(0, "forward"), (1, "forward"), (1, "receive"), (0, "receive")])
def test_a_late_rank_changes_nothing(delay_rank, where):
    plain = spawn_ranks(_run, 2, 2)
    late = spawn_ranks(_run, 2, 2, delay_rank, where)
    for r in range(2):
        _same(plain[r], late[r])


def test_a_late_rank_in_an_interleaved_pipeline_changes_nothing():
    plain = spawn_ranks(_run, 2, 2, None, "forward", 0.0, 2)
    late = spawn_ranks(_run, 2, 2, 1, "receive", 0.02, 2)
    for r in range(2):
        _same(plain[r], late[r])
