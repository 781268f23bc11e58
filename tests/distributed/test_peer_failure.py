"""A pipeline rank that fails between steps stops every other rank with an error.

Runs the device engine as gloo ranks on the CPU: rank ``victim`` raises when it
starts step 2 (nothing of that step launched), reports through the job's store
and exits; the other ranks must end with an error well inside the peer timeout
instead of blocking in a receive.  The 2-GPU NCCL variant lives in
tests/test_peer_failure_gpu.py.
"""

import time

import pytest

from meshtrain_b200.parallel.spawn import spawn_ranks

GPT = {"type": "gpt", "layers": 3, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32,
       "dtype": "float32"}


def _run_until_failure(victim: int, fail_at: int, device: str = "cpu"):
    from meshtrain_b200.api import PipelineTrainer

    trainer = PipelineTrainer(GPT, num_microbatches=2, optimizer="adam", lr=1e-3, device=device, microbatch_size=2,
                              link_probe=False)
    if trainer.rank == victim:
        real = trainer.engine.train_step

        def failing(step, *args, **kwargs):
            if step == fail_at:
                raise RuntimeError("injected failure before launching the step")
            return real(step, *args, **kwargs)
        trainer.engine.train_step = failing
    outcome = {"rank": trainer.rank, "error": None, "steps": 0}
    t0 = time.monotonic()
    try:
        for step in range(6):
            x, y = trainer.spec.make_batch(step, 4)
            trainer.step(step, x, y)
            outcome["steps"] += 1
    except Exception as exc:  # noqa: BLE001 - the outcome is what the test checks
        outcome.update(error=type(exc).__name__, message=str(exc)[:300])
    outcome["seconds"] = time.monotonic() - t0
    if trainer.rank == victim:
        time.sleep(3)  # rank 0 hosts the job's store here: keep it up while the others read the report
    trainer.close()
    return outcome


@pytest.mark.parametrize("victim", [0, 1, 2])
def test_failure_of_one_rank_stops_all_ranks(victim):
    env = {"MESHTRAIN_PG_TIMEOUT_S": "30", "MESHTRAIN_PEER_TIMEOUT_S": "10"}
    outcomes = spawn_ranks(_run_until_failure, 3, victim, 2, env=env, timeout_s=120)
    assert outcomes[victim]["error"] == "RuntimeError" and outcomes[victim]["steps"] == 2
    for o in outcomes:
        assert o["error"] is not None, o          # nobody trains on past the failure
        assert o["steps"] <= 3, o                  # at most the step that was in flight
        assert o["seconds"] < 25, o                # well inside the process-group timeout
    survivors = [o for i, o in enumerate(outcomes) if i != victim]
    assert any(o["error"] == "PeerFailure" and f"rank {victim}" in o["message"] for o in survivors), survivors
