"""Interleaved 1F1B: the per-rank programs, their ledger, and the split into pieces."""

import pytest

from meshtrain_b200.parallel.engine import interleaved_split
from meshtrain_b200.parallel.schedule import (ActionKind, ChunkLedger, SchedulerError, interleaved_schedule,
                                              simulate, simulate_interleaved, stage_schedule)


def _fmt(program):
    return " ".join(map(str, program))


def test_single_chunk_is_plain_1f1b():
    for S in (1, 2, 3, 5):
        for M in (1, 4, 7):
            for r in range(S):
                plain = [(a.kind, a.microbatch) for a in stage_schedule("1f1b", r, S, M)]
                inter = [(a.kind, a.microbatch) for a in interleaved_schedule(r, S, M, 1)]
                assert inter == plain
                assert all(a.chunk == 0 for a in interleaved_schedule(r, S, M, 1))


def test_two_chunk_programs_of_two_ranks():
    # microbatches in groups of S = 2; chunk 1 follows chunk 0 within a group; backwards walk the chunks back
    assert _fmt(interleaved_schedule(0, 2, 4, 2)) == "F0 F1 F0.1 F1.1 F2 B0.1 F3 B1.1 F2.1 B0 F3.1 B1 B2.1 B3.1 B2 B3"
    assert _fmt(interleaved_schedule(1, 2, 4, 2)) == "F0 F1 F0.1 B0.1 F1.1 B1.1 F2 B0 F3 B1 F2.1 B2.1 F3.1 B3.1 B2 B3"


@pytest.mark.parametrize("S,v", [(2, 2), (2, 3), (3, 2), (4, 2), (4, 4), (8, 2), (8, 3)])
def test_every_chunk_of_every_microbatch_once_forward_before_backward(S, v):
    M = 4 * S
    for r in range(S):
        prog = interleaved_schedule(r, S, M, v)
        assert len(prog) == 2 * v * M
        seen = set()
        for a in prog:
            key = (a.chunk, a.microbatch)
            if a.kind is ActionKind.FORWARD:
                assert key not in seen
                seen.add(key)
            else:
                assert key in seen
        assert seen == {(c, m) for c in range(v) for m in range(M)}


@pytest.mark.parametrize("S", [2, 3, 4, 8])
@pytest.mark.parametrize("v", [2, 3, 4])
def test_no_deadlock_and_smaller_bubble(S, v):
    M = 4 * S
    r = simulate_interleaved(S, M, v)
    assert r["complete"], (S, v)
    plain = simulate("1f1b", S, M)
    assert r["bubble_fraction"] < plain["bubble_fraction"]


def test_bubble_at_eight_ranks():
    # (S - 1) / (M + S - 1) for plain 1F1B; about half with two chunks
    assert simulate_interleaved(8, 32, 1)["bubble_fraction"] == pytest.approx(7 / 39, rel=1e-9)
    assert simulate_interleaved(8, 32, 2)["bubble_fraction"] < 0.11


def test_microbatches_must_fill_groups():
    with pytest.raises(ValueError):
        interleaved_schedule(0, 4, 6, 2)


def test_chunk_ledger_accepts_its_program_and_rejects_out_of_order():
    S, M, v = 3, 6, 2
    for r in range(S):
        led = ChunkLedger(r, S, M, 0, v)
        for a in led.actions:
            first = r == 0 and a.chunk == 0
            last = r == S - 1 and a.chunk == v - 1
            if a.kind is ActionKind.FORWARD and not first:
                led.input_arrived(a.chunk, a.microbatch)
            if a.kind is ActionKind.BACKWARD and not last:
                led.gradient_arrived(a.chunk, a.microbatch)
            led.run(a)
            led.finish(a)
        assert led.all_complete()
    led = ChunkLedger(1, S, M, 0, v)
    with pytest.raises(SchedulerError):
        led.run(led.actions[1])
    with pytest.raises(SchedulerError):  # first action of rank 1 needs its input
        led.run(led.actions[0])


def test_interleaved_split_is_contiguous_and_balances_ranks():
    costs = [1.0] + [5.0, 4.0] * 24 + [12.0]  # embedding, 24 blocks as halves, an expensive head
    for S, v in ((2, 2), (4, 2), (8, 2)):
        pieces = interleaved_split(costs, S, v)
        assert len(pieces) == S * v
        assert pieces[0][0] == 0 and pieces[-1][1] == len(costs)
        assert all(a < b for a, b in pieces) and all(pieces[i][1] == pieces[i + 1][0] for i in range(len(pieces) - 1))
        cost = [sum(costs[a:b]) for a, b in pieces]
        per_rank = [sum(cost[r::S]) for r in range(S)]
        assert max(per_rank) <= 1.15 * sum(costs) / S  # pieces are whole units of 4-5


def test_interleaved_memory_estimate_per_rank():
    from meshtrain_b200.api import check_interleaved_memory
    from meshtrain_b200.models import build_model_spec
    from meshtrain_b200.planner.graph import analytic_layer_flops

    spec = build_model_spec({"type": "gpt", "layers": 24, "hidden_size": 1280, "heads": 20, "vocab_size": 50257,
                             "seq_len": 2048, "dtype": "bfloat16", "split_blocks": True})
    pieces = interleaved_split(analytic_layer_flops(spec), 8, 2)
    ests = check_interleaved_memory(spec, pieces, 8, 2, 32, 4, "adam", memory_gb=180.0)
    assert len(ests) == 8 and all(e.fits for e in ests)
    # rank 0 keeps the most chunk-forwards alive
    assert ests[0].saved_activations >= ests[-1].saved_activations
    with pytest.raises(RuntimeError, match="does not fit"):
        check_interleaved_memory(spec, pieces, 8, 2, 32, 4, "adam", memory_gb=2.0)


def test_simulation_with_piece_costs():
    # equal pieces reproduce the unit-cost simulation
    uniform = simulate_interleaved(4, 8, 2)
    pieces = simulate_interleaved(4, 8, 2, piece_costs=[0.5] * 8)
    assert pieces["makespan"] == pytest.approx(uniform["makespan"])
    # one heavy piece lengthens the step
    heavy = simulate_interleaved(4, 8, 2, piece_costs=[0.5] * 7 + [1.0])
    assert heavy["makespan"] > uniform["makespan"]
    with pytest.raises(ValueError):
        simulate_interleaved(4, 8, 2, piece_costs=[1.0] * 3)


def test_interleaving_forecast():
    from meshtrain_b200.api import forecast_interleaving

    rows = forecast_interleaving([1.0] * 48, 8, 32, chunk_options=(1, 2, 3))
    assert [r["chunks"] for r in rows] == [1, 2, 3]
    assert rows[0]["bubble_fraction"] == pytest.approx(7 / 39, rel=1e-6)
    assert rows[0]["relative_step"] == 1.0
    assert rows[2]["bubble_fraction"] < rows[1]["bubble_fraction"] < rows[0]["bubble_fraction"]
    assert all(r["rank_imbalance"] == pytest.approx(1.0) for r in rows)
    # microbatches not a multiple of the ranks: only the plain program is forecast
    assert [r["chunks"] for r in forecast_interleaving([1.0] * 48, 8, 30)] == [1]
