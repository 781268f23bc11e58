"""Schedules (programs per stage) and the step ledger that enforces the protocol."""

import itertools
import random

import pytest

from meshtrain_b200.parallel.schedule import (Action, ActionKind, SchedulerError, StepLedger, format_schedule,
                                              max_inflight_of, simulate, stage_schedule, warmup_forwards)

F, B = ActionKind.FORWARD, ActionKind.BACKWARD


def _prog(text: str) -> list[Action]:
    return [Action(F if t[0] == "F" else B, int(t[1:])) for t in text.split()]


# ------------------------------------------------------------------ programs
def test_canonical_orders():
    # GPipe: all forwards then all backwards; the last stage alternates (its loss is local)
    assert stage_schedule("gpipe", 0, 3, 4) == _prog("F0 F1 F2 F3 B0 B1 B2 B3")
    assert stage_schedule("gpipe", 2, 3, 4) == _prog("F0 B0 F1 B1 F2 B2 F3 B3")
    # 1F1B with S=3, M=6: warm-up 2 / 1 / 0 forwards
    assert format_schedule(stage_schedule("1f1b", 0, 3, 6)) == "F0 F1 F2 B0 F3 B1 F4 B2 F5 B3 B4 B5"
    assert format_schedule(stage_schedule("1f1b", 1, 3, 6)) == "F0 F1 B0 F2 B1 F3 B2 F4 B3 F5 B4 B5"
    assert format_schedule(stage_schedule("1f1b", 2, 3, 6)) == "F0 B0 F1 B1 F2 B2 F3 B3 F4 B4 F5 B5"


def _reference_1f1b(stage, S, M, cap=None):
    """The textbook three-phase construction: warm-up, steady 1F1B, cool-down."""
    w = warmup_forwards("1f1b", stage, S, M, cap)
    out = [Action(F, m) for m in range(w)]
    for i in range(M - w):
        out += [Action(F, w + i), Action(B, i)]
    return out + [Action(B, m) for m in range(M - w, M)]


@pytest.mark.parametrize("S,M,cap", list(itertools.product(range(1, 9), (1, 2, 5, 8, 32), (None, 1, 2, 3))))
def test_budget_rule_equals_three_phase_1f1b(S, M, cap):
    for s in range(S):
        assert stage_schedule("1f1b", s, S, M, cap) == _reference_1f1b(s, S, M, cap)


@pytest.mark.parametrize("schedule", ["gpipe", "1f1b"])
@pytest.mark.parametrize("S,M", [(1, 1), (1, 4), (2, 1), (2, 8), (3, 2), (4, 16), (5, 3), (8, 32)])
def test_every_microbatch_forward_then_backward_once(schedule, S, M):
    for s in range(S):
        prog = stage_schedule(schedule, s, S, M)
        assert len(prog) == 2 * M and len(set(prog)) == 2 * M
        pos = {a: i for i, a in enumerate(prog)}
        assert all(pos[Action(F, m)] < pos[Action(B, m)] for m in range(M))
        # backwards leave in microbatch order (the upstream stage receives them FIFO)
        assert [a.microbatch for a in prog if a.kind is B] == list(range(M))


@pytest.mark.parametrize("S,M", [(2, 8), (3, 8), (4, 16), (8, 32)])
def test_contexts_held_per_stage(S, M):
    for s in range(S):
        assert max_inflight_of(stage_schedule("gpipe", s, S, M)) == (M if s < S - 1 else 1)
        assert max_inflight_of(stage_schedule("1f1b", s, S, M)) == min(S - s, M)
        for cap in (1, 2, 3):
            assert max_inflight_of(stage_schedule("1f1b", s, S, M, max_inflight=cap)) <= cap


def test_warmup_never_grows_down_the_pipeline():
    for S, M, cap in itertools.product(range(1, 9), range(1, 12), (None, 1, 2, 3)):
        w = [warmup_forwards("1f1b", s, S, M, cap) for s in range(S)]
        assert w == sorted(w, reverse=True)


@pytest.mark.parametrize("schedule", ["gpipe", "1f1b"])
def test_no_deadlock(schedule):
    for S, M in itertools.product(range(1, 8), range(1, 14)):
        for cap in ((None,) if schedule == "gpipe" else (None, 1, 2, 3)):
            assert simulate(schedule, S, M, cap)["complete"], (schedule, S, M, cap)


def test_simulator_detects_a_deadlock():
    import meshtrain_b200.parallel.schedule as sched

    real = sched.stage_schedule

    def backwards_first(schedule, stage, S, M, cap=None):
        prog = real(schedule, stage, S, M, cap)
        return sorted(prog, key=lambda a: a.kind is F) if stage == 0 else prog

    sched.stage_schedule = backwards_first
    try:
        assert not simulate("1f1b", 2, 2)["complete"]
    finally:
        sched.stage_schedule = real


def test_bubble_matches_closed_form():
    # unit costs F=1, B=2: bubble = (S-1) / (M+S-1) for both schedules
    for S, M in [(2, 4), (4, 8), (4, 32), (8, 32)]:
        for name in ("gpipe", "1f1b"):
            assert simulate(name, S, M)["bubble_fraction"] == pytest.approx((S - 1) / (M + S - 1))


def test_unknown_schedule_and_bad_counts():
    with pytest.raises(ValueError):
        stage_schedule("zero-bubble", 0, 2, 2)
    with pytest.raises(ValueError):
        stage_schedule("1f1b", 2, 2, 4)
    with pytest.raises(ValueError):
        stage_schedule("1f1b", 0, 2, 0)


# ------------------------------------------------------------------ ledger
def _run(ledger, action):
    ledger.run(action)
    ledger.finish(action)


def test_ledger_middle_stage_lifecycle():
    lg = StepLedger(1, 3, 2, step=0, schedule="1f1b")
    a = lg.next_action()
    assert a == Action(F, 0) and not lg.ready(a)
    with pytest.raises(SchedulerError, match="not ready"):
        lg.run(a)
    lg.input_arrived(0)
    _run(lg, a)
    lg.forward_sent(0)
    assert lg.describe(0) == "input+forward+sent"
    lg.input_arrived(1)
    _run(lg, lg.next_action())           # F1 (warm-up of 1 on stage 1 of 3)
    b0 = lg.next_action()
    assert b0 == Action(B, 0) and not lg.ready(b0)
    lg.gradient_arrived(0)
    _run(lg, b0)
    assert lg.inflight == 1 and lg.peak_inflight == 2 and not lg.all_complete()


def test_ledger_rejects_protocol_violations():
    lg = StepLedger(1, 3, 2, step=0)
    with pytest.raises(SchedulerError, match="before its forward"):
        lg.gradient_arrived(0)
    lg.input_arrived(0)
    with pytest.raises(SchedulerError, match="duplicate activation"):
        lg.input_arrived(0)
    with pytest.raises(SchedulerError, match="unknown microbatch"):
        lg.input_arrived(9)
    with pytest.raises(SchedulerError, match="not the next action"):
        lg.run(Action(B, 0))
    _run(lg, Action(F, 0))
    lg.gradient_arrived(0)
    with pytest.raises(SchedulerError, match="duplicate gradient"):
        lg.gradient_arrived(0)


def test_gradient_may_arrive_before_the_send_completes():
    lg = StepLedger(0, 2, 1, step=0)
    _run(lg, Action(F, 0))
    lg.gradient_arrived(0)                # the peer answered before our send callback ran
    assert lg.ready(Action(B, 0))
    lg.forward_sent(0)
    _run(lg, Action(B, 0))
    assert lg.done and lg.all_complete()


def test_last_stage_needs_no_gradient_message():
    lg = StepLedger(1, 2, 2, step=0, schedule="gpipe")
    for m in range(2):
        lg.input_arrived(m)
        _run(lg, Action(F, m))
        _run(lg, Action(B, m))
    assert lg.done and lg.all_complete()
    assert lg.snapshot()["next_action"] is None


@pytest.mark.parametrize("schedule", ["gpipe", "1f1b"])
def test_ledgers_of_a_whole_pipeline_complete_under_random_delivery(schedule):
    rng = random.Random(3)
    S, M = 4, 6
    ledgers = [StepLedger(s, S, M, 0, schedule) for s in range(S)]
    in_flight = []  # (stage, "input"|"grad", mb) messages not yet delivered
    for _ in range(10_000):
        if all(lg.done for lg in ledgers):
            break
        if in_flight and rng.random() < 0.5:
            s, kind, m = in_flight.pop(rng.randrange(len(in_flight)))
            (ledgers[s].input_arrived if kind == "input" else ledgers[s].gradient_arrived)(m)
            continue
        for s, lg in enumerate(ledgers):
            a = lg.next_action()
            if a is not None and lg.ready(a):
                _run(lg, a)
                if a.kind is F and s < S - 1:
                    in_flight.append((s + 1, "input", a.microbatch))
                if a.kind is B and s > 0:
                    in_flight.append((s - 1, "grad", a.microbatch))
    assert all(lg.all_complete() for lg in ledgers)
