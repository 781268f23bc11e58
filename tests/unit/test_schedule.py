import itertools

import pytest

from meshtrain_b200.parallel.schedule import (ActionKind, Event, MicrobatchState, SchedulerError, StageStateMachine,
                                              format_schedule, max_inflight_of, simulate, stage_schedule,
                                              warmup_forwards)


def test_gpipe_orders():
    assert format_schedule(stage_schedule("gpipe", 0, 3, 4)) == "F0 F1 F2 F3 B0 B1 B2 B3"
    assert format_schedule(stage_schedule("gpipe", 2, 3, 4)) == "F0 B0 F1 B1 F2 B2 F3 B3"


def test_1f1b_three_stages_six_microbatches():
    assert format_schedule(stage_schedule("1f1b", 0, 3, 6)) == "F0 F1 F2 B0 F3 B1 F4 B2 F5 B3 B4 B5"
    assert format_schedule(stage_schedule("1f1b", 1, 3, 6)) == "F0 F1 B0 F2 B1 F3 B2 F4 B3 F5 B4 B5"
    assert format_schedule(stage_schedule("1f1b", 2, 3, 6)) == "F0 B0 F1 B1 F2 B2 F3 B3 F4 B4 F5 B5"


@pytest.mark.parametrize("schedule", ["gpipe", "1f1b"])
@pytest.mark.parametrize("S,M", [(1, 1), (1, 4), (2, 1), (2, 8), (3, 2), (4, 16), (5, 3), (8, 32)])
def test_each_microbatch_once_forward_first(schedule, S, M):
    for s in range(S):
        acts = stage_schedule(schedule, s, S, M)
        fwd = [a.microbatch for a in acts if a.kind is ActionKind.FORWARD]
        bwd = [a.microbatch for a in acts if a.kind is ActionKind.BACKWARD]
        assert sorted(fwd) == list(range(M)) and sorted(bwd) == list(range(M))
        for m in range(M):
            assert acts.index(next(a for a in acts if a.kind is ActionKind.FORWARD and a.microbatch == m)) < \
                acts.index(next(a for a in acts if a.kind is ActionKind.BACKWARD and a.microbatch == m))


@pytest.mark.parametrize("S,M", [(2, 8), (3, 8), (4, 16)])
def test_inflight_bounds(S, M):
    for s in range(S):
        assert max_inflight_of(stage_schedule("gpipe", s, S, M)) == (M if s < S - 1 else 1)
        assert max_inflight_of(stage_schedule("1f1b", s, S, M)) == min(S - s, M)
        assert max_inflight_of(stage_schedule("1f1b", s, S, M, max_inflight=2)) <= 2


def test_warmup_is_monotone_in_stage():
    for S, M, cap in itertools.product(range(1, 8), range(1, 10), (None, 1, 2, 3)):
        w = [warmup_forwards("1f1b", s, S, M, cap) for s in range(S)]
        assert all(a >= b for a, b in zip(w, w[1:]))


@pytest.mark.parametrize("schedule", ["gpipe", "1f1b"])
def test_deadlock_free(schedule):
    for S, M in itertools.product(range(1, 7), range(1, 13)):
        for cap in (None, 1, 2, 3):
            res = simulate(schedule, S, M, cap if schedule == "1f1b" else None)
            assert res["complete"], (schedule, S, M, cap)


def test_bubble_fraction_matches_closed_form():
    # unit costs F=1, B=2: bubble = (S-1) / (M + S - 1) for both schedules
    for S, M in [(2, 4), (4, 8), (4, 32)]:
        for sched in ("gpipe", "1f1b"):
            res = simulate(sched, S, M)
            assert res["bubble_fraction"] == pytest.approx((S - 1) / (M + S - 1))


def test_state_machine_middle_stage():
    sm = StageStateMachine(1, 3, 2, step=0, schedule="1f1b")
    a = sm.next_action()
    assert a.kind is ActionKind.FORWARD and not sm.ready(a)
    sm.on(Event.ACTIVATION_RECEIVED, 0)
    assert sm.ready(a)
    sm.on(Event.FORWARD_STARTED, 0)
    sm.on(Event.FORWARD_FINISHED, 0)
    sm.on(Event.SEND_COMPLETED, 0)
    assert sm.mbs[0].state is MicrobatchState.SENT_FORWARD
    sm.on(Event.GRADIENT_RECEIVED, 0)
    sm.on(Event.BACKWARD_STARTED, 0)
    sm.on(Event.BACKWARD_FINISHED, 0)
    assert sm.mbs[0].state is MicrobatchState.COMPLETE and sm.inflight == 0 and sm.peak_inflight == 1


def test_state_machine_rejects_violations():
    sm = StageStateMachine(1, 3, 2, step=0)
    with pytest.raises(SchedulerError, match="gradient"):
        sm.on(Event.GRADIENT_RECEIVED, 0)
    sm.on(Event.ACTIVATION_RECEIVED, 0)
    with pytest.raises(SchedulerError, match="duplicate"):
        sm.on(Event.ACTIVATION_RECEIVED, 0)
    with pytest.raises(SchedulerError, match="unknown"):
        sm.on(Event.ACTIVATION_RECEIVED, 9)
    with pytest.raises(SchedulerError, match="expected"):
        sm.on(Event.BACKWARD_STARTED, 0)


def test_gradient_before_send_completion():
    sm = StageStateMachine(0, 2, 1, step=0)
    sm.on(Event.FORWARD_STARTED, 0)
    sm.on(Event.FORWARD_FINISHED, 0)
    sm.on(Event.GRADIENT_RECEIVED, 0)
    assert sm.ready(sm.actions[1])
    sm.on(Event.SEND_COMPLETED, 0)
    assert sm.mbs[0].state is MicrobatchState.BACKWARD_READY


def test_unknown_schedule():
    with pytest.raises(ValueError):
        stage_schedule("zero-bubble", 0, 2, 2)
