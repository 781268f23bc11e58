"""Pipeline schedules and the per-stage microbatch state machine.

For one stage and one global step a schedule is the ordered list of
``F<m>`` / ``B<m>`` actions that stage performs (reference
runtime/scheduler.py:61-98):

* ``gpipe``: every forward, then every backward; the last stage alternates
  F/B because its loss is local.
* ``1f1b`` (PipeDream-flush): ``w_s = min(S-s-1, cap-1, M)`` warm-up
  forwards, then alternating F/B, then the remaining backwards.  Stage s holds
  at most ``min(S-s, cap, M)`` microbatch contexts.  Deadlock freedom:
  ``w_{s+1} <= w_s``, so stage s+1 can always emit its first gradient after
  stage s has sent the forwards it needs.

The schedule only reorders work inside one parameter version: one optimizer
step per global step, loss scaled by 1/M, gradients accumulated.

``StageStateMachine`` tracks each microbatch through QUEUED -> FORWARD_READY
-> FORWARD_RUNNING -> FORWARD_DONE -> SENT_FORWARD -> BACKWARD_READY ->
BACKWARD_RUNNING -> COMPLETE and rejects illegal transitions (duplicate
activations/gradients, gradient before forward, unknown microbatch).
"""

from __future__ import annotations

import enum
from dataclasses import dataclass, field


class ActionKind(str, enum.Enum):
    FORWARD = "F"
    BACKWARD = "B"


@dataclass(frozen=True)
class Action:
    kind: ActionKind
    microbatch: int

    def __str__(self) -> str:
        return f"{self.kind.value}{self.microbatch}"


SCHEDULES = ("gpipe", "1f1b")


def warmup_forwards(schedule: str, stage: int, num_stages: int, num_microbatches: int,
                    max_inflight: int | None = None) -> int:
    """Forwards a stage runs before its first backward."""
    if schedule == "gpipe":
        return num_microbatches if stage < num_stages - 1 else 0
    cap = num_microbatches if max_inflight is None else max(1, max_inflight)
    return max(0, min(num_stages - stage - 1, cap - 1, num_microbatches))


def stage_schedule(schedule: str, stage: int, num_stages: int, num_microbatches: int,
                   max_inflight: int | None = None) -> list[Action]:
    if schedule not in SCHEDULES:
        raise ValueError(f"unknown schedule {schedule!r}; expected one of {SCHEDULES}")
    if not 0 <= stage < num_stages or num_microbatches < 1:
        raise ValueError("invalid stage/microbatch counts")
    M = num_microbatches
    fwd = [Action(ActionKind.FORWARD, m) for m in range(M)]
    bwd = [Action(ActionKind.BACKWARD, m) for m in range(M)]
    if schedule == "gpipe" and stage < num_stages - 1:
        return fwd + bwd
    w = warmup_forwards(schedule, stage, num_stages, M, max_inflight)
    out = fwd[:w]
    for i in range(M - w):
        out.append(fwd[w + i])
        out.append(bwd[i])
    out.extend(bwd[M - w:])
    return out


def max_inflight_of(actions: list[Action]) -> int:
    """Peak number of microbatches forwarded but not yet backwarded."""
    live = peak = 0
    for a in actions:
        live += 1 if a.kind == ActionKind.FORWARD else -1
        peak = max(peak, live)
    return peak


def format_schedule(actions: list[Action]) -> str:
    return " ".join(str(a) for a in actions)


def simulate(schedule: str, num_stages: int, num_microbatches: int, max_inflight: int | None = None,
             fwd_cost: float = 1.0, bwd_cost: float = 2.0) -> dict:
    """Dependency simulation of a whole pipeline (unit-cost model).

    Returns the makespan, per-stage busy time, the bubble fraction and whether
    the schedule completes (deadlock detection).
    """
    S, M = num_stages, num_microbatches
    sched = [stage_schedule(schedule, s, S, M, max_inflight) for s in range(S)]
    cursor = [0] * S
    clock = [0.0] * S
    f_done: dict[tuple[int, int], float] = {}
    b_done: dict[tuple[int, int], float] = {}
    busy = [0.0] * S
    progressed = True
    while progressed:
        progressed = False
        for s in range(S):
            while cursor[s] < len(sched[s]):
                a = sched[s][cursor[s]]
                m = a.microbatch
                if a.kind == ActionKind.FORWARD:
                    dep = 0.0 if s == 0 else f_done.get((s - 1, m))
                    cost = fwd_cost
                else:
                    if s == S - 1:
                        dep = f_done.get((s, m))
                    else:
                        dep = b_done.get((s + 1, m))
                    cost = bwd_cost
                if dep is None:
                    break
                start = max(clock[s], dep)
                clock[s] = start + cost
                busy[s] += cost
                (f_done if a.kind == ActionKind.FORWARD else b_done)[(s, m)] = clock[s]
                cursor[s] += 1
                progressed = True
    complete = all(cursor[s] == len(sched[s]) for s in range(S))
    makespan = max(clock) if complete else float("inf")
    return {
        "complete": complete,
        "makespan": makespan,
        "busy": busy,
        "bubble_fraction": (1.0 - sum(busy) / (S * makespan)) if complete and makespan > 0 else None,
    }


class MicrobatchState(str, enum.Enum):
    QUEUED = "QUEUED"
    FORWARD_READY = "FORWARD_READY"
    FORWARD_RUNNING = "FORWARD_RUNNING"
    FORWARD_DONE = "FORWARD_DONE"
    SENT_FORWARD = "SENT_FORWARD"
    BACKWARD_READY = "BACKWARD_READY"
    BACKWARD_RUNNING = "BACKWARD_RUNNING"
    BACKWARD_DONE = "BACKWARD_DONE"
    COMPLETE = "COMPLETE"


class Event(str, enum.Enum):
    ACTIVATION_RECEIVED = "ACTIVATION_RECEIVED"
    FORWARD_STARTED = "FORWARD_STARTED"
    FORWARD_FINISHED = "FORWARD_FINISHED"
    GRADIENT_RECEIVED = "GRADIENT_RECEIVED"
    BACKWARD_STARTED = "BACKWARD_STARTED"
    BACKWARD_FINISHED = "BACKWARD_FINISHED"
    SEND_COMPLETED = "SEND_COMPLETED"


class SchedulerError(RuntimeError):
    pass


@dataclass
class _MB:
    state: MicrobatchState = MicrobatchState.QUEUED
    have_input: bool = False
    have_grad: bool = False
    forward_sent: bool = False
    history: list[str] = field(default_factory=list)


class StageStateMachine:
    """Per-stage, per-step microbatch states plus a cursor into the schedule."""

    def __init__(self, stage: int, num_stages: int, num_microbatches: int, step: int,
                 schedule: str = "gpipe", max_inflight: int | None = None):
        self.stage, self.num_stages, self.step = stage, num_stages, step
        self.is_first, self.is_last = stage == 0, stage == num_stages - 1
        self.actions = stage_schedule(schedule, stage, num_stages, num_microbatches, max_inflight)
        self.cursor = 0
        self.mbs = {m: _MB() for m in range(num_microbatches)}
        self.inflight = 0
        self.peak_inflight = 0
        if self.is_first:  # the first stage owns the data
            for st in self.mbs.values():
                st.have_input = True
                st.state = MicrobatchState.FORWARD_READY

    def on(self, event: Event, mb: int) -> None:
        st = self.mbs.get(mb)
        if st is None:
            raise SchedulerError(f"event {event.value} for unknown microbatch {mb}")
        st.history.append(event.value)
        S = MicrobatchState
        if event is Event.ACTIVATION_RECEIVED:
            if st.have_input:
                raise SchedulerError(f"duplicate activation for microbatch {mb}")
            st.have_input = True
            st.state = S.FORWARD_READY
        elif event is Event.FORWARD_STARTED:
            self._expect(st, mb, S.FORWARD_READY)
            st.state = S.FORWARD_RUNNING
        elif event is Event.FORWARD_FINISHED:
            self._expect(st, mb, S.FORWARD_RUNNING)
            st.state = S.FORWARD_DONE
            self.inflight += 1
            self.peak_inflight = max(self.peak_inflight, self.inflight)
            if self.is_last:
                st.have_grad = True
                st.state = S.BACKWARD_READY
        elif event is Event.SEND_COMPLETED:
            st.forward_sent = True
            if st.state is S.FORWARD_DONE:
                st.state = S.SENT_FORWARD
            if st.have_grad and st.state in (S.FORWARD_DONE, S.SENT_FORWARD):
                st.state = S.BACKWARD_READY
        elif event is Event.GRADIENT_RECEIVED:
            if st.have_grad:
                raise SchedulerError(f"duplicate gradient for microbatch {mb}")
            if st.state not in (S.FORWARD_DONE, S.SENT_FORWARD):
                raise SchedulerError(f"gradient for microbatch {mb} in state {st.state.value}")
            st.have_grad = True
            st.state = S.BACKWARD_READY
        elif event is Event.BACKWARD_STARTED:
            self._expect(st, mb, S.BACKWARD_READY)
            st.state = S.BACKWARD_RUNNING
        elif event is Event.BACKWARD_FINISHED:
            self._expect(st, mb, S.BACKWARD_RUNNING)
            st.state = S.COMPLETE
            self.inflight -= 1

    @staticmethod
    def _expect(st: _MB, mb: int, state: MicrobatchState) -> None:
        if st.state is not state:
            raise SchedulerError(f"microbatch {mb} is {st.state.value}, expected {state.value}")

    @property
    def done(self) -> bool:
        return self.cursor >= len(self.actions)

    def next_action(self) -> Action | None:
        return None if self.done else self.actions[self.cursor]

    def ready(self, action: Action) -> bool:
        st = self.mbs[action.microbatch]
        if action.kind is ActionKind.FORWARD:
            return st.state is MicrobatchState.FORWARD_READY
        return st.state is MicrobatchState.BACKWARD_READY

    def advance(self) -> None:
        self.cursor += 1

    def all_complete(self) -> bool:
        return all(m.state is MicrobatchState.COMPLETE for m in self.mbs.values())

    def snapshot(self) -> dict:
        return {
            "stage": self.stage, "step": self.step,
            "next_action": str(self.next_action()) if not self.done else None,
            "remaining": format_schedule(self.actions[self.cursor:]),
            "inflight": self.inflight,
            "microbatches": {m: s.state.value for m, s in self.mbs.items()},
        }
