"""Pipeline schedules as per-stage programs, and the ledger that checks them.

Program
-------
For one stage and one global step, a schedule is the ordered list of forward
(``F<m>``) and backward (``B<m>``) actions the stage runs.  Both supported
schedules come from one rule: *run the next forward while fewer than
``budget`` microbatches are in flight on this stage, otherwise run the oldest
pending backward*.  The budget is ``warm-up + 1``:

* ``gpipe`` (reference runtime/scheduler.py:82-89): every stage but the last
  has an unlimited budget (all forwards, then all backwards); the last stage
  computes its loss locally, so its budget is 1 and it alternates F/B.
* ``1f1b`` (PipeDream-flush, reference runtime/scheduler.py:64-81): stage s
  warms up with ``min(S-s-1, cap-1, M)`` forwards, so it never holds more than
  ``min(S-s, cap, M)`` microbatch contexts.  The warm-up shrinks down the
  pipeline, so stage s+1 can always return the gradient stage s waits for:
  the schedule cannot deadlock (``simulate`` checks this exhaustively in the
  tests).

A schedule only reorders work: all microbatches of a step see one parameter
version, the loss is scaled by 1/M, gradients accumulate, and the optimizer
steps once per global step.

Ledger
------
``StepLedger`` keeps five flags per microbatch (input here, forward done,
forward sent, gradient here, backward done) and refuses what the protocol
forbids: events for unknown microbatches, a second activation or gradient, a
gradient before its forward, running an action whose inputs are missing.
Both the host runtime (parallel/pipeline.py) and the device engine
(parallel/engine.py) drive their steps through it.
"""

from __future__ import annotations

import enum
from dataclasses import dataclass


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
    last = stage == num_stages - 1
    if schedule == "gpipe":
        return 0 if last else num_microbatches
    cap = num_microbatches if max_inflight is None else max(1, max_inflight)
    return max(0, min(num_stages - 1 - stage, cap - 1, num_microbatches))


def stage_schedule(schedule: str, stage: int, num_stages: int, num_microbatches: int,
                   max_inflight: int | None = None) -> list[Action]:
    """The stage's action list for one global step."""
    if schedule not in SCHEDULES:
        raise ValueError(f"unknown schedule {schedule!r}; expected one of {SCHEDULES}")
    if num_microbatches < 1 or not 0 <= stage < num_stages:
        raise ValueError("invalid stage/microbatch counts")
    budget = warmup_forwards(schedule, stage, num_stages, num_microbatches, max_inflight) + 1
    program: list[Action] = []
    forwards = backwards = 0
    while backwards < num_microbatches:
        if forwards < num_microbatches and forwards - backwards < budget:
            program.append(Action(ActionKind.FORWARD, forwards))
            forwards += 1
        else:
            program.append(Action(ActionKind.BACKWARD, backwards))
            backwards += 1
    return program


def max_inflight_of(actions: list[Action]) -> int:
    """Peak number of microbatches forwarded but not yet backwarded."""
    peak = live = 0
    for a in actions:
        live += 1 if a.kind is ActionKind.FORWARD else -1
        peak = max(peak, live)
    return peak


def format_schedule(actions: list[Action]) -> str:
    return " ".join(map(str, actions))


def simulate(schedule: str, num_stages: int, num_microbatches: int, max_inflight: int | None = None,
             fwd_cost: float = 1.0, bwd_cost: float = 2.0) -> dict:
    """Runs every stage's program against the pipeline's data dependencies.

    Each stage executes its actions in order, one at a time; ``F<m>`` on stage
    s waits for ``F<m>`` on s-1, ``B<m>`` waits for ``B<m>`` on s+1 (or for the
    stage's own ``F<m>`` on the last stage).  Events are processed in time
    order (earliest possible start first), so the result is the schedule's
    makespan under the given unit costs; a state where no stage can move is a
    deadlock (``complete`` False).
    """
    S, M = num_stages, num_microbatches
    programs = [stage_schedule(schedule, s, S, M, max_inflight) for s in range(S)]
    pc = [0] * S
    free_at = [0.0] * S
    busy = [0.0] * S
    finished: dict[tuple[str, int, int], float] = {}

    def ready_time(s: int):
        a = programs[s][pc[s]]
        if a.kind is ActionKind.FORWARD:
            dep = 0.0 if s == 0 else finished.get(("F", s - 1, a.microbatch))
        else:
            dep = finished.get(("F", s, a.microbatch) if s == S - 1 else ("B", s + 1, a.microbatch))
        return None if dep is None else max(dep, free_at[s])

    while True:
        candidates = [(t, s) for s in range(S) if pc[s] < len(programs[s])
                      for t in (ready_time(s),) if t is not None]
        if not candidates:
            break
        start, s = min(candidates)
        a = programs[s][pc[s]]
        cost = fwd_cost if a.kind is ActionKind.FORWARD else bwd_cost
        free_at[s] = start + cost
        busy[s] += cost
        finished[(a.kind.value, s, a.microbatch)] = free_at[s]
        pc[s] += 1
    complete = all(pc[s] == len(programs[s]) for s in range(S))
    makespan = max(free_at) if complete else float("inf")
    return {"complete": complete, "makespan": makespan, "busy": busy,
            "bubble_fraction": 1.0 - sum(busy) / (S * makespan) if complete and makespan > 0 else None}


class SchedulerError(RuntimeError):
    pass


# ledger flags
HAVE_INPUT, FORWARDED, SENT, HAVE_GRAD, BACKWARDED = 1, 2, 4, 8, 16
_FLAG_NAMES = ((HAVE_INPUT, "input"), (FORWARDED, "forward"), (SENT, "sent"), (HAVE_GRAD, "grad"),
               (BACKWARDED, "backward"))


class StepLedger:
    """Microbatch progress of one stage in one global step, plus the program cursor."""

    def __init__(self, stage: int, num_stages: int, num_microbatches: int, step: int,
                 schedule: str = "gpipe", max_inflight: int | None = None, actions: list[Action] | None = None):
        self.stage, self.num_stages, self.step = stage, num_stages, step
        self.is_first, self.is_last = stage == 0, stage == num_stages - 1
        self.actions = (list(actions) if actions is not None else
                        stage_schedule(schedule, stage, num_stages, num_microbatches, max_inflight))
        self.cursor = 0
        self.flags = [HAVE_INPUT if self.is_first else 0] * num_microbatches  # the first stage owns the data
        self.inflight = 0
        self.peak_inflight = 0

    # -- events ------------------------------------------------------------
    def _flags(self, mb: int, what: str) -> int:
        if not 0 <= mb < len(self.flags):
            raise SchedulerError(f"{what} for unknown microbatch {mb}")
        return self.flags[mb]

    def input_arrived(self, mb: int) -> None:
        f = self._flags(mb, "activation")
        if f & HAVE_INPUT:
            raise SchedulerError(f"duplicate activation for microbatch {mb}")
        self.flags[mb] = f | HAVE_INPUT

    def gradient_arrived(self, mb: int) -> None:
        f = self._flags(mb, "gradient")
        if f & HAVE_GRAD:
            raise SchedulerError(f"duplicate gradient for microbatch {mb}")
        if not f & FORWARDED or f & BACKWARDED:
            raise SchedulerError(f"gradient for microbatch {mb} before its forward ({self.describe(mb)})")
        self.flags[mb] = f | HAVE_GRAD

    def forward_sent(self, mb: int) -> None:
        self.flags[mb] = self._flags(mb, "send completion") | SENT

    def run(self, action: Action) -> None:
        """Marks ``action`` started; it must be the program's next action and ready."""
        if self.done or action != self.actions[self.cursor]:
            raise SchedulerError(f"{action} is not the next action ({self.next_action()})")
        if not self.ready(action):
            raise SchedulerError(f"{action} is not ready ({self.describe(action.microbatch)})")

    def finish(self, action: Action) -> None:
        """Records ``action`` as done and moves the cursor."""
        mb = action.microbatch
        if action.kind is ActionKind.FORWARD:
            self.flags[mb] |= FORWARDED | (HAVE_GRAD if self.is_last else 0)  # the loss is local
            self.inflight += 1
            self.peak_inflight = max(self.peak_inflight, self.inflight)
        else:
            self.flags[mb] |= BACKWARDED
            self.inflight -= 1
        self.cursor += 1

    # -- queries -----------------------------------------------------------
    def ready(self, action: Action) -> bool:
        f = self.flags[action.microbatch]
        if action.kind is ActionKind.FORWARD:
            return f & (HAVE_INPUT | FORWARDED) == HAVE_INPUT
        return f & (FORWARDED | HAVE_GRAD | BACKWARDED) == FORWARDED | HAVE_GRAD

    @property
    def done(self) -> bool:
        return self.cursor >= len(self.actions)

    def next_action(self) -> Action | None:
        return None if self.done else self.actions[self.cursor]

    def all_complete(self) -> bool:
        return all(f & BACKWARDED for f in self.flags)

    def describe(self, mb: int) -> str:
        f = self.flags[mb]
        return "+".join(name for bit, name in _FLAG_NAMES if f & bit) or "nothing"

    def snapshot(self) -> dict:
        return {"stage": self.stage, "step": self.step,
                "next_action": None if self.done else str(self.next_action()),
                "remaining": format_schedule(self.actions[self.cursor:]), "inflight": self.inflight,
                "microbatches": {m: self.describe(m) for m in range(len(self.flags))}}


# ---------------------------------------------------------------- interleaved 1F1B
# A rank may hold several non-adjacent pieces ("chunks") of the model: with S
# ranks and v chunks, virtual stage c*S + r is chunk c of rank r, so a
# microbatch crosses every rank v times.  The program is the interleaved 1F1B
# order of Narayanan et al., "Efficient Large-Scale Language Model Training on
# GPU Clusters Using Megatron-LM" (SC'21, section 2.2): microbatches go in
# groups of S; the k-th forward of a rank is chunk (k // S) mod v of microbatch
# (k // (S v)) S + k mod S, the k-th backward walks the chunks in reverse; rank
# r warms up with 2 (S - r - 1) + (v - 1) S forwards, then alternates one
# forward and one backward.  The pipeline bubble shrinks by about v (8 ranks,
# 32 microbatches: 18 % -> 10 % at v = 2), at the price of v times as many
# stage-boundary messages.  One optimizer step per global step, as before.


@dataclass(frozen=True)
class ChunkAction:
    kind: ActionKind
    chunk: int
    microbatch: int

    def __str__(self) -> str:
        return f"{self.kind.value}{self.microbatch}" + (f".{self.chunk}" if self.chunk else "")


def interleaved_warmup(stage: int, num_stages: int, num_microbatches: int, chunks: int) -> int:
    total = chunks * num_microbatches
    if chunks == 1:
        return min(num_stages - 1 - stage, num_microbatches)
    return min(total, 2 * (num_stages - stage - 1) + (chunks - 1) * num_stages)


def interleaved_schedule(stage: int, num_stages: int, num_microbatches: int, chunks: int) -> list[ChunkAction]:
    """Rank ``stage``'s program over its ``chunks`` model chunks (``chunks`` = 1: plain 1F1B)."""
    S, M, v = num_stages, num_microbatches, chunks
    if v < 1 or not 0 <= stage < S or M < 1:
        raise ValueError("invalid stage / microbatch / chunk counts")
    if v > 1 and M % S:
        raise ValueError(f"interleaving {v} chunks needs the microbatch count ({M}) to be a multiple of the "
                         f"number of ranks ({S})")
    group = S * v

    def forward(k: int) -> ChunkAction:
        return ChunkAction(ActionKind.FORWARD, (k // S) % v, (k // group) * S + k % S)

    def backward(k: int) -> ChunkAction:
        return ChunkAction(ActionKind.BACKWARD, v - 1 - (k // S) % v, (k // group) * S + k % S)

    total = v * M
    warm = interleaved_warmup(stage, S, M, v)
    program = [forward(k) for k in range(warm)]
    for i in range(total - warm):
        program += [forward(warm + i), backward(i)]
    program += [backward(i) for i in range(total - warm, total)]
    return program


def simulate_interleaved(num_stages: int, num_microbatches: int, chunks: int, fwd_cost: float = 1.0,
                         bwd_cost: float = 2.0, piece_costs: list[float] | None = None) -> dict:
    """``simulate`` for the interleaved programs: virtual stage c*S + r is chunk c of rank r.

    Without ``piece_costs`` each chunk action costs 1/chunks of a whole stage's.  With them,
    ``piece_costs[c*S + r]`` is the forward cost of virtual stage c*S + r and its backward
    costs ``bwd_cost / fwd_cost`` times that (the real, unequal pieces of a model)."""
    S, M, v = num_stages, num_microbatches, chunks
    if piece_costs is not None and len(piece_costs) != S * v:
        raise ValueError(f"{len(piece_costs)} piece costs for {v} x {S} virtual stages")
    programs = [interleaved_schedule(r, S, M, v) for r in range(S)]
    pc = [0] * S
    free_at = [0.0] * S
    busy = [0.0] * S
    finished: dict[tuple, float] = {}

    def ready_time(r: int):
        a = programs[r][pc[r]]
        c, m = a.chunk, a.microbatch
        if a.kind is ActionKind.FORWARD:
            if r == 0 and c == 0:
                dep = 0.0
            else:
                dep = finished.get(("F", r - 1, c, m) if r > 0 else ("F", S - 1, c - 1, m))
        elif r < S - 1:
            dep = finished.get(("B", r + 1, c, m))
        elif c < v - 1:
            dep = finished.get(("B", 0, c + 1, m))
        else:
            dep = finished.get(("F", r, c, m))
        return None if dep is None else max(dep, free_at[r])

    while True:
        candidates = [(t, r) for r in range(S) if pc[r] < len(programs[r]) for t in (ready_time(r),) if t is not None]
        if not candidates:
            break
        start, r = min(candidates)
        a = programs[r][pc[r]]
        if piece_costs is None:
            cost = (fwd_cost if a.kind is ActionKind.FORWARD else bwd_cost) / v
        else:
            fwd = piece_costs[a.chunk * S + r]
            cost = fwd if a.kind is ActionKind.FORWARD else fwd * bwd_cost / fwd_cost
        free_at[r] = start + cost
        busy[r] += cost
        finished[(a.kind.value, r, a.chunk, a.microbatch)] = free_at[r]
        pc[r] += 1
    complete = all(pc[r] == len(programs[r]) for r in range(S))
    makespan = max(free_at) if complete else float("inf")
    return {"complete": complete, "makespan": makespan, "busy": busy,
            "bubble_fraction": 1.0 - sum(busy) / (S * makespan) if complete and makespan > 0 else None}


class ChunkLedger:
    """The ledger of a rank that runs an interleaved program: one ``StepLedger`` per
    chunk, each for its virtual stage (chunk c of rank r is virtual stage c*S + r of
    v*S, so the first and last virtual stages own the data and the loss), and the
    rank's cursor over the whole program."""

    def __init__(self, stage: int, num_stages: int, num_microbatches: int, step: int, chunks: int):
        self.stage, self.step = stage, step
        self.actions = interleaved_schedule(stage, num_stages, num_microbatches, chunks)
        self.ledgers = [StepLedger(c * num_stages + stage, chunks * num_stages, num_microbatches, step,
                                   actions=[Action(a.kind, a.microbatch) for a in self.actions if a.chunk == c])
                        for c in range(chunks)]
        self.cursor = 0
        self.inflight = 0
        self.peak_inflight = 0

    def input_arrived(self, chunk: int, mb: int) -> None:
        self.ledgers[chunk].input_arrived(mb)

    def gradient_arrived(self, chunk: int, mb: int) -> None:
        self.ledgers[chunk].gradient_arrived(mb)

    def forward_sent(self, chunk: int, mb: int) -> None:
        self.ledgers[chunk].forward_sent(mb)

    def run(self, action: ChunkAction) -> None:
        if self.cursor >= len(self.actions) or action != self.actions[self.cursor]:
            nxt = self.actions[self.cursor] if self.cursor < len(self.actions) else None
            raise SchedulerError(f"{action} is not the next action ({nxt})")
        self.ledgers[action.chunk].run(Action(action.kind, action.microbatch))

    def finish(self, action: ChunkAction) -> None:
        self.ledgers[action.chunk].finish(Action(action.kind, action.microbatch))
        self.inflight += 1 if action.kind is ActionKind.FORWARD else -1
        self.peak_inflight = max(self.peak_inflight, self.inflight)
        self.cursor += 1

    def all_complete(self) -> bool:
        return all(led.all_complete() for led in self.ledgers)

    def snapshot(self) -> dict:
        return {"stage": self.stage, "step": self.step, "cursor": self.cursor,
                "remaining": " ".join(map(str, self.actions[self.cursor:])),
                "chunks": [led.snapshot() for led in self.ledgers]}
