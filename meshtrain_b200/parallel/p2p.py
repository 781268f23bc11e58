"""NCCL point-to-point links between adjacent pipeline stages.

Stage-boundary activations go s -> s+1 and activation gradients s+1 -> s as
NCCL send/recv over NVLink (NVSwitch) - the B200 replacement of the
reference's D2H -> TCP -> H2D hop (reference runtime/outbox.py:105-133,
networking/tcp.py:64-91, worker/device.py:253-286).

Each direction of each adjacent pair gets its own two-rank communicator, so
each runs on its own NCCL stream: a forward activation never queues behind a
backward gradient (and vice versa), which removes the classic 1F1B p2p
deadlock (stage s sending F(m+1) while stage s+1 sends B(m)) without having
to pair sends and receives into grouped calls.  Within one direction the
message order is the schedule order on both ends, so NCCL's per-communicator
FIFO matching routes every message to the right (step, microbatch).

Receives are posted ahead of use (``prefetch``) so the transfer overlaps the
current action's compute; the compute stream waits on the receive only when it
needs the data (``Work.wait`` is a stream wait, not a host block).
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field

import torch
import torch.distributed as dist


@dataclass
class LinkStats:
    bytes_sent: int = 0
    bytes_received: int = 0
    sends: int = 0
    recvs: int = 0
    transfer_ms: list[float] = field(default_factory=list)


class StageLinks:
    """NCCL p2p links of one pipeline stage (rank == stage index in its pipeline)."""

    def __init__(self, stage: int, num_stages: int, ranks: list[int] | None = None, ring: bool = False):
        if not dist.is_initialized():
            raise RuntimeError("torch.distributed must be initialised before StageLinks")
        self.stage = stage
        self.num_stages = num_stages
        self.ranks = ranks or list(range(num_stages))
        self.prev_rank = self.ranks[stage - 1] if stage > 0 else None
        self.next_rank = self.ranks[stage + 1] if stage < num_stages - 1 else None
        self.stats = LinkStats()
        # Every rank creates every pair group in the same order (new_group is collective).
        self._fwd: dict[int, dist.ProcessGroup] = {}
        self._bwd: dict[int, dist.ProcessGroup] = {}
        for s in range(num_stages - 1):
            pair = [self.ranks[s], self.ranks[s + 1]]
            self._fwd[s] = dist.new_group(pair)
            self._bwd[s] = dist.new_group(pair)
        # ring: the last rank's chunk c feeds the first rank's chunk c+1 (interleaved schedules)
        self.ring = ring and num_stages > 1
        self._ring_fwd = self._ring_bwd = None
        if self.ring:
            pair = [self.ranks[-1], self.ranks[0]]
            self._ring_fwd = dist.new_group(pair)
            self._ring_bwd = dist.new_group(pair)
        self.timing = os.environ.get("TORCH_NCCL_ENABLE_TIMING", "0") == "1"

    # groups touching this stage
    @property
    def fwd_out(self):
        return self._fwd.get(self.stage)

    @property
    def fwd_in(self):
        return self._fwd.get(self.stage - 1)

    @property
    def bwd_out(self):
        return self._bwd.get(self.stage - 1)

    @property
    def bwd_in(self):
        return self._bwd.get(self.stage)

    def warmup(self, device: torch.device) -> None:
        """Create every communicator up front with a one-element exchange per direction.

        Done in stage order so no rank blocks in communicator setup while its
        peer is still busy elsewhere.
        """
        t = torch.zeros(1, device=device)
        for s in range(self.num_stages - 1):
            for groups in (self._fwd, self._bwd):
                g = groups[s]
                if self.stage == s:
                    dist.send(t, self.ranks[s + 1], group=g) if groups is self._fwd else dist.recv(t, self.ranks[s + 1], group=g)
                elif self.stage == s + 1:
                    dist.recv(t, self.ranks[s], group=g) if groups is self._fwd else dist.send(t, self.ranks[s], group=g)
        if self.ring:
            first, last = self.ranks[0], self.ranks[-1]
            for g, src in ((self._ring_fwd, last), (self._ring_bwd, first)):
                dst = first if src == last else last
                if self.ranks[self.stage] == src:
                    dist.send(t, dst, group=g)
                elif self.ranks[self.stage] == dst:
                    dist.recv(t, src, group=g)
        if device.type == "cuda":
            torch.cuda.synchronize(device)

    def send_activation(self, t: torch.Tensor):
        self.stats.bytes_sent += t.numel() * t.element_size()
        self.stats.sends += 1
        return dist.isend(t, self.next_rank, group=self.fwd_out)

    def recv_activation(self, buf: torch.Tensor):
        self.stats.bytes_received += buf.numel() * buf.element_size()
        self.stats.recvs += 1
        return dist.irecv(buf, self.prev_rank, group=self.fwd_in)

    def send_gradient(self, t: torch.Tensor):
        self.stats.bytes_sent += t.numel() * t.element_size()
        self.stats.sends += 1
        return dist.isend(t, self.prev_rank, group=self.bwd_out)

    def recv_gradient(self, buf: torch.Tensor):
        self.stats.bytes_received += buf.numel() * buf.element_size()
        self.stats.recvs += 1
        return dist.irecv(buf, self.next_rank, group=self.bwd_in)

    # the wrap-around link of interleaved schedules (last rank <-> first rank)
    def send_activation_ring(self, t: torch.Tensor):
        self.stats.bytes_sent += t.numel() * t.element_size()
        self.stats.sends += 1
        return dist.isend(t, self.ranks[0], group=self._ring_fwd)

    def recv_activation_ring(self, buf: torch.Tensor):
        self.stats.bytes_received += buf.numel() * buf.element_size()
        self.stats.recvs += 1
        return dist.irecv(buf, self.ranks[-1], group=self._ring_fwd)

    def send_gradient_ring(self, t: torch.Tensor):
        self.stats.bytes_sent += t.numel() * t.element_size()
        self.stats.sends += 1
        return dist.isend(t, self.ranks[-1], group=self._ring_bwd)

    def recv_gradient_ring(self, buf: torch.Tensor):
        self.stats.bytes_received += buf.numel() * buf.element_size()
        self.stats.recvs += 1
        return dist.irecv(buf, self.ranks[0], group=self._ring_bwd)

    def groups(self) -> list:
        """Every pair communicator of this pipeline (for aborting them on a failure)."""
        ring = [g for g in (self._ring_fwd, self._ring_bwd) if g is not None]
        return list(self._fwd.values()) + list(self._bwd.values()) + ring

    def reset_stats(self) -> LinkStats:
        old, self.stats = self.stats, LinkStats()
        return old

    def destroy(self) -> None:
        for groups in (self._fwd, self._bwd):
            for g in groups.values():
                try:
                    dist.destroy_process_group(g)
                except Exception:
                    pass
        for g in (self._ring_fwd, self._ring_bwd):
            if g is not None:
                try:
                    dist.destroy_process_group(g)
                except Exception:
                    pass
        self._fwd.clear()
        self._bwd.clear()
        self._ring_fwd = self._ring_bwd = None


def work_duration_ms(work) -> float | None:
    """Device duration (ms) of a finished NCCL op when TORCH_NCCL_ENABLE_TIMING=1
    (``Work._get_duration``; None where the backend keeps no timing, e.g. gloo)."""
    getter = getattr(work, "_get_duration", None) or getattr(work, "get_duration", None)
    if getter is None:
        return None
    try:
        ms = float(getter())
    except Exception:  # noqa: BLE001 - timing off, or a backend without it
        return None
    return ms if ms >= 0 else None
