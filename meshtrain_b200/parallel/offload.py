"""Host offload of a stage's fp32 master weights and Adam moments, streamed through the GPU.

With offload the device keeps only what forward/backward touch - the bf16
compute copy of the parameters and the fp32 gradient accumulators - while the
fp32 master copy and both Adam moments (12 bytes per parameter) live in pinned
host DRAM.  The optimizer step streams that state through a ring of device
staging slots in chunks:

    h2d stream :  H2D(c0) H2D(c1) ......... H2D(c2) ........ H2D(c3)
    compute    :          adam(c0) adam(c1)        adam(c2)        ...
    d2h stream :                   D2H(c0)  D2H(c1)         D2H(c2)

Each chunk's Adam update runs on the device (the fused Adam kernel, which also
writes the new bf16 compute weights in place), then the updated master and
moments go back to the host on a second copy stream, so the two copy
directions and the math overlap.  A slot is refilled only after its previous
chunk has been copied out (event on the d2h stream).

``prefetch`` issues the host-to-device copies of as many chunks as there are
slots at the start of a step, so they overlap the step's forward and backward
and the optimizer finds them resident.  The slot count follows a device
budget (``device_budget_gb``): the more slots, the less of the stream is left
for the optimizer phase, where the non-resident chunks cost one PCIe transfer
each way (both directions run at once).  The last chunks' device-to-host
copies finish under the next step's forward.  The reference declares
parameter/optimizer tiers but keeps every tensor resident (reference
runtime/tensor_store.py:1-60, future.py:1-46); this module is the B200
implementation of that tier.
"""

from __future__ import annotations

import torch

from meshtrain_b200 import ops

ALIGN = 64  # elements; every chunk starts 256-byte aligned


def slot_ring_bytes(state_elems: int, *, chunk_mb: float = 256.0, min_slots: int = 2, prefetch_ahead: int = 1,
                    device_budget_gb: float | None = None) -> int:
    """Device bytes of the staging ring a ``HostOffload`` with these settings allocates for a stage
    whose flat state has ``state_elems`` elements (each slot holds master + two moments of a chunk)."""
    chunk = max(ALIGN, int(chunk_mb * 1024 ** 2 / 4) // ALIGN * ALIGN)
    slots = max(min_slots, prefetch_ahead + 1)
    if device_budget_gb is not None:
        slots = max(min_slots, int(device_budget_gb * 1024 ** 3 // (12 * chunk)))
    chunks = max(1, -(-int(state_elems) // chunk))
    return min(slots, chunks) * 3 * chunk * 4


class HostOffload:
    def __init__(self, prefetch_ahead: int = 1, chunk_mb: float = 256.0, min_slots: int = 2,
                 device_budget_gb: float | None = None):
        self.prefetch_ahead = max(0, int(prefetch_ahead))
        self.chunk_elems = max(ALIGN, int(chunk_mb * 1024 ** 2 / 4) // ALIGN * ALIGN)
        self.nslots = max(min_slots, self.prefetch_ahead + 1)
        if device_budget_gb is not None:  # every slot holds master + two moments of one chunk
            self.nslots = max(min_slots, int(device_budget_gb * 1024 ** 3 // (12 * self.chunk_elems)))
        self.flat = None
        self.stats = {"steps": 0, "h2d_bytes": 0, "d2h_bytes": 0, "chunks": 0}

    def ring_settings(self) -> dict:
        """``slot_ring_bytes`` arguments that reproduce this ring (for the memory estimate)."""
        return {"chunk_mb": self.chunk_elems * 4 / 1024 ** 2, "min_slots": self.nslots, "prefetch_ahead": 0}

    # ------------------------------------------------------------ setup
    def attach(self, flat) -> None:
        self.flat = flat
        self.cuda = flat.device.type == "cuda"
        n = flat.numel
        self.chunks = [(o, min(self.chunk_elems, n - o)) for o in range(0, n, self.chunk_elems)]
        self.nslots = min(self.nslots, len(self.chunks))
        self.slots = [torch.empty(3, self.chunk_elems, dtype=torch.float32, device=flat.device)
                      for _ in range(self.nslots)]
        if self.cuda:
            self.h2d = torch.cuda.Stream(device=flat.device)
            self.d2h = torch.cuda.Stream(device=flat.device)
            self.loaded = [torch.cuda.Event() for _ in self.chunks]
            self.freed = [None] * self.nslots  # event: slot's last D2H finished
        self._issued: set[int] = set()

    def device_bytes(self) -> int:
        return sum(s.numel() * s.element_size() for s in self.slots)

    # ------------------------------------------------------------ copies
    def _load(self, i: int) -> None:
        """Copy chunk ``i`` of master / exp_avg / exp_avg_sq into its slot."""
        if i in self._issued or i >= len(self.chunks):
            return
        f = self.flat
        o, n = self.chunks[i]
        slot = self.slots[i % self.nslots]
        if self.cuda:
            with torch.cuda.stream(self.h2d):
                ev = self.freed[i % self.nslots]
                if ev is not None:
                    self.h2d.wait_event(ev)
                for row, src in enumerate((f.master, f.exp_avg, f.exp_avg_sq)):
                    slot[row, :n].copy_(src[o:o + n], non_blocking=True)
                self.loaded[i].record(self.h2d)
        else:
            for row, src in enumerate((f.master, f.exp_avg, f.exp_avg_sq)):
                slot[row, :n].copy_(src[o:o + n])
        self.stats["h2d_bytes"] += 12 * n
        self._issued.add(i)

    def _store(self, i: int) -> None:
        f = self.flat
        o, n = self.chunks[i]
        s = i % self.nslots
        slot = self.slots[s]
        if self.cuda:
            done = torch.cuda.Event()
            done.record(torch.cuda.current_stream(f.device))
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(done)
                for row, dst in enumerate((f.master, f.exp_avg, f.exp_avg_sq)):
                    dst[o:o + n].copy_(slot[row, :n], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.d2h)
                self.freed[s] = ev
        else:
            for row, dst in enumerate((f.master, f.exp_avg, f.exp_avg_sq)):
                dst[o:o + n].copy_(slot[row, :n])
        self.stats["d2h_bytes"] += 12 * n

    def prefetch(self, engine=None) -> None:
        """Start loading one chunk into every slot (called at the start of a step, ahead of its
        optimizer phase); a slot still being copied out waits for that copy on the h2d stream."""
        if self.prefetch_ahead:
            for i in range(min(self.nslots, len(self.chunks))):
                self._load(i)

    def resident_fraction(self) -> float:
        """Share of the offloaded state that the slots hold at once."""
        return min(1.0, self.nslots / max(1, len(self.chunks)))

    # ------------------------------------------------------------ the streamed optimizer step
    def step(self, engine) -> None:
        f = self.flat
        lowp = None if f.compute is f.master else f.compute
        cur = torch.cuda.current_stream(f.device) if self.cuda else None
        for i, (o, n) in enumerate(self.chunks):
            self._load(i)
            if self.cuda:
                cur.wait_event(self.loaded[i])
            slot = self.slots[i % self.nslots]
            p, m, v = slot[0, :n], slot[1, :n], slot[2, :n]
            out = lowp[o:o + n] if lowp is not None else None
            if engine.opt_name == "sgd":
                p.add_(f.grad[o:o + n], alpha=-engine.lr)
                if out is not None:
                    out.copy_(p)
            else:
                ops.adam_(p, f.grad[o:o + n], m, v, out, lr=engine.lr, beta1=engine.betas[0], beta2=engine.betas[1],
                          eps=engine.eps, weight_decay=engine.wd, decoupled=engine.opt_name == "adamw",
                          step=engine.opt_steps)
            self._store(i)
            # refill: the slot this chunk used serves chunk i + nslots once its D2H has finished
            if i + self.nslots < len(self.chunks):
                self._load(i + self.nslots)
        self._issued.clear()
        self.stats["steps"] += 1
        self.stats["chunks"] += len(self.chunks)
        if f.compute is f.master:  # fp32 compute without a device copy (CPU tests)
            return

    def synchronize(self) -> None:
        """Wait until every host copy is current (before reading master/moments on the host)."""
        if self.cuda:
            self.d2h.synchronize()
            self.h2d.synchronize()
