"""Device adapters: the only place that knows CUDA / MPS / CPU specifics.

The host-side pipeline runtime moves tensors across explicit network
boundaries through an adapter (reference worker/device.py:22-412):

    send:    begin_d2h (compute thread) -> finish() (sender thread)
    receive: recv_buffer (reader thread) -> begin_h2d -> finish_h2d -> after_use

The CUDA adapter stages through pinned pool buffers on a dedicated transfer
stream ordered against the compute stream with events.  (GPU stages inside a
B200 box do not go through this path at all: they use NCCL p2p and the
device-side engine, see parallel/engine.py.)
"""

from __future__ import annotations

import abc
import os
import platform

import psutil
import torch

from meshtrain_b200.utils.buffers import BufferPool

OP_PROBES = ("matmul", "linear", "gelu", "layer_norm", "softmax", "sdpa", "embedding", "cross_entropy", "adamw")
EMULATED_MEMORY_ENV = "MESHTRAIN_EMULATE_DEVICE_MEMORY_GB"


class DeviceAdapter(abc.ABC):
    backend: str = "abstract"

    def __init__(self, index: int = 0):
        self.index = index
        self.host_pool = BufferPool(pinned=False, enabled=True)
        self._prober = None

    @property
    @abc.abstractmethod
    def device(self) -> torch.device: ...

    # -- staging --------------------------------------------------------------
    def configure_transfers(self, pinned: bool = True, pool: bool = True) -> None:
        self.host_pool = BufferPool(pinned=pinned and self.supports("pinned_memory"), enabled=pool)

    def recv_buffer(self, shape, dtype: torch.dtype) -> torch.Tensor:
        return self.host_pool.acquire(shape, dtype)

    def begin_h2d(self, host: torch.Tensor):
        """Start moving a received host tensor to the device -> (handle, token)."""
        t = self.move_tensor(host)
        self.synchronize()
        self.host_pool.release(host)
        return t, None

    def finish_h2d(self, handle) -> torch.Tensor:
        return handle

    def after_use(self, token) -> None:
        if token is not None:
            self.host_pool.release(token)

    def begin_d2h(self, tensor: torch.Tensor):
        """Ordering point on the compute thread; returns finish() -> (cpu_tensor, release)."""
        cpu = tensor.detach().to("cpu")
        self.synchronize()
        return lambda: (cpu, None)

    def to_host(self, tensor: torch.Tensor) -> torch.Tensor:
        return tensor.detach().to("cpu")

    def move_tensor(self, tensor: torch.Tensor) -> torch.Tensor:
        if not self.supports_dtype(tensor.dtype):
            raise TypeError(f"{self.backend} does not support dtype {tensor.dtype}")
        return tensor.to(self.device)

    def move_module(self, module: torch.nn.Module) -> torch.nn.Module:
        for p in module.parameters():
            if not self.supports_dtype(p.dtype):
                raise TypeError(f"{self.backend} does not support parameter dtype {p.dtype}")
        return module.to(self.device)

    def synchronize(self) -> None:
        """Wait for all queued device work (no-op on CPU)."""

    def sync_compute(self) -> None:
        """Wait for the compute stream only (transfers on other streams keep running)."""
        self.synchronize()

    # -- memory ----------------------------------------------------------------
    @abc.abstractmethod
    def name(self) -> str: ...

    @abc.abstractmethod
    def memory_total(self) -> int: ...

    def memory_stats(self) -> dict:
        return {"total": self.memory_total(), "allocated": 0, "reserved": 0, "peak_allocated": 0, "unified": False}

    def reset_peak_memory(self) -> None:
        pass

    def available_memory(self, in_use: int = 0) -> int:
        st = self.memory_stats()
        return max(0, int(st.get("total", 0)) - int(st.get("allocated", 0)))

    # -- capabilities ------------------------------------------------------------
    def supports_dtype(self, dtype: torch.dtype) -> bool:
        return True

    def supports(self, operation: str, dtype: str | None = None) -> bool:
        if dtype is not None or operation in OP_PROBES:
            return self.prober.supports(operation, dtype or "float32")
        return {"float64": self.supports_dtype(torch.float64), "bfloat16": self.supports_dtype(torch.bfloat16),
                "float16": self.supports_dtype(torch.float16)}.get(operation, True)

    @property
    def prober(self):
        if self._prober is None:
            from meshtrain_b200.worker.capabilities import CapabilityProber

            self._prober = CapabilityProber(self.device, self.supports_dtype)
        return self._prober

    def capabilities(self) -> dict:
        st = self.memory_stats()
        return {"backend": self.backend, "device_name": self.name(), "total_memory": int(self.memory_total()),
                "available_memory": int(self.available_memory()), "unified_memory": bool(st.get("unified")),
                "pinned_memory": self.supports("pinned_memory"), "async_copy": self.supports("async_copy"),
                "nccl": self.supports("nccl"), **self.prober.report()}

    def describe(self) -> dict:
        return {"backend": self.backend, "name": self.name(), "memory_total": self.memory_total(),
                "unified_memory": bool(self.memory_stats().get("unified"))}

    def __repr__(self) -> str:
        return f"{type(self).__name__}({self.device})"


class CPUDeviceAdapter(DeviceAdapter):
    backend = "cpu"

    @property
    def device(self) -> torch.device:
        return torch.device("cpu")

    def begin_d2h(self, tensor):
        t = tensor.detach()  # already host memory: send straight from it
        return lambda: (t, None)

    def begin_h2d(self, host):
        # the received buffer is the device tensor; it returns to the pool after backward
        return host, host

    def name(self) -> str:
        return platform.processor() or platform.machine() or "cpu"

    def memory_total(self) -> int:
        return psutil.virtual_memory().total

    def memory_stats(self):
        vm = psutil.virtual_memory()
        rss = psutil.Process().memory_info().rss
        return {"total": vm.total, "available": vm.available, "allocated": rss, "reserved": rss,
                "peak_allocated": rss, "unified": False}

    def supports(self, operation, dtype=None):
        if dtype is None and operation in ("pinned_memory", "nccl", "async_copy"):
            return False
        return super().supports(operation, dtype)

    def available_memory(self, in_use: int = 0) -> int:
        emulated = os.environ.get(EMULATED_MEMORY_ENV)
        if emulated:  # fault injection: pretend the device is this small
            return max(0, int(float(emulated) * 1024 ** 3) - in_use)
        return int(psutil.virtual_memory().available)


class CUDADeviceAdapter(DeviceAdapter):
    """Pinned staging on a dedicated transfer stream, ordered by events."""

    backend = "cuda"

    def __init__(self, index: int = 0):
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA requested but torch.cuda.is_available() is False")
        super().__init__(index)
        self.host_pool = BufferPool(pinned=True, enabled=True)
        with torch.cuda.device(index):
            self.transfer_stream = torch.cuda.Stream()

    @property
    def device(self) -> torch.device:
        return torch.device("cuda", self.index)

    def synchronize(self) -> None:
        torch.cuda.synchronize(self.device)

    def sync_compute(self) -> None:
        torch.cuda.current_stream(self.device).synchronize()

    def begin_d2h(self, tensor):
        t = tensor.detach()
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(self.device))

        def finish():
            with torch.cuda.device(self.index):
                buf = self.host_pool.acquire(t.shape, t.dtype)
                with torch.cuda.stream(self.transfer_stream):
                    self.transfer_stream.wait_event(ready)
                    buf.copy_(t, non_blocking=buf.is_pinned())
                    done = torch.cuda.Event()
                    done.record(self.transfer_stream)
                done.synchronize()
            return buf, (lambda: self.host_pool.release(buf))

        return finish

    def to_host(self, tensor):
        return tensor.detach().to("cpu")

    def begin_h2d(self, host):
        if not self.supports_dtype(host.dtype):
            raise TypeError(f"cuda does not support dtype {host.dtype}")
        with torch.cuda.device(self.index), torch.cuda.stream(self.transfer_stream):
            t = host.to(self.device, non_blocking=host.is_pinned())
            ev = torch.cuda.Event()
            ev.record(self.transfer_stream)
        self.host_pool.release(host, ev)
        return (t, ev), None

    def finish_h2d(self, handle):
        t, ev = handle
        compute = torch.cuda.current_stream(self.device)
        compute.wait_event(ev)
        t.record_stream(compute)
        return t

    def name(self) -> str:
        return torch.cuda.get_device_name(self.index)

    def memory_total(self) -> int:
        return torch.cuda.get_device_properties(self.index).total_memory

    def memory_stats(self):
        free, total = torch.cuda.mem_get_info(self.index)
        return {"total": total, "free": free, "allocated": torch.cuda.memory_allocated(self.index),
                "reserved": torch.cuda.memory_reserved(self.index),
                "peak_allocated": torch.cuda.max_memory_allocated(self.index), "unified": False}

    def reset_peak_memory(self) -> None:
        torch.cuda.reset_peak_memory_stats(self.index)

    def available_memory(self, in_use: int = 0) -> int:
        free, _ = torch.cuda.mem_get_info(self.index)
        cached = torch.cuda.memory_reserved(self.index) - torch.cuda.memory_allocated(self.index)
        return int(free + max(0, cached))

    def supports_dtype(self, dtype):
        return torch.cuda.is_bf16_supported() if dtype == torch.bfloat16 else True

    def supports(self, operation, dtype=None):
        if dtype is None and operation in ("pinned_memory", "nccl", "autocast", "async_copy"):
            return True
        return super().supports(operation, dtype)


class MPSDeviceAdapter(DeviceAdapter):
    """Apple Silicon (unified memory, no fp64, synchronous copies)."""

    backend = "mps"

    def __init__(self, index: int = 0):
        if not (getattr(torch.backends, "mps", None) and torch.backends.mps.is_available()):
            raise RuntimeError("MPS requested but torch.backends.mps.is_available() is False")
        super().__init__(index)

    @property
    def device(self) -> torch.device:
        return torch.device("mps")

    def synchronize(self) -> None:
        torch.mps.synchronize()

    def supports(self, operation, dtype=None):
        if dtype is None and operation in ("pinned_memory", "nccl", "async_copy"):
            return False
        if dtype is None and operation == "bfloat16":
            return self.prober.supports("dtype", "bfloat16")
        return super().supports(operation, dtype)

    def name(self) -> str:
        return f"Apple {platform.machine()} (MPS)"

    def memory_total(self) -> int:
        fn = getattr(torch.mps, "recommended_max_memory", None)
        if fn is not None:
            try:
                return int(fn())
            except RuntimeError:
                pass
        return psutil.virtual_memory().total

    def memory_stats(self):
        allocated = int(torch.mps.current_allocated_memory())
        driver = int(getattr(torch.mps, "driver_allocated_memory", lambda: allocated)())
        return {"total": self.memory_total(), "allocated": allocated, "reserved": driver,
                "peak_allocated": driver, "unified": True}

    def supports_dtype(self, dtype):
        return dtype != torch.float64

    def available_memory(self, in_use: int = 0) -> int:
        st = self.memory_stats()
        return max(0, int(st["total"]) - int(st["reserved"]))


ADAPTERS: dict[str, type[DeviceAdapter]] = {"cpu": CPUDeviceAdapter, "cuda": CUDADeviceAdapter,
                                            "mps": MPSDeviceAdapter}


def available_backends() -> list[str]:
    out = []
    if torch.cuda.is_available():
        out.append("cuda")
    if getattr(torch.backends, "mps", None) is not None and torch.backends.mps.is_available():
        out.append("mps")
    out.append("cpu")
    return out


def select_device(preferred: str | None = None, index: int | None = None) -> DeviceAdapter:
    """Adapter for ``preferred`` ('cuda', 'cuda:3', 'mps', 'cpu', 'auto'), else CUDA > MPS > CPU.

    Unlike the reference (which drops the index of ``cuda:N``), the device index
    is honoured, so one process can host a stage on any local GPU.
    """
    if preferred in (None, "", "auto"):
        preferred = available_backends()[0]
    backend, _, idx = preferred.partition(":")
    if backend not in ADAPTERS:
        raise ValueError(f"unknown backend {backend!r}; expected one of {sorted(ADAPTERS)}")
    if index is None:
        index = int(idx) if idx else 0
    return ADAPTERS[backend](index)
