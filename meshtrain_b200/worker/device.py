"""Device adapters: everything the host runtime needs to know about CUDA, MPS or CPU.

An adapter is assembled from three parts:

* a **memory view** (``HostMemory``, ``CudaMemory``, ``MpsMemory``): totals,
  allocator statistics and how much a new stage could still allocate;
* a **stager** that moves tensors across a process boundary:
  ``InPlaceStager`` (CPU: the received host buffer *is* the tensor),
  ``BlockingStager`` (MPS: synchronous copies) and ``StreamStager`` (CUDA:
  pinned pool buffers and a dedicated transfer stream, ordered against the
  compute stream by events, so copies overlap compute);
* a **capability table**: dtypes and features (pinned memory, async copy,
  NCCL), plus op probes run on demand by ``worker/capabilities.py``.

The staging protocol the host runtime follows (reference worker/device.py:22-412):

    send:    begin_d2h(t) on the compute thread -> finish() on the sender thread
    receive: recv_buffer() on the reader thread -> begin_h2d() -> finish_h2d() -> after_use()

GPU stages inside one box do not use this path: the device engine keeps
activations on the GPU and exchanges them with NCCL (parallel/engine.py).
``select_device("cuda:N")`` keeps the GPU index (the reference drops it).
"""

from __future__ import annotations

import os
import platform

import psutil
import torch

from meshtrain_b200.utils.buffers import BufferPool

OP_PROBES = ("matmul", "linear", "gelu", "layer_norm", "softmax", "sdpa", "embedding", "cross_entropy", "adamw")
EMULATED_MEMORY_ENV = "MESHTRAIN_EMULATE_DEVICE_MEMORY_GB"
FEATURES = ("pinned_memory", "async_copy", "nccl", "autocast")


# ---------------------------------------------------------------------------- memory views
class HostMemory:
    """System RAM seen from this process; ``MESHTRAIN_EMULATE_DEVICE_MEMORY_GB`` caps what is free."""

    unified = False

    def total(self) -> int:
        return psutil.virtual_memory().total

    def stats(self) -> dict:
        vm = psutil.virtual_memory()
        rss = psutil.Process().memory_info().rss
        return {"total": vm.total, "available": vm.available, "allocated": rss, "reserved": rss,
                "peak_allocated": rss, "unified": False}

    def free(self, in_use: int) -> int:
        emulated = os.environ.get(EMULATED_MEMORY_ENV)
        if emulated:  # fault injection: pretend the device has only this much
            return max(0, int(float(emulated) * 1024 ** 3) - in_use)
        return int(psutil.virtual_memory().available)

    def reset_peak(self) -> None:
        pass


class CudaMemory:
    unified = False

    def __init__(self, index: int):
        self.index = index

    def total(self) -> int:
        return torch.cuda.get_device_properties(self.index).total_memory

    def stats(self) -> dict:
        free, total = torch.cuda.mem_get_info(self.index)
        return {"total": total, "free": free, "allocated": torch.cuda.memory_allocated(self.index),
                "reserved": torch.cuda.memory_reserved(self.index),
                "peak_allocated": torch.cuda.max_memory_allocated(self.index), "unified": False}

    def free(self, in_use: int) -> int:
        # free device memory plus what this process's caching allocator holds but does not use
        free, _ = torch.cuda.mem_get_info(self.index)
        idle_cache = torch.cuda.memory_reserved(self.index) - torch.cuda.memory_allocated(self.index)
        return int(free + max(0, idle_cache))

    def reset_peak(self) -> None:
        torch.cuda.reset_peak_memory_stats(self.index)


class MpsMemory:
    """Apple unified memory: the budget is the recommended maximum working set."""

    unified = True

    def total(self) -> int:
        limit = getattr(torch.mps, "recommended_max_memory", None)
        if limit is not None:
            try:
                return int(limit())
            except RuntimeError:
                pass
        return psutil.virtual_memory().total

    def stats(self) -> dict:
        allocated = int(torch.mps.current_allocated_memory())
        driver = getattr(torch.mps, "driver_allocated_memory", None)
        reserved = int(driver()) if driver is not None else allocated
        return {"total": self.total(), "allocated": allocated, "reserved": reserved, "peak_allocated": reserved,
                "unified": True}

    def free(self, in_use: int) -> int:
        st = self.stats()
        return max(0, int(st["total"]) - int(st["reserved"]))

    def reset_peak(self) -> None:
        pass


# ---------------------------------------------------------------------------- stagers
class InPlaceStager:
    """CPU: tensors are already host memory; the receive buffer becomes the stage input."""

    def __init__(self, adapter):
        self.adapter = adapter

    def begin_d2h(self, tensor):
        host = tensor.detach()
        return lambda: (host, None)

    def begin_h2d(self, host):
        return host, host  # handle and token are the same buffer: it returns to the pool after backward

    def finish_h2d(self, handle):
        return handle


class BlockingStager:
    """Synchronous copies through the pool (devices without pinned memory or copy streams)."""

    def __init__(self, adapter):
        self.adapter = adapter

    def begin_d2h(self, tensor):
        host = tensor.detach().to("cpu")
        self.adapter.synchronize()
        return lambda: (host, None)

    def begin_h2d(self, host):
        on_device = self.adapter.move_tensor(host)
        self.adapter.synchronize()
        self.adapter.host_pool.release(host)
        return on_device, None

    def finish_h2d(self, handle):
        return handle


class StreamStager:
    """CUDA: pinned buffers, a transfer stream and events against the compute stream."""

    def __init__(self, adapter):
        self.adapter = adapter
        with torch.cuda.device(adapter.index):
            self.stream = torch.cuda.Stream()

    def begin_d2h(self, tensor):
        a = self.adapter
        src = tensor.detach()
        produced = torch.cuda.Event()
        produced.record(torch.cuda.current_stream(a.device))  # the ordering point on the compute thread

        def finish():
            with torch.cuda.device(a.index):
                host = a.host_pool.acquire(src.shape, src.dtype)
                with torch.cuda.stream(self.stream):
                    self.stream.wait_event(produced)
                    host.copy_(src, non_blocking=host.is_pinned())
                    copied = torch.cuda.Event()
                    copied.record(self.stream)
                copied.synchronize()
            return host, (lambda: a.host_pool.release(host))

        return finish

    def begin_h2d(self, host):
        a = self.adapter
        if not a.supports_dtype(host.dtype):
            raise TypeError(f"cuda does not support dtype {host.dtype}")
        with torch.cuda.device(a.index), torch.cuda.stream(self.stream):
            on_device = host.to(a.device, non_blocking=host.is_pinned())
            landed = torch.cuda.Event()
            landed.record(self.stream)
        a.host_pool.release(host, landed)  # the host buffer is reusable once the copy has read it
        return (on_device, landed), None

    def finish_h2d(self, handle):
        on_device, landed = handle
        compute = torch.cuda.current_stream(self.adapter.device)
        compute.wait_event(landed)
        on_device.record_stream(compute)
        return on_device


# ---------------------------------------------------------------------------- adapter
class DeviceAdapter:
    backend: str = "abstract"
    features: frozenset = frozenset()
    unsupported_dtypes: frozenset = frozenset()

    def __init__(self, index: int, device: torch.device, memory, stager_cls, pinned_pool: bool):
        self.index = index
        self._device = device
        self.memory = memory
        self.host_pool = BufferPool(pinned=pinned_pool, enabled=True)
        self.stager = stager_cls(self)
        self._prober = None

    @property
    def device(self) -> torch.device:
        return self._device

    # -- staging (delegated to the stager) ---------------------------------------
    def configure_transfers(self, pinned: bool = True, pool: bool = True) -> None:
        self.host_pool = BufferPool(pinned=pinned and self.supports("pinned_memory"), enabled=pool)

    def recv_buffer(self, shape, dtype: torch.dtype) -> torch.Tensor:
        return self.host_pool.acquire(shape, dtype)

    def begin_h2d(self, host: torch.Tensor):
        """Starts moving a received host tensor to the device -> (handle, token)."""
        return self.stager.begin_h2d(host)

    def finish_h2d(self, handle) -> torch.Tensor:
        return self.stager.finish_h2d(handle)

    def after_use(self, token) -> None:
        if token is not None:
            self.host_pool.release(token)

    def begin_d2h(self, tensor: torch.Tensor):
        """Ordering point on the compute thread; returns finish() -> (host tensor, release or None)."""
        return self.stager.begin_d2h(tensor)

    def to_host(self, tensor: torch.Tensor) -> torch.Tensor:
        return tensor.detach().to("cpu")

    def move_tensor(self, tensor: torch.Tensor) -> torch.Tensor:
        if not self.supports_dtype(tensor.dtype):
            raise TypeError(f"{self.backend} does not support dtype {tensor.dtype}")
        return tensor.to(self.device)

    def move_module(self, module: torch.nn.Module) -> torch.nn.Module:
        bad = {p.dtype for p in module.parameters() if not self.supports_dtype(p.dtype)}
        if bad:
            raise TypeError(f"{self.backend} does not support parameter dtype {sorted(map(str, bad))[0]}")
        return module.to(self.device)

    def synchronize(self) -> None:
        """Waits for all queued device work."""

    def sync_compute(self) -> None:
        """Waits for the compute stream only (copies on other streams keep running)."""
        self.synchronize()

    # -- memory -------------------------------------------------------------------
    def name(self) -> str:
        raise NotImplementedError

    def memory_total(self) -> int:
        return self.memory.total()

    def memory_stats(self) -> dict:
        return self.memory.stats()

    def reset_peak_memory(self) -> None:
        self.memory.reset_peak()

    def available_memory(self, in_use: int = 0) -> int:
        return self.memory.free(in_use)

    # -- capabilities ---------------------------------------------------------------
    def supports_dtype(self, dtype: torch.dtype) -> bool:
        return dtype not in self.unsupported_dtypes

    def supports(self, operation: str, dtype: str | None = None) -> bool:
        """A feature (``pinned_memory``, ``nccl``, ...), a dtype name, or an op probed in ``dtype``."""
        if dtype is None and operation in FEATURES:
            return operation in self.features
        if dtype is None and operation in ("float64", "float16", "bfloat16"):
            return self.supports_dtype(getattr(torch, operation))
        if dtype is None and operation not in OP_PROBES:
            return True
        return self.prober.supports(operation, dtype or "float32")

    @property
    def prober(self):
        if self._prober is None:
            from meshtrain_b200.worker.capabilities import CapabilityProber

            self._prober = CapabilityProber(self.device, self.supports_dtype)
        return self._prober

    def capabilities(self) -> dict:
        return {"backend": self.backend, "device_name": self.name(), "total_memory": int(self.memory_total()),
                "available_memory": int(self.available_memory()), "unified_memory": self.memory.unified,
                "pinned_memory": self.supports("pinned_memory"), "async_copy": self.supports("async_copy"),
                "nccl": self.supports("nccl"), **self.prober.report()}

    def describe(self) -> dict:
        return {"backend": self.backend, "name": self.name(), "memory_total": self.memory_total(),
                "unified_memory": self.memory.unified}

    def __repr__(self) -> str:
        return f"{type(self).__name__}({self.device})"


class CPUDeviceAdapter(DeviceAdapter):
    backend = "cpu"

    def __init__(self, index: int = 0):
        super().__init__(index, torch.device("cpu"), HostMemory(), InPlaceStager, pinned_pool=False)

    def name(self) -> str:
        return platform.processor() or platform.machine() or "cpu"


class CUDADeviceAdapter(DeviceAdapter):
    backend = "cuda"
    features = frozenset({"pinned_memory", "async_copy", "nccl", "autocast"})

    def __init__(self, index: int = 0):
        if not torch.cuda.is_available():
            raise RuntimeError("CUDA requested but torch.cuda.is_available() is False")
        super().__init__(index, torch.device("cuda", index), CudaMemory(index), StreamStager, pinned_pool=True)

    @property
    def transfer_stream(self):
        return self.stager.stream

    def synchronize(self) -> None:
        torch.cuda.synchronize(self.device)

    def sync_compute(self) -> None:
        torch.cuda.current_stream(self.device).synchronize()

    def name(self) -> str:
        return torch.cuda.get_device_name(self.index)

    def supports_dtype(self, dtype):
        return torch.cuda.is_bf16_supported() if dtype == torch.bfloat16 else True


class MPSDeviceAdapter(DeviceAdapter):
    """Apple Silicon: unified memory, no fp64, synchronous copies."""

    backend = "mps"
    unsupported_dtypes = frozenset({torch.float64})

    def __init__(self, index: int = 0):
        mps = getattr(torch.backends, "mps", None)
        if mps is None or not mps.is_available():
            raise RuntimeError("MPS requested but torch.backends.mps.is_available() is False")
        super().__init__(index, torch.device("mps"), MpsMemory(), BlockingStager, pinned_pool=False)

    def synchronize(self) -> None:
        torch.mps.synchronize()

    def name(self) -> str:
        return f"Apple {platform.machine()} (MPS)"

    def supports(self, operation, dtype=None):
        if dtype is None and operation == "bfloat16":  # depends on the macOS version: probe it
            return self.prober.supports("dtype", "bfloat16")
        return super().supports(operation, dtype)


ADAPTERS: dict[str, type[DeviceAdapter]] = {"cuda": CUDADeviceAdapter, "mps": MPSDeviceAdapter,
                                            "cpu": CPUDeviceAdapter}


def available_backends() -> list[str]:
    """Usable backends in preference order (CUDA, MPS, CPU)."""
    found = []
    if torch.cuda.is_available():
        found.append("cuda")
    mps = getattr(torch.backends, "mps", None)
    if mps is not None and mps.is_available():
        found.append("mps")
    return found + ["cpu"]


def select_device(preferred: str | None = None, index: int | None = None) -> DeviceAdapter:
    """Adapter for ``preferred`` ('cuda', 'cuda:3', 'mps', 'cpu', 'auto'); by default the best available."""
    spec = preferred if preferred not in (None, "", "auto") else available_backends()[0]
    backend, _, suffix = spec.partition(":")
    adapter = ADAPTERS.get(backend)
    if adapter is None:
        raise ValueError(f"unknown backend {backend!r}; expected one of {sorted(ADAPTERS)}")
    return adapter(index if index is not None else int(suffix or 0))
