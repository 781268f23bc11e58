"""Device adapters and backend selection without the hardware (reference worker/device.py)."""

import types

import pytest
import torch

from meshtrain_b200.worker import device as dv


def test_cpu_adapter_basics():
    a = dv.CPUDeviceAdapter()
    assert a.device.type == "cpu" and a.backend == "cpu"
    assert "cpu" in dv.available_backends()


def test_mps_adapter_with_faked_backend(monkeypatch):
    """Apple path: unified memory, no fp64, no pinned memory / NCCL, memory from torch.mps."""
    monkeypatch.setattr(torch.backends.mps, "is_available", lambda: True)
    fake = types.SimpleNamespace(synchronize=lambda: None, recommended_max_memory=lambda: 16 << 30,
                                 current_allocated_memory=lambda: 1 << 30, driver_allocated_memory=lambda: 3 << 30)
    monkeypatch.setattr(torch, "mps", fake, raising=False)
    a = dv.MPSDeviceAdapter()
    assert a.device == torch.device("mps") and a.backend == "mps"
    a.synchronize()
    assert a.memory_total() == 16 << 30
    st = a.memory_stats()
    assert st["allocated"] == 1 << 30 and st["reserved"] == 3 << 30 and st["unified"]
    assert a.available_memory() == (16 << 30) - (3 << 30)
    assert not a.supports_dtype(torch.float64) and a.supports_dtype(torch.float32)
    assert not a.supports("pinned_memory") and not a.supports("nccl")
    assert "mps" in dv.available_backends()


def test_mps_adapter_refuses_without_backend(monkeypatch):
    monkeypatch.setattr(torch.backends.mps, "is_available", lambda: False)
    with pytest.raises(RuntimeError):
        dv.MPSDeviceAdapter()
