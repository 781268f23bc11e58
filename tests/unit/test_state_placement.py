"""Tier of the optimizer state (fp32 master weights and Adam moments): fixed, or "auto" from the
startup memory estimate."""

import pytest

from meshtrain_b200.config import parse_config
from meshtrain_b200.coordinator.scheduler import plan_job
from meshtrain_b200.coordinator.state import WorkerRecord
from meshtrain_b200.parallel.placement import StateTierPolicy, config_mode, decide
from meshtrain_b200.parallel.tensor_store import MemoryTier

GB = 1024 ** 3


def test_policy_places_only_optimizer_state_on_the_host():
    host = StateTierPolicy(offload_state=True)
    assert host.place("model.layers.3.qkv.weight.optim.exp_avg", 1, "per_step") is MemoryTier.LOCAL_RAM
    assert host.place("model.layers.3.qkv.weight", 1, "per_microbatch") is MemoryTier.LOCAL_ACCELERATOR
    resident = StateTierPolicy(offload_state=False)
    assert resident.place("model.layers.3.qkv.weight.optim.exp_avg", 1, "per_step") is MemoryTier.LOCAL_ACCELERATOR


def test_decide_and_config_modes():
    asked = []
    assert decide("host", lambda: asked.append(1) or True).offload_state and not asked
    assert not decide("device", lambda: False).offload_state
    assert decide("auto", lambda: False).offload_state and not decide("auto", lambda: True).offload_state
    with pytest.raises(ValueError):
        decide("sometimes", lambda: True)
    base = {"model": {"type": "gpt"}}
    assert config_mode(parse_config({**base, "offload": {"optimizer": "auto"}}).offload) == "auto"
    assert config_mode(parse_config({**base, "offload": {"optimizer": "auto", "params": "host"}}).offload) == "host"
    assert config_mode(parse_config(base).offload) == "device"


LLAMA_2L = {"type": "llama", "layers": 4, "hidden_size": 4096, "heads": 32, "n_kv_heads": 8, "ffn_hidden": 14336,
            "vocab_size": 128256, "seq_len": 4096, "dtype": "bfloat16"}


def _gpu_workers(n, memory_gb):
    return [WorkerRecord(f"g{i}", f"g{i}", {"hostname": "box", "host_id": "box"}, "cuda",
                         {"memory_total": int(memory_gb * GB)}, "127.0.0.1", 100 + i) for i in range(n)]


@pytest.mark.parametrize("memory_gb,expect_offload", [(180, False), (20, True)])
def test_coordinator_offloads_state_only_when_the_resident_plan_does_not_fit(memory_gb, expect_offload):
    cfg = parse_config({"job": {"name": "auto"}, "model": LLAMA_2L, "network": {"tensor_transport": "nccl"},
                        "training": {"batch_size": 8, "microbatch_size": 1, "optimizer": "adam"},
                        "offload": {"optimizer": "auto"}, "placement": {"strategy": "auto", "num_stages": 2},
                        "workers": {"allow": ["cuda"]}})
    plan = plan_job(cfg, _gpu_workers(2, memory_gb))
    assert plan.feasible
    assert plan.state_offload is expect_offload


def test_trainer_auto_offload_from_the_estimate():
    """One CPU rank: a roomy budget keeps the state on the device, a tight one streams it from the host."""
    from meshtrain_b200.api import PipelineTrainer

    model = {"type": "gpt", "layers": 2, "hidden_size": 256, "heads": 4, "vocab_size": 1000, "seq_len": 64,
             "dtype": "float32"}
    roomy = PipelineTrainer(model, num_microbatches=2, device="cpu", microbatch_size=2, offload="auto",
                            memory_gb=64.0)
    assert not roomy.state_tier.offload_state and roomy.engine.offload is None
    roomy.close()
    # params and activations of this model fit in 0.05 GB; with the fp32 state as well they do not
    tight = PipelineTrainer(model, num_microbatches=2, device="cpu", microbatch_size=2, offload="auto",
                            memory_gb=0.05, offload_options={"chunk_mb": 1})
    assert tight.state_tier.offload_state and tight.engine.offload is not None
    x, y = tight.spec.make_batch(0, 4)
    assert tight.loss_value(tight.step(0, x, y)) > 0
    tight.close()
