"""Configuration of the newer device-engine options: activation recompute and rebalancing keys."""

import pytest

from meshtrain_b200.config import parse_config

BASE = {"model": {"type": "gpt", "layers": 2, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32}}


@pytest.mark.parametrize("policy", ["none", "all", "every:2", "largest:3"])
def test_recompute_policies_parse(policy):
    cfg = parse_config({**BASE, "training": {"activation_recompute": policy}})
    assert cfg.training.activation_recompute == policy


def test_unknown_recompute_policy_is_refused():
    with pytest.raises(Exception, match="recompute"):
        parse_config({**BASE, "training": {"activation_recompute": "sometimes"}})


def test_rebalance_and_compression_keys():
    cfg = parse_config({**BASE, "pipeline": {"rebalance_after_steps": 5}, "network": {"compression": "bf16"}})
    assert cfg.pipeline.rebalance_after_steps == 5 and cfg.network.compression == "bf16"
    with pytest.raises(Exception):
        parse_config({**BASE, "pipeline": {"rebalance_after_steps": 1}})
    with pytest.raises(Exception):
        parse_config({**BASE, "network": {"compression": "int4"}})
