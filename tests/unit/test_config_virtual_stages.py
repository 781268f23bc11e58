"""Config keys of the device engine: virtual stages and the offload slot budget."""

import pytest

from meshtrain_b200.config import parse_config

BASE = {"job": {"name": "t"}, "model": {"type": "gpt", "layers": 4, "hidden_size": 64, "heads": 4,
                                        "vocab_size": 96, "seq_len": 32},
        "training": {"steps": 1, "batch_size": 8, "microbatch_size": 2}}


def _cfg(**sections):
    d = {k: dict(v) for k, v in BASE.items()}
    for k, v in sections.items():
        d[k] = v
    return parse_config(d)


def test_defaults():
    c = _cfg()
    assert c.pipeline.virtual_stages == 1
    assert c.offload.device_budget_gb is None


def test_virtual_stages_and_budget_parse():
    c = _cfg(pipeline={"schedule": "1f1b", "virtual_stages": 2}, offload={"optimizer": "host", "device_budget_gb": 8})
    assert c.pipeline.virtual_stages == 2
    assert c.offload.device_budget_gb == 8


@pytest.mark.parametrize("bad", [0, 9])
def test_virtual_stages_bounds(bad):
    with pytest.raises(Exception):
        _cfg(pipeline={"virtual_stages": bad})


def test_virtual_stages_need_1f1b_and_may_checkpoint():
    with pytest.raises(Exception, match="1f1b"):
        _cfg(pipeline={"schedule": "gpipe", "virtual_stages": 2})
    c = _cfg(pipeline={"virtual_stages": 2}, training={"steps": 2, "batch_size": 8, "microbatch_size": 2,
                                                        "checkpoint_every": 1})
    assert c.training.checkpoint_every == 1
