"""The tiny-Transformer correctness gate: 3 CPU stage processes over TCP, GPipe and 1F1B,
Adam 1e-3, uniform tokens; every step's loss within 2e-7 (relative) of one process."""

import pytest

from meshtrain_b200.experiments.transformer import C1_TOLERANCE, run_c1_gate


@pytest.mark.parametrize("schedule", ["gpipe", "1f1b"])
def test_three_tcp_stages_match_one_process(schedule):
    result = run_c1_gate(schedule, steps=10)
    assert len(result["losses"]) == 10
    assert result["losses"][-1] < result["losses"][0]
    assert result["max_rel_deviation"] <= C1_TOLERANCE, result["max_rel_deviation"]
