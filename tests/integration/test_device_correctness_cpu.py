"""The device-correctness experiment with every stage on the CPU: three stage
processes over loopback TCP against the single-process oracle, 3 steps of AdamW.
Both sides run single-threaded, so every compared quantity agrees to 2e-7."""

from meshtrain_b200.experiments.device_correctness import CPU_TOL, run_device_correctness


def test_cpu_stages_match_the_oracle():
    r = run_device_correctness(["cpu", "cpu", "cpu"], steps=3)
    assert r["tolerance"] == CPU_TOL == 2e-7
    assert r["passed"], r["errors"]
    assert set(r["errors"]) == {"loss", "gradient", "grad_norm", "param_delta", "logits"}
    assert len(r["losses"]) == 3
