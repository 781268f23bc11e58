"""``meshtrain train CONFIG --local`` for both runtimes, with checkpoint + resume on the device engine."""

import json
from pathlib import Path

import pytest
import yaml

from meshtrain_b200.cli import main
from meshtrain_b200.telemetry import read_jsonl


def _write(tmp_path, name, cfg):
    p = tmp_path / name
    p.write_text(yaml.safe_dump(cfg))
    return str(p)


def _losses(run_root):
    runs = sorted(Path(run_root).iterdir(), key=lambda p: p.stat().st_mtime)
    recs = read_jsonl(runs[-1] / "metrics.jsonl")
    return [r["loss"] for r in sorted((r for r in recs if "loss" in r), key=lambda r: r["step"])]


def test_host_runtime_local_training(tmp_path):
    cfg = {"job": {"name": "host", "runs_dir": str(tmp_path / "runs")}, "model": {"type": "mlp"},
           "training": {"batch_size": 32, "microbatch_size": 8, "steps": 6, "optimizer": "adam",
                        "learning_rate": 0.001, "log_every": 2},
           "placement": {"strategy": "equal", "num_stages": 2}, "network": {"tensor_transport": "pipe"}}
    assert main(["train", _write(tmp_path, "h.yaml", cfg), "--local"]) == 0
    run = next((tmp_path / "runs").iterdir())
    for f in ("metrics.jsonl", "summary.json", "timeline.json"):
        assert (run / f).exists()
    assert json.loads((run / "summary.json").read_text())["steps"] == 6


def test_device_engine_checkpoint_and_resume(tmp_path):
    base = {"model": {"type": "gpt", "layers": 2, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32},
            "network": {"tensor_transport": "nccl", "timeout_s": 60},
            "placement": {"strategy": "equal", "num_stages": 2}}
    full = {**base, "job": {"name": "full", "runs_dir": str(tmp_path / "full")},
            "training": {"batch_size": 8, "microbatch_size": 2, "steps": 6, "optimizer": "adamw",
                         "learning_rate": 0.001, "log_every": 1}}
    assert main(["train", _write(tmp_path, "full.yaml", full), "--local"]) == 0
    ref = _losses(tmp_path / "full")
    ck = str(tmp_path / "ck")
    part1 = {**base, "job": {"name": "p1", "runs_dir": str(tmp_path / "p1")},
             "training": {**full["training"], "steps": 3, "checkpoint_every": 3, "checkpoint_dir": ck}}
    assert main(["train", _write(tmp_path, "p1.yaml", part1), "--local"]) == 0
    assert (Path(ck) / "step-3" / "stage-0.safetensors").exists()
    # resume with a different stage split: the checkpoint is keyed by layer ids
    part2 = {**base, "job": {"name": "p2", "runs_dir": str(tmp_path / "p2")},
             "placement": {"strategy": "equal", "num_stages": 3},
             "training": {**full["training"], "steps": 3, "resume_from": ck}}
    assert main(["train", _write(tmp_path, "p2.yaml", part2), "--local"]) == 0
    assert _losses(tmp_path / "p1") + _losses(tmp_path / "p2") == pytest.approx(ref, rel=1e-5)


def test_interleaved_checkpoint_resumes_on_another_layout(tmp_path):
    """Two ranks with two model chunks each write one file per chunk (virtual stages 0-3);
    a plain three-stage run resumes from it, and the interleaved layout resumes from a
    plain checkpoint: both continue the uninterrupted loss curve."""
    base = {"model": {"type": "gpt", "layers": 4, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32},
            "network": {"tensor_transport": "nccl", "timeout_s": 60}}
    train = {"batch_size": 8, "microbatch_size": 2, "steps": 6, "optimizer": "adam", "learning_rate": 0.001,
             "log_every": 1}
    interleaved = {"placement": {"strategy": "equal", "num_stages": 2}, "pipeline": {"virtual_stages": 2}}
    plain = {"placement": {"strategy": "equal", "num_stages": 3}}

    def run(name, layout, **training):
        cfg = {**base, **layout, "job": {"name": name, "runs_dir": str(tmp_path / name)},
               "training": {**train, **training}}
        assert main(["train", _write(tmp_path, f"{name}.yaml", cfg), "--local"]) == 0
        return _losses(tmp_path / name)

    ref = run("full", interleaved)
    ck_a, ck_b = str(tmp_path / "ck_a"), str(tmp_path / "ck_b")
    first = run("a1", interleaved, steps=3, checkpoint_every=3, checkpoint_dir=ck_a)
    files = sorted(p.name for p in (Path(ck_a) / "step-3").glob("stage-*.json"))
    assert files == [f"stage-{v}.json" for v in range(4)]
    assert first + run("a2", plain, steps=3, resume_from=ck_a) == pytest.approx(ref, rel=1e-5)
    first = run("b1", plain, steps=3, checkpoint_every=3, checkpoint_dir=ck_b)
    assert first + run("b2", interleaved, steps=3, resume_from=ck_b) == pytest.approx(ref, rel=1e-5)
