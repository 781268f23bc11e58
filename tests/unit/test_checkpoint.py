import pytest
import torch

from meshtrain_b200.checkpoint import (latest_step, load_for_layers, load_host_stage, load_stage_checkpoint,
                                       load_tensors, save_host_stage, save_stage_checkpoint, save_tensors,
                                       write_manifest)
from meshtrain_b200.models import build_model_spec
from meshtrain_b200.parallel.engine import PipelineEngine
from meshtrain_b200.parallel.stage import Stage

GPT = {"type": "gpt", "layers": 3, "hidden_size": 64, "heads": 4, "vocab_size": 96, "seq_len": 32, "dtype": "float32"}


def test_file_format_roundtrip_and_safetensors_compat(tmp_path):
    ts = {"a": torch.randn(3, 5), "b": torch.arange(7, dtype=torch.int64), "c": torch.randn(4).to(torch.bfloat16),
          "e": torch.empty(0, 3)}
    save_tensors(tmp_path / "x.safetensors", ts, {"step": 3})
    back = load_tensors(tmp_path / "x.safetensors")
    for k, v in ts.items():
        assert back[k].dtype == v.dtype and torch.equal(back[k], v)
    st = pytest.importorskip("safetensors.torch")
    lib = st.load_file(str(tmp_path / "x.safetensors"))
    assert all(torch.equal(lib[k], v) for k, v in ts.items())


def _engine(rng, spec):
    return PipelineEngine(spec, layer_range=rng, stage=0, num_stages=1, device="cpu", num_microbatches=2,
                          optimizer="adamw", lr=1e-3, weight_decay=0.01)


def _train(eng, spec, steps):
    out = []
    for s in steps:
        x, y = spec.make_batch(s, 4)
        out.append(float(eng.train_step(s, x, y).loss))
    return out


def test_resume_matches_uninterrupted_training(tmp_path):
    spec = build_model_spec(GPT, seed=5)
    n = spec.num_layers
    ref = _train(_engine((0, n), spec), spec, range(4))
    eng = _engine((0, n), spec)
    first = _train(eng, spec, range(2))
    save_stage_checkpoint(tmp_path, eng, step=2)
    write_manifest(tmp_path, 2, ranges=[(0, n)], config=GPT)
    assert latest_step(tmp_path) == 2
    fresh = _engine((0, n), build_model_spec(GPT, seed=99))  # different init: everything must come from the file
    assert load_stage_checkpoint(tmp_path, fresh) == 2
    assert first + _train(fresh, spec, range(2, 4)) == pytest.approx(ref, rel=1e-6)


def test_checkpoint_repartitions_across_stage_counts(tmp_path):
    spec = build_model_spec(GPT, seed=1)
    n = spec.num_layers
    ranges = [(0, 2), (2, n)]
    engines = []
    for i, r in enumerate(ranges):
        e = _engine(r, spec)
        e.stage = i
        engines.append(e)
        save_stage_checkpoint(tmp_path, e, step=7)
    write_manifest(tmp_path, 7, ranges=ranges)
    whole = load_for_layers(tmp_path, 7, (0, n))
    for e in engines:
        for k, v in e.state_dict().items():
            if k != "optim.step":
                assert torch.equal(whole[k], v), k
    mid = load_for_layers(tmp_path, 7, (1, 3))
    assert {int(k.split(".")[2]) for k in mid if k.startswith("model.")} == {1, 2}


def test_incomplete_step_is_refused(tmp_path):
    spec = build_model_spec(GPT)
    e = _engine((0, 2), spec)
    save_stage_checkpoint(tmp_path, e, step=1)
    with pytest.raises(FileNotFoundError, match="incomplete"):
        write_manifest(tmp_path, 1, ranges=[(0, 2), (2, 5)])


def test_host_stage_roundtrip(tmp_path):
    spec = build_model_spec({"type": "mlp"}, seed=0)
    st = Stage(spec.build_stage(0, 3), stage_index=0, num_stages=2, optimizer="adam", lr=1e-3)
    x, _ = spec.make_batch(0, 8)
    st.module(x).sum().backward()
    st.optimizer.step()
    save_host_stage(tmp_path, st, step=1, layers=(0, 3))
    write_manifest(tmp_path, 1, ranges=[(0, 3)])
    other = Stage(build_model_spec({"type": "mlp"}, seed=3).build_stage(0, 3), stage_index=0, num_stages=2,
                  optimizer="adam", lr=1e-3)
    assert load_host_stage(tmp_path, other, (0, 3)) == 1
    for (n, a), (_, b) in zip(st.module.named_parameters(), other.module.named_parameters()):
        assert torch.equal(a, b), n
        assert torch.equal(st.optimizer.state[a]["exp_avg"], other.optimizer.state[b]["exp_avg"])
