import pytest

from meshtrain_b200.models import build_model_spec
from meshtrain_b200.planner.cost import NVLINK_P2P_BPS, NetworkModel, boundary_transfer_time, pipeline_step_time
from meshtrain_b200.planner.graph import LayerProfile, analytic_profile, profile_model
from meshtrain_b200.planner.memory import estimate_stage_memory
from meshtrain_b200.planner.partition import PlannerOptions, WorkerProfile, b200_box, make_plan, plan_manual
from meshtrain_b200.planner.report import format_accuracy, format_placement, prediction_accuracy

GB = 1024 ** 3


def _workers():
    return [WorkerProfile("a", "gpu-small", "cuda", 8 * GB, 10e12),
            WorkerProfile("b", "gpu-large", "cuda", 12 * GB, 14e12),
            WorkerProfile("c", "laptop", "mps", 10 * GB, 3e12, unified_memory=True,
                          supported_dtypes=("float32", "float16")),
            WorkerProfile("d", "old-pc", "cpu", 4 * GB, 0.1e12)]


@pytest.fixture(scope="module")
def big_layers():
    spec = build_model_spec({"type": "tiny_transformer", "layers": 32, "hidden_size": 1536, "heads": 16,
                             "vocab_size": 8192, "seq_len": 64})
    return profile_model(spec, 2)


def _L(i, flops, act, params=1000):
    return LayerProfile(i, f"l{i}", params // 4, params, act, act, act, flops)


def test_profile_counts_parameters_exactly():
    spec = build_model_spec({"type": "mlp"})
    layers = profile_model(spec, 8)
    assert sum(l.params for l in layers) == sum(p.numel() for p in spec.build_full().parameters())


def test_transfer_time_asymmetric_links_and_step_formula():
    nm = NetworkModel(latency={("a", "b"): 0.001, ("b", "a"): 0.002}, bandwidth={("a", "b"): 100e6, ("b", "a"): 50e6})
    assert nm.transfer_time(100e6, "a", "b") == pytest.approx(1.001)
    assert nm.transfer_time(100e6, "b", "a") == pytest.approx(2.002)
    assert nm.transfer_time(1e9, "a", "a") == 0.0
    assert pipeline_step_time([1.0, 2.0, 1.5], 4) == pytest.approx(12.0)


def test_nvlink_links_skip_host_staging():
    ws, nm = b200_box(2)
    t = boundary_transfer_time(770e6, ws[0], ws[1], nm)
    assert t["kind"] == "nccl" and t["d2h_s"] == 0 and t["h2d_s"] == 0
    assert t["total_s"] == pytest.approx(1e-5 + 770e6 / NVLINK_P2P_BPS)
    host = WorkerProfile("h", "h", "cuda", 8 * GB, 1e12, d2h_Bps=1e9, h2d_Bps=1e9)
    t2 = boundary_transfer_time(1e8, ws[0], host, nm)
    assert t2["kind"] == "host" and t2["h2d_s"] == pytest.approx(0.1)


@pytest.mark.parametrize("strategy", ["equal", "compute", "auto", "topology_aware"])
def test_plans_are_contiguous_and_cover_all_layers(strategy, big_layers):
    opts = PlannerOptions(optimizer="adam", num_microbatches=4, allow_backends=("cuda", "mps"))
    plan = make_plan(strategy, big_layers, _workers(), opts=opts)
    assert plan.stages[0].start == 0 and plan.stages[-1].end == len(big_layers)
    assert all(a.end == b.start for a, b in zip(plan.stages, plan.stages[1:]))
    assert "old-pc" in plan.excluded


def test_auto_respects_budgets_and_needs_several_devices(big_layers):
    opts = PlannerOptions(optimizer="adam", num_microbatches=4, allow_backends=("cuda", "mps"))
    plan = make_plan("auto", big_layers, _workers(), opts=opts)
    assert plan.feasible, plan.format()
    assert all(s.memory.required <= s.memory.budget for s in plan.stages)
    assert not any(make_plan("auto", big_layers, [w], opts=opts).feasible for w in _workers()[:3])
    eq = make_plan("equal", big_layers, _workers(), opts=opts)
    if eq.feasible:
        assert plan.predicted_step_s <= eq.predicted_step_s * 1.001


def test_infeasible_is_reported(big_layers):
    tiny = [WorkerProfile("x", "t1", "cuda", 2 * GB, 1e12), WorkerProfile("y", "t2", "cuda", 2 * GB, 1e12)]
    plan = make_plan("auto", big_layers, tiny, opts=PlannerOptions(optimizer="adam"))
    assert not plan.feasible and plan.violations


def test_dtype_support_excludes_worker():
    layers = profile_model(build_model_spec({"type": "mlp"}), 8)
    plan = make_plan("auto", layers, _workers(), opts=PlannerOptions(dtype="bfloat16"))
    assert "laptop" in plan.excluded


def test_manual_plan_by_id_or_name():
    layers = profile_model(build_model_spec({"type": "mlp"}), 8)
    plan = plan_manual(layers, _workers(), NetworkModel(), PlannerOptions(), [("a", 0, 3), ("gpu-large", 3, 7)])
    assert plan.feasible and [s.worker_name for s in plan.stages] == ["gpu-small", "gpu-large"]
    with pytest.raises(ValueError):
        plan_manual(layers, _workers(), NetworkModel(), PlannerOptions(), [("nope", 0, 7)])


def test_memory_components_and_schedules():
    layers = profile_model(build_model_spec({"type": "tiny_transformer", "layers": 4, "hidden_size": 256,
                                             "heads": 4, "vocab_size": 512, "seq_len": 64}), 4)
    kw = dict(total=8 * GB, num_microbatches=8, is_last=False, stage_index=0, num_stages=3, backend="cuda")
    adam = estimate_stage_memory(layers, optimizer="adamw", schedule="gpipe", **kw)
    sgd = estimate_stage_memory(layers, optimizer="sgd", schedule="gpipe", **kw)
    f1b = estimate_stage_memory(layers, optimizer="adamw", schedule="1f1b", **kw)
    P = adam.parameters
    assert adam.optimizer_state == 2 * P and adam.gradients == P and adam.optimizer_step_temporary == P
    assert sgd.optimizer_state == 0
    assert adam.in_flight == 8 and f1b.in_flight == 3
    assert adam.usable == int(8 * GB * 0.85) - int(0.4 * GB)


def test_device_engine_accounting_and_offload():
    spec = build_model_spec({"type": "gpt", "layers": 4, "hidden_size": 512, "heads": 8, "vocab_size": 1024,
                             "seq_len": 128, "dtype": "bfloat16"})
    layers = analytic_profile(spec, 4)
    n = sum(l.params for l in layers)
    dev = estimate_stage_memory(layers, total=180 * GB, optimizer="adamw", num_microbatches=8, is_last=True,
                                engine="device", param_dtype_bytes=2)
    assert dev.parameters == 2 * n and dev.gradients == 4 * n and dev.master_weights == 4 * n
    assert dev.optimizer_state == 8 * n
    ring = {"chunk_mb": 4.0}  # small chunks: this stage's state is only ~50 MB
    off = estimate_stage_memory(layers, total=180 * GB, optimizer="adamw", num_microbatches=8, is_last=True,
                                engine="device", param_dtype_bytes=2, offload=True, offload_ring=ring)
    assert off.master_weights == 0 and off.optimizer_state == 0 and off.host_offload == 12 * n
    assert off.offload_slots == 2 * 3 * (4 * 1024 ** 2 // 4) * 4  # two slots of master + two moments
    assert off.required < dev.required
    # the default 256 MB chunks give one full-size slot even for a small stage
    default = estimate_stage_memory(layers, total=180 * GB, optimizer="adamw", num_microbatches=8, is_last=True,
                                    engine="device", param_dtype_bytes=2, offload=True)
    assert default.offload_slots == 3 * 256 * 1024 ** 2


def test_llama_8b_needs_more_than_one_b200_and_plans_on_eight():
    spec = build_model_spec({"type": "llama", "layers": 32, "hidden_size": 4096, "heads": 32, "n_kv_heads": 8,
                             "ffn_hidden": 14336, "vocab_size": 128256, "seq_len": 4096, "dtype": "bfloat16"})
    layers = analytic_profile(spec, 1)
    opts = PlannerOptions(optimizer="adamw", num_microbatches=16, schedule="1f1b", engine="device",
                          param_dtype_bytes=2, dtype="bfloat16", num_stages=8)
    ws, nm = b200_box(8)
    plan = make_plan("auto", layers, ws, nm, opts)
    assert plan.feasible, plan.format()
    assert len(plan.stages) == 8
    assert all(s.comm_detail.get("forward", {}).get("kind", "nccl") == "nccl" for s in plan.stages[:-1])
    one = make_plan("auto", layers, ws[:1], nm, PlannerOptions(optimizer="adamw", engine="device",
                                                               param_dtype_bytes=2, dtype="bfloat16"))
    assert not one.feasible


def test_async_transport_overlaps_communication():
    layers = [_L(i, 1e9, 10_000_000) for i in range(4)]
    ws = [WorkerProfile("a", "a", "cpu", 8 * GB, 1e10), WorkerProfile("b", "b", "cpu", 8 * GB, 1e10)]
    net = NetworkModel(bandwidth={("a", "b"): 1e7, ("b", "a"): 1e7})
    sync = make_plan("equal", layers, ws, net, PlannerOptions(num_stages=2))
    asy = make_plan("equal", layers, ws, net, PlannerOptions(num_stages=2, async_transport=True))
    assert asy.predicted_step_s < sync.predicted_step_s


def test_report_and_prediction_accuracy():
    layers = profile_model(build_model_spec({"type": "mlp"}), 8)
    plan = make_plan("equal", layers, _workers()[:2], opts=PlannerOptions(num_stages=2))
    text = format_placement(plan)
    assert "Stage 0" in text and "Stage 1" in text
    summary = {"mean_step_s": plan.predicted_step_s * 2, "stages": {0: {"compute_s": 0.001}, 1: {"compute_s": 0.001}}}
    acc = prediction_accuracy(plan.to_dict(), summary)
    assert acc["step_error"] == pytest.approx(-0.5, rel=1e-6)
    assert "step" in format_accuracy(acc)
