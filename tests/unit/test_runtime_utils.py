import json
import queue
import threading
import time

import pytest
import torch

from meshtrain_b200.networking.packet import MessageType
from meshtrain_b200.parallel.outbox import Outbox, OutboxError
from meshtrain_b200.parallel.tensor_store import LocalTensorStore, MemoryTier, TensorRole, parameter_id
from meshtrain_b200.summary import format_summary, summarize
from meshtrain_b200.telemetry import EventLogger, MetricsWriter
from meshtrain_b200.utils.buffers import BufferPool, size_class
from meshtrain_b200.utils.timeline import Timeline, covered, sweep, write_chrome_trace
from meshtrain_b200.utils.trace_report import ascii_timeline, format_breakdown, write_run_timeline
from meshtrain_b200.worker.device import CPUDeviceAdapter


# ----------------------------------------------------------------- buffers
class _Ev:
    def __init__(self):
        self.done = False

    def query(self):
        return self.done


def test_buffer_pool_reuses_and_defers_until_event_completes():
    pool = BufferPool()
    a = pool.acquire((4, 4), torch.float32)
    ev = _Ev()
    pool.release(a, ev)
    b = pool.acquire((4, 4), torch.float32)
    assert b.data_ptr() != a.data_ptr() and pool.stats()["deferred"] == 1
    ev.done = True
    pool.release(b)
    c = pool.acquire((4, 4), torch.float32)
    d = pool.acquire((4, 4), torch.float32)
    assert {c.data_ptr(), d.data_ptr()} == {a.data_ptr(), b.data_ptr()}
    assert pool.stats()["reuse_count"] == 2 and pool.stats()["allocation_count"] == 2


def test_buffer_pool_shares_slabs_across_shapes_and_dtypes_of_one_size_class():
    pool = BufferPool()
    a = pool.acquire((1000,), torch.float32)          # 4000 B
    assert size_class(4000) >= 4000 and size_class(4000) <= 4000 * 1.125
    ptr = a.data_ptr()
    pool.release(a)
    b = pool.acquire((30, 33), torch.bfloat16)        # 1980 B: a smaller class, new slab
    c = pool.acquire((999,), torch.int32)             # 3996 B: same class as a
    assert c.data_ptr() == ptr and c.shape == (999,) and c.dtype == torch.int32
    assert b.data_ptr() != ptr
    pool.release(b)
    pool.release(c)
    pool.release(c)  # a second release of the same view is ignored
    assert pool.stats()["bytes_reserved"] == size_class(4000) + size_class(1980)


def test_size_classes_waste_at_most_an_eighth():
    for n in (1, 255, 257, 4097, 20 * 2 ** 20 + 3, 3 * 2 ** 30 + 1):
        c = size_class(n)
        assert c >= n and (n <= 256 or c <= n * 1.125 + 256)


def test_buffer_pool_caps_idle_memory_and_can_be_disabled():
    pool = BufferPool(max_idle_per_class=1, max_bytes=1024)
    x, y = pool.acquire((5,), torch.float32), pool.acquire((5,), torch.float32)
    pool.release(x)
    pool.release(y)  # a second idle slab of the class: over the per-class cap, dropped
    assert pool.stats()["bytes_reserved"] == size_class(20)
    big = pool.acquire((1000,), torch.float32)
    pool.release(big)  # 4000 B > the byte cap: dropped
    assert pool.stats()["bytes_reserved"] == size_class(20)
    off = BufferPool(enabled=False)
    t = off.acquire((3,), torch.int64)
    off.release(t)
    assert off.stats()["allocation_count"] == 0


# ----------------------------------------------------------------- timeline
def test_interval_sweep():
    assert covered([(0, 2), (1, 3), (5, 6)]) == pytest.approx(4.0)
    assert covered([(0, 1.5), (2, 3), (3, 2)]) == pytest.approx(2.5)  # inverted interval ignored
    t = sweep([(0, 3, "a"), (2, 5, "b"), (4, 4, "a")])
    assert t[frozenset("a")] == pytest.approx(2.0) and t[frozenset("b")] == pytest.approx(2.0)
    assert t[frozenset("ab")] == pytest.approx(1.0) and frozenset() not in t


def test_step_metrics_overlap_and_idle():
    tl = Timeline("w", 0)
    t0 = 1000.0
    tl.add("FORWARD_COMPUTE", t0, t0 + 0.4, 0, 0)
    tl.add("NETWORK_SEND", t0 + 0.3, t0 + 0.6, 0, 0)
    m = tl.step_metrics(0, (t0, t0 + 1.0))
    assert m["compute_s"] == pytest.approx(0.4) and m["communication_s"] == pytest.approx(0.3)
    assert m["overlapped_s"] == pytest.approx(0.1) and m["exposed_communication_s"] == pytest.approx(0.2)
    assert m["idle_s"] == pytest.approx(0.4)


def test_chrome_trace_and_ascii(tmp_path):
    tl = Timeline("w", 1)
    with tl.span("FORWARD_COMPUTE", 3, 0):
        time.sleep(0.002)
    with tl.span("NETWORK_SEND", 3, 0):
        time.sleep(0.002)
    path = write_chrome_trace(tmp_path / "t.json", [tl.to_chrome_events()])
    ev = json.loads(path.read_text())["traceEvents"]
    assert any(e.get("ph") == "X" and e["name"] == "FORWARD_COMPUTE mb0" for e in ev)
    run = write_run_timeline(tmp_path / "run.json", [(1, "w", tl.export())])
    assert run.exists()
    txt = ascii_timeline([(1, "w", tl.export())], step=3, width=40)
    assert "F" in txt and ">" in txt and "stage 1" in txt
    assert "no spans" in ascii_timeline([(1, "w", tl.export())], step=9)


def test_breakdown_text():
    s = {"mean_step_s": 1.0, "stages": {0: {"worker": "a", "backend": "cpu", "compute_s": 0.5, "comm_s": 0.2,
                                            "exposed_communication_s": 0.1, "idle_s": 0.4, "overlap_ratio": 0.5}}}
    out = format_breakdown(s)
    assert "Worker a" in out and "50%" in out


# ----------------------------------------------------------------- tensor store
def test_tensor_store_roles_tiers_manifest():
    st = LocalTensorStore("w0")
    w = torch.randn(3, 4)
    pid = parameter_id(5, "fc1.weight")
    st.put(pid, w, TensorRole.PARAMETER)
    st.put("a", torch.zeros(10), TensorRole.ACTIVATION)
    assert st.get(pid) is w and st.locate(pid).tier is MemoryTier.LOCAL_RAM
    assert st.bytes_by_role()[TensorRole.PARAMETER.value] == 48
    assert [m["tensor_id"] for m in st.manifest()] == sorted([pid, "a"])
    st.evict(pid, MemoryTier.LOCAL_RAM)  # already host-resident: no-op
    with pytest.raises(NotImplementedError):
        st.evict(pid, MemoryTier.REMOTE_RAM)
    st.discard("a")
    with pytest.raises(KeyError):
        st.get("a")


# ----------------------------------------------------------------- outbox
class _Recorder:
    def __init__(self, delay=0.0, fail=False):
        self.sent, self.delay, self.fail, self.bytes_sent = [], delay, fail, 0

    def send_packet(self, pkt):
        if self.fail:
            raise ConnectionError("peer gone")
        time.sleep(self.delay)
        self.sent.append(pkt)
        self.bytes_sent += len(pkt.payload)


@pytest.mark.parametrize("async_mode", [False, True])
def test_outbox_delivers_in_order_and_notifies(async_mode):
    link = _Recorder(delay=0.001)
    events = queue.Queue()
    ob = Outbox({"down": link}, Timeline(), async_mode=async_mode, events=events)
    dev = CPUDeviceAdapter()
    for mb in range(5):
        ob.submit_tensor("down", torch.full((4,), float(mb)), MessageType.FORWARD_ACTIVATION, device=dev, step=0,
                         microbatch=mb, notify=True)
    ob.flush(5)
    assert [p.microbatch_id for p in link.sent] == list(range(5))
    assert ob.bytes_sent["down"] == 5 * 16
    assert sorted(events.get_nowait()[3] for _ in range(5)) == list(range(5))
    ob.close()


def test_outbox_surfaces_send_failures():
    ob = Outbox({"down": _Recorder(fail=True)}, Timeline(), async_mode=True, timeout_s=2)
    ob.submit_tensor("down", torch.zeros(2), MessageType.FORWARD_ACTIVATION, device=CPUDeviceAdapter(), step=0,
                     microbatch=0)
    with pytest.raises(OutboxError, match="peer gone"):
        ob.flush(2)
    ob.close()


def test_outbox_backpressure_when_queue_full():
    gate = threading.Event()

    class Blocked(_Recorder):
        def send_packet(self, pkt):
            gate.wait(5)
            super().send_packet(pkt)

    ob = Outbox({"down": Blocked()}, Timeline(), async_mode=True, max_queue=1, timeout_s=0.3)
    dev = CPUDeviceAdapter()
    with pytest.raises(OutboxError, match="full"):
        for mb in range(4):
            ob.submit_tensor("down", torch.zeros(2), MessageType.FORWARD_ACTIVATION, device=dev, step=0, microbatch=mb)
    gate.set()
    ob.close()


# ----------------------------------------------------------------- telemetry / summary
def test_logger_and_metrics_roundtrip(tmp_path):
    log = EventLogger("w", "job", jsonl_path=tmp_path / "events.jsonl")
    line = log.log("STEP_COMPLETE", step=1, loss=0.5)
    assert "STEP_COMPLETE" in line and "loss=0.5" in line
    log.close()
    mw = MetricsWriter(tmp_path / "m.jsonl")
    recs = [{"event": "STEP_COMPLETE", "stage": s, "step": i, "step_s": 0.1 * (s + 1), "loss": 2.0 - i * 0.1,
             "worker": f"w{s}", "backend": "cpu", "samples_per_s": 10.0} for i in range(4) for s in range(2)]
    for r in recs:
        mw.write(r)
    back = mw.read()
    assert len(back) == 8
    s = summarize(back, warmup_steps=1)
    assert s["steps"] == 4 and s["timed_steps"] == 3 and s["mean_step_s"] == pytest.approx(0.2)
    assert s["final_loss"] == pytest.approx(1.7)
    assert "mean step" in format_summary(s)


def test_work_duration_reads_torch_work_timing():
    """NCCL works expose their device time as ``Work._get_duration`` (ms)."""
    from meshtrain_b200.parallel.p2p import work_duration_ms

    class Timed:
        def _get_duration(self):
            return 0.25

    class Untimed:
        def _get_duration(self):
            raise RuntimeError("timing not enabled")

    assert work_duration_ms(Timed()) == 0.25
    assert work_duration_ms(Untimed()) is None
    assert work_duration_ms(object()) is None
