"""Worker heartbeat: a 404 re-registers, other HTTP failures are counted and reported, never raised."""

import httpx

from meshtrain_b200.worker.heartbeat import Heartbeat


def _status_error(code: int) -> httpx.HTTPStatusError:
    request = httpx.Request("POST", "http://coordinator/workers/w/heartbeat")
    return httpx.HTTPStatusError("error", request=request, response=httpx.Response(code, request=request))


def test_beat_outcomes():
    outcomes = [False, True, _status_error(404), _status_error(500), httpx.ConnectError("refused"), True]
    forgotten, failed = [], []

    def send():
        result = outcomes.pop(0)
        if isinstance(result, Exception):
            raise result
        return result

    hb = Heartbeat(send, every_s=60, forgotten=lambda: forgotten.append(1), failed=failed.append)
    hb.beat()  # nothing to report yet
    assert hb.sent == 0 and hb.consecutive_failures == 0
    hb.beat()
    assert hb.sent == 1
    hb.beat()  # the coordinator forgot this worker
    assert forgotten == [1] and not failed and hb.consecutive_failures == 1
    hb.beat()
    hb.beat()
    assert len(failed) == 2 and hb.consecutive_failures == 3
    hb.beat()
    assert hb.sent == 2 and hb.consecutive_failures == 0


def test_thread_beats_until_stopped():
    calls = []
    hb = Heartbeat(lambda: calls.append(1) or True, every_s=0.01).start()
    import time

    deadline = time.monotonic() + 5
    while len(calls) < 3 and time.monotonic() < deadline:
        time.sleep(0.01)
    hb.stop()
    assert len(calls) >= 3
