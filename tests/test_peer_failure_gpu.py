"""Two GPU stages over NCCL: a rank that fails between steps stops the other one.

Same scenario as tests/distributed/test_peer_failure.py on two B200s: the
victim raises when it starts step 2 (none of its kernels or NCCL calls of that
step launched), reports through the job's store and leaves; the survivor must
end with ``PeerFailure`` naming the victim within seconds.  NVLS is off
(``NCCL_NVLS_ENABLE=0``): no memory of a rank that leaves is bound to an NVLink
multicast object.
"""

import pytest

from meshtrain_b200.parallel.spawn import spawn_ranks
from distributed.test_peer_failure import _run_until_failure

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


@pytest.mark.parametrize("victim", [0, 1])
def test_nccl_pipeline_rank_failure_stops_the_other_rank(victim):
    env = {"MESHTRAIN_PG_TIMEOUT_S": "30", "MESHTRAIN_PEER_TIMEOUT_S": "10", "NCCL_NVLS_ENABLE": "0"}
    outcomes = spawn_ranks(_run_until_failure, 2, victim, 2, None, env=env, timeout_s=180)
    survivor = outcomes[1 - victim]
    assert outcomes[victim]["error"] == "RuntimeError" and outcomes[victim]["steps"] == 2
    assert survivor["error"] == "PeerFailure" and f"rank {victim}" in survivor["message"], survivor
    assert survivor["steps"] <= 3 and survivor["seconds"] < 25, survivor
