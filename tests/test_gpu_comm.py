"""The NCCL binding of the sharded forward (comm.NcclComm) on one GPU: a one-rank communicator
through ncclCommInitRank, the logits all-gather of sharding.gather_rows on device arrays, the
bounded wait and the teardown.  (Several ranks need several GPUs; their host logic runs as gloo
ranks in test_multirank.py.)"""
import numpy as np
import pytest

from salt_b200 import device as D
from salt_b200.comm import NcclComm, new_unique_id, nccl_version
from salt_b200.sharding import gather_rows

pytestmark = pytest.mark.gpu


def test_one_rank_all_gather_round_trip():
    assert nccl_version() >= 21800
    comm = NcclComm(0, 1, new_unique_id())
    rows = np.arange(12 * 10, dtype=np.int32).reshape(12, 10) * 7 - 3
    local = D.to_device(rows, np.int32)
    out = gather_rows(local, comm)
    comm.wait(30.0)
    assert out.shape == (12, 10)
    np.testing.assert_array_equal(out.numpy(), rows)
    comm.close()


def test_gather_rejects_mismatched_buffers():
    comm = NcclComm(0, 1, new_unique_id())
    with pytest.raises(ValueError):
        comm.all_gather(D.empty((4, 3), np.int32), D.empty((5, 3), np.int32))
    comm.close()
