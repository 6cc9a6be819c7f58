"""GPU-queued submit (descriptor ring + done_idx) through the queue client: this
library's ring consumer and, where it was built, the reference's own CPU poller on the
same submit kernel (gfd_b200/csrc/queue_client.cu built against both header trees).
Both must land the same bytes the oracle gathers."""
import os

import numpy as np
import pytest

from gfd_b200 import entries_array
from gfd_b200 import workloads as wl
from tests.golden.cases import oracle_gather

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
OURS = os.path.join(ROOT, "gfd_b200", "libgfd_queue_client.so")
REF = os.path.join(ROOT, "oracle", "_ref", "libgfd_ref_queue.so")


@pytest.mark.parametrize("path", [OURS, REF], ids=["ours", "reference"])
@pytest.mark.parametrize("n,size", [(256, 4096), (3000, 1024), (64, 65536)])
def test_queue_mode_lands_oracle_bytes(gpu_ctx, path, n, size):
    import torch
    import bench
    if not os.path.exists(path):
        pytest.skip("reference queue client not built")
    pool = gpu_ctx.pool(2 * n * size)
    wl.fill_bytes(pool.ptr, pool.nbytes, n)
    dst = torch.zeros(n * size, dtype=torch.uint8, device="cuda")
    addrs = np.uint64(pool.ptr) + wl.permutation(2 * n, size)[:n].astype(np.uint64) * np.uint64(size)
    qc = bench.QueueClientLib(path, 0, dst.data_ptr(), pool.ptr, pool.nbytes)
    try:
        for _ in range(3):  # ring positions advance between rounds
            dst.zero_()
            torch.cuda.synchronize()
            assert qc.run_us(addrs, size) > 0
            got = dst.cpu().numpy()
            want = np.zeros(n * size, np.uint8)
            e = entries_array(np.uint64(want.ctypes.data) + np.arange(n, dtype=np.uint64) * np.uint64(size),
                              addrs, size)
            assert oracle_gather(want, want.ctypes.data, e) == -1
            assert np.array_equal(got, want)
    finally:
        qc.close()
        pool.free()
