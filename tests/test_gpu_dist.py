"""Sharded reductions, argmax and batched matmul through the product path:
two ranks (spawned processes over gloo) each run the CUDA kernels on their
slice on cuda:0, then the gathered results are checked against the unsharded
computation.  The ranks' kernels are independent (no kernel waits on another
rank), so both ranks may share one GPU."""
import pytest

from test_dist_gloo import check_sharded, run_sharded

pytestmark = pytest.mark.gpu


def test_sharded_ops_on_gpu():
    check_sharded(run_sharded(2, use_gpu=True), 2, exact_rows=False)
