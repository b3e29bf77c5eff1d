"""Bounded waits of the expert-parallel communicator (no GPU kernel waits).

The reference's device layer waits on fences without a bound
(har/crates/har-vulkan/src/lib.rs:2174) and its serving seam fails closed on
any GPU error (har/crates/har-serve/src/vulkan.rs:18-19).  Here a rank that
never joins makes har_cuda_ep_create_timeout return HAR_CUDA_ERR_TIMEOUT
after the bound instead of blocking its caller forever: the failure is made
on the host (the second rank simply does not exist), so no kernel is in
flight and no GPU wait is involved.  The aborted communicator leaves the
context usable."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import har_cuda  # noqa: E402


@pytest.mark.timeout(120)
def test_ep_create_times_out_when_a_rank_never_joins():
    ctx = har_cuda.Context(0)
    uid = har_cuda.ep_unique_id()
    t0 = time.monotonic()
    with pytest.raises(har_cuda.HarCudaError) as e:
        ctx.ep_create(uid, 2, 0, timeout_ms=3000)  # rank 1 of 2 never comes
    dt = time.monotonic() - t0
    assert e.value.status == har_cuda.ERR_TIMEOUT
    assert 2.5 < dt < 60.0, dt
    # the context still works
    x = torch.ones(4, device="cuda")
    torch.cuda.synchronize()
    ctx.synchronize()
    assert float(x.sum()) == 4.0
    # a one-rank communicator joins at once and frees cleanly
    ep = ctx.ep_create(har_cuda.ep_unique_id(), 1, 0, timeout_ms=10000)
    ep.abort()
    ep.free()
    ctx.close()
