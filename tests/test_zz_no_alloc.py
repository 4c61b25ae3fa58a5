"""gpo_reduction_sum_noalloc: the two_pass sum for callers that cannot
allocate device memory (plug-in hosts that own all device memory and hand
a kernel library only its input and output buffers; latency-critical
callers that cannot take the device synchronisation of cudaMalloc/cudaFree).

It is checked through the C-ABI against the existing two_pass strategy of
gpo_launch (which uses a caller-allocated partial-sum buffer) on two calls
in a row — a large one, then a smaller one, so partial sums the first call
left in the shared array must not leak into the second — and the size limit
is checked to be refused before anything is launched.  This file is
collected last so a run that stops at the first failure has already run
every other test.
"""

import pytest
import torch

from gpu_optimizer_b200 import _lib
from gpu_optimizer_b200.runner import build_callable, check_device_status
from oracle import reference as O

pytestmark = pytest.mark.gpu


def existing_two_pass(x, n, bs, warps):
    cfg = {"BLOCK_SIZE": bs, "num_warps": warps, "strategy": "two_pass", "dtype": "float32"}
    return build_callable("reduction", (n,), cfg, (x,)).fn().clone()


def test_noalloc_matches_two_pass_on_consecutive_calls():
    stream = torch.cuda.current_stream().cuda_stream
    rtol, atol = O.tolerance("reduction", "float32")
    out = torch.empty(1, dtype=torch.float32, device="cuda")
    for n, bs, warps, seed in (((1 << 24) + 3, 1024, 8, 0), (100_003, 256, 2, 1)):
        (x,) = O.make_inputs("reduction", (n,), "float32", seed)
        x = x.cuda()
        rc = _lib.reduction_sum_noalloc(x.data_ptr(), n, out.data_ptr(), bs, warps, stream)
        assert rc == _lib.OK, _lib.status_name(rc)
        got = out.clone()
        want = existing_two_pass(x, n, bs, warps)
        check_device_status()
        v = O.check(got.cpu(), want.cpu(), rtol, atol)
        assert v["passed"], (n, v)
        assert O.check(got.cpu(), O.reference("reduction", (x.cpu(),)), rtol, atol)["passed"]


def test_noalloc_refuses_sizes_beyond_its_array():
    stream = torch.cuda.current_stream().cuda_stream
    bs = 256
    n = _lib.NOALLOC_MAX_PARTIALS * bs + 1  # one partial more than the array holds
    x = torch.zeros(n, dtype=torch.float32, device="cuda")
    out = torch.full((1,), 7.0, device="cuda")
    rc = _lib.reduction_sum_noalloc(x.data_ptr(), n, out.data_ptr(), bs, 4, stream)
    assert rc == _lib.BAD_ARGS
    torch.cuda.synchronize()
    assert out.item() == 7.0  # nothing was launched
    # the largest accepted size works
    n_max = _lib.NOALLOC_MAX_PARTIALS * bs
    rc = _lib.reduction_sum_noalloc(x.data_ptr(), n_max, out.data_ptr(), bs, 4, stream)
    assert rc == _lib.OK
    torch.cuda.synchronize()
    assert out.item() == 0.0
