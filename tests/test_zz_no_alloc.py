"""vtq_linear_host_noalloc: the integer linear for callers that cannot allocate
device memory (their memory belongs to a pool or budget they do not control).

It stages x, y and the status word in the library's static device array
instead of a cudaMalloc'd buffer. Called twice in a row through the C ABI, it
must give exactly the result of vtq_linear with host pointers (bit-exact, the
tolerance every parity test here uses). This file is collected last so that a
stop-at-first-failure run has already run every other test.
"""
import numpy as np
import pytest

import vtq
from vtq import synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,n,r,batch", [(vtq.Q4_K, 4096, 1100, 1), (vtq.Q6_K, 2048, 300, 3)])
def test_noalloc_matches_vtq_linear_twice(dtype, n, r, batch):
    import torch
    lib = vtq.load_library()
    w = synth.weight(dtype, "noalloc.w", r, n)
    # Weights in caller-owned device memory (here torch's), in the kernels' layout.
    raw = torch.from_numpy(w).cuda()
    dst = torch.empty(lib.vtq_device_layout_bytes(dtype, n, r), dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert lib.vtq_device_repack(dtype, n, r, raw.data_ptr(), dst.data_ptr(), st) == vtq.OK
    torch.cuda.synchronize()
    ctx = vtq.Context(0)
    wt = ctx.upload(dtype, w, n, r)
    xs = [synth.activation(f"noalloc.x{call}", batch, n) for call in range(2)]
    refs = [ctx.linear(wt, x, batch) for x in xs]
    # A first call on this device looks up the static array's address (and
    # CUDA may load the library's device code on first use); after it, the
    # calls must leave the device's free memory unchanged.
    y = np.empty(batch * r, np.float32)
    assert lib.vtq_linear_host_noalloc(dtype, dst.data_ptr(), n, r, xs[0].ctypes.data,
                                       y.ctypes.data, batch, st) == vtq.OK
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for call, (x, ref) in enumerate(zip(xs, refs)):
        y = np.full(batch * r, np.nan, np.float32)
        assert lib.vtq_linear_host_noalloc(dtype, dst.data_ptr(), n, r, x.ctypes.data,
                                           y.ctypes.data, batch, st) == vtq.OK
        assert np.array_equal(y.view(np.uint32), ref.view(np.uint32)), f"call {call}"
    assert torch.cuda.mem_get_info()[0] == free0
    ctx.close()


def test_noalloc_rejects_sizes_over_its_limit():
    lib = vtq.load_library()
    x = np.zeros(4, np.float32)
    y = np.zeros(4, np.float32)
    # 200 rows of 4096 inputs: 819,200 staged x floats > the 262,144-float array.
    assert lib.vtq_linear_host_noalloc(vtq.Q4_K, 16, 4096, 1, x.ctypes.data, y.ctypes.data, 200,
                                       None) == vtq.ERR_INTERNAL
