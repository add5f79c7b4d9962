"""GPU: failure detection without a GPU fault.

Every wait in this library's kernels (mbarrier phases between the load, MMA, producer and
softmax warps) goes through one bounded wait.  The self-test entry point runs that wait on an
mbarrier that nothing arrives on: the wait must give up after its time limit (2 s), report
NVFP4KV_DEVERR_TIMEOUT in the caller's error word and let the kernel return, so that the CUDA
context stays usable; a decode call afterwards must run clean and match the oracle.
"""
import ctypes
import math
import time

import numpy as np
import pytest
import torch

from glm53_flash_dual_dgx_spark_b200 import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    from glm53_flash_dual_dgx_spark_b200 import glm53_nvfp4_runtime as rt
    lib = _lib.lib()
    torch.cuda.set_device(0)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    t0 = time.monotonic()
    _lib.check(lib.nvfp4kv_selftest_bounded_wait(ctypes.c_void_p(err.data_ptr()), stream), "selftest")
    torch.cuda.synchronize()                      # a fault or a hang would surface here
    elapsed = time.monotonic() - t0
    assert int(err.item()) == _lib.DEVERR_TIMEOUT
    assert 1.5 < elapsed < 30.0, f"the bounded wait ended after {elapsed:.2f} s"

    # the context is still usable
    rt.device_errors()
    g = torch.Generator().manual_seed(9)
    pages, ctx = 16, 1000
    pool_np = O.quant_new(torch.randn(pages * 64, 512, generator=g).to(torch.bfloat16))
    pool = torch.from_numpy(pool_np).cuda().view(pages, 64, 288)
    tables = torch.randperm(pages, generator=g)[:16].view(1, 16).to(torch.int32)
    q = torch.randn(1, 1, 64, 576, generator=g).to(torch.bfloat16)
    sl = torch.tensor([ctx], dtype=torch.int32)
    sm = 1.0 / math.sqrt(576)
    out = rt.mla_decode(q.cuda(), pool, None, 128, 512, 64, tables.cuda(), sl.cuda(), ctx, bmm1_scale=sm)
    torch.cuda.synchronize()
    assert rt.device_errors() == 0
    ref = O.mla_decode(q.float(), pool_np, tables.numpy(), sl.numpy(), sparse=False, bmm1_scale=sm)
    assert np.allclose(out.float().cpu().numpy(), ref, rtol=2e-2, atol=1e-2)
