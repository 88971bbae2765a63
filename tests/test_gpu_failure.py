"""The device-side failure path on a GPU, without faulting it.

Every wait in the kernels is bounded; a wait that runs out sets a bit of the device error word and the kernel
returns.  vk_test_bounded_wait makes one such wait run out on purpose (an mbarrier that nothing arrives on, a
2 ms limit, no copy in flight).  The host must read the bit through vk_read_device_errors, the probe must have
waited at least its limit, and the context must stay usable: a decode-attention launch right after it gives
the same output as before, with a clean error word.
"""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _attention(q, k, v, lens):
    from viktor_b200.ops import decode_attention
    return decode_attention(q, k, v, lens)


def test_bounded_wait_runs_out_and_is_reported():
    from viktor_b200._lib import call, read_device_errors
    torch.cuda.init()
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    B, S = 16, 700
    q = torch.randn(B, 8, 64, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, S, 2, 64, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, S, 2, 64, generator=g, device="cuda").to(torch.bfloat16)
    lens = torch.randint(1, S + 1, (B,), generator=g, device="cuda", dtype=torch.int32)
    before = _attention(q, k, v, lens)
    torch.cuda.synchronize()
    assert read_device_errors(clear=True) == 0

    limit_ns = 2_000_000
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    t0 = time.perf_counter()
    call("vk_test_bounded_wait", limit_ns, waited.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    bits = read_device_errors(clear=True)
    assert bits == 1, f"device error word {bits:#x}: expected only the wait-ran-out bit"
    assert waited.item() >= limit_ns, waited.item()
    assert wall < 5.0

    after = _attention(q, k, v, lens)
    torch.cuda.synchronize()
    assert read_device_errors(clear=True) == 0
    assert torch.equal(after, before)
