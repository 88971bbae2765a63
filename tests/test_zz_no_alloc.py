"""The allocation-free decode attention entry point gives the same results as the workspace one.

Some hosts of this library cannot allocate device memory for a kernel's scratch space (inference-server plugin
APIs that pass a kernel only its inputs and outputs, FFI callers without a CUDA allocator, serving code that
must not allocate after start-up).  vk_decode_attention_noalloc serves them from a fixed array inside the
library.  This test calls it through the C ABI twice in a row (the array keeps the previous call's contents)
and compares it with vk_decode_attention using a freshly allocated workspace, and both with an fp32 attention
computed by PyTorch, at the tolerance of the other decode-attention tests (0.01 max-abs; the two entry points
share one kernel, so their outputs are expected to be identical).
It is collected last so that a failure here never hides the rest of the suite, and it needs no state from
other tests.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(seed, B, S):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    lens = torch.randint(1, S + 1, (B,), generator=g, device="cuda", dtype=torch.int32)
    lens[0], lens[-1] = 1, S
    q = torch.randn(B, 8, 64, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, S, 2, 64, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, S, 2, 64, generator=g, device="cuda").to(torch.bfloat16)
    return q, k, v, lens


def _run(name, q, k, v, lens, ws=None):
    from viktor_b200._lib import call
    B, S = q.shape[0], k.shape[1]
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream().cuda_stream
    if ws is None:
        call(name, q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr(), out.data_ptr(), B, 0, B, S,
             k.stride(0), k.stride(1), stream)
    else:
        call(name, q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr(), out.data_ptr(), B, 0, B, S,
             k.stride(0), k.stride(1), ws.data_ptr(), ws.numel(), stream)
    return out


def _fp32_attention(q, k, v, lens):
    """softmax(q . K[:L]^T / 8) . V[:L] per query in fp32 (GQA: query head h reads KV head h // 4)."""
    B, S = k.shape[0], k.shape[1]
    kk = k.float().permute(0, 2, 1, 3).repeat_interleave(4, 1)  # [B, 8, S, 64]
    vv = v.float().permute(0, 2, 1, 3).repeat_interleave(4, 1)
    mask = (torch.arange(S, device=k.device)[None, :] < lens[:, None].long())[:, None, None, :]
    o = torch.nn.functional.scaled_dot_product_attention(q.float()[:, :, None, :], kk, vv, attn_mask=mask)
    return o[:, :, 0, :]


def test_noalloc_matches_workspace_entry_point_twice():
    from viktor_b200._lib import check_device_errors, load
    lib = load()
    # calls in a row, different shapes; the last at the array's limit of 4096 positions
    for seed, B, S in [(0, 256, 3200), (1, 48, 700), (3, 64, 4096)]:
        q, k, v, lens = _inputs(seed, B, S)
        ws = torch.zeros(lib.vk_decode_attention_workspace_bytes(B, S), dtype=torch.uint8, device="cuda")
        ref = _run("vk_decode_attention", q, k, v, lens, ws)
        got = _run("vk_decode_attention_noalloc", q, k, v, lens)
        torch.cuda.synchronize()
        check_device_errors()
        assert (got.float() - ref.float()).abs().max().item() < 0.01
        exact = _fp32_attention(q, k, v, lens)
        assert (got.float() - exact).abs().max().item() < 0.01
        assert (ref.float() - exact).abs().max().item() < 0.01


def test_noalloc_clears_stale_tickets():
    """An earlier call that stopped before its merge leaves tickets set; the next call must clear them itself."""
    from viktor_b200._lib import call, check_device_errors, load
    lib = load()
    q, k, v, lens = _inputs(2, 128, 2600)
    ws = torch.zeros(lib.vk_decode_attention_workspace_bytes(128, 2600), dtype=torch.uint8, device="cuda")
    ref = _run("vk_decode_attention", q, k, v, lens, ws)
    stream = torch.cuda.current_stream().cuda_stream
    call("vk_test_noalloc_poison", stream)
    got = torch.full_like(q, float("nan"))  # rows that never merged would keep the NaN
    call("vk_decode_attention_noalloc", q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr(), got.data_ptr(),
         128, 0, 128, 2600, k.stride(0), k.stride(1), stream)
    torch.cuda.synchronize()
    check_device_errors()
    assert not got.isnan().any()
    assert (got.float() - ref.float()).abs().max().item() < 0.01


def test_noalloc_rejects_sizes_beyond_its_array():
    from viktor_b200._lib import VK_ERR_ARG, load
    lib = load()
    q = torch.empty(257, 8, 64, dtype=torch.bfloat16, device="cuda")
    k = torch.empty(257, 16, 2, 64, dtype=torch.bfloat16, device="cuda")
    lens = torch.ones(257, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.vk_decode_attention_noalloc(q.data_ptr(), k.data_ptr(), k.data_ptr(), lens.data_ptr(), q.data_ptr(),
                                         257, 0, 257, 16, k.stride(0), k.stride(1), stream)
    assert rc == VK_ERR_ARG
    # (the buffers match the requested shape, so even an unguarded launch would stay in bounds)
    k2 = torch.zeros(4, 4097, 2, 64, dtype=torch.bfloat16, device="cuda")
    rc = lib.vk_decode_attention_noalloc(q.data_ptr(), k2.data_ptr(), k2.data_ptr(), lens.data_ptr(), q.data_ptr(),
                                         4, 0, 4, 4097, k2.stride(0), k2.stride(1), stream)
    assert rc == VK_ERR_ARG
