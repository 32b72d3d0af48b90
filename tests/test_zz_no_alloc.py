"""The allocation-free quantize entry point (nvfp4_quantize_auto_scale_noalloc).

It exists for callers that cannot allocate device memory — a plugin inside another runtime's
enqueue call where allocation is forbidden, a process whose device memory belongs to a pool it
does not control, code with a fixed memory budget. Instead of a caller workspace it uses a fixed
32 KiB scratch array inside the library. These tests call it through the C ABI and check that it
gives the same bytes and scale as the workspace entry point, on two calls in a row (the scratch
keeps the previous call's contents, so the second call must not be influenced by the first), and
that inputs beyond its 2^30-element limit are refused up front.

This file is collected last so that a run stopping at its first failure has already run every
other test."""
import pytest
import torch

from my_nvfp4_gemm_b200 import capi

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _outputs(x):
    q = torch.empty(x.numel() // 2, dtype=torch.uint8, device="cuda")
    sf = torch.empty(x.numel() // 16, dtype=torch.uint8, device="cuda")
    s = torch.empty((), dtype=torch.float32, device="cuda")
    return q, sf, s


def _with_workspace(x):
    q, sf, s = _outputs(x)
    ws_bytes = capi.quantize_auto_scale_workspace_bytes(x.numel())
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    capi.check(capi.quantize_auto_scale(x.data_ptr(), x.numel(), q.data_ptr(), sf.data_ptr(),
                                        s.data_ptr(), ws.data_ptr(), ws_bytes, _stream()),
               "nvfp4_quantize_auto_scale")
    torch.cuda.synchronize()
    return q, sf, s


def _without_allocation(x):
    q, sf, s = _outputs(x)
    capi.check(capi.quantize_auto_scale_noalloc(x.data_ptr(), x.numel(), q.data_ptr(),
                                                sf.data_ptr(), s.data_ptr(), _stream()),
               "nvfp4_quantize_auto_scale_noalloc")
    torch.cuda.synchronize()
    return q, sf, s


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    g = torch.Generator(device="cuda").manual_seed(5)
    # First call: many chunks and a large amax; second call: few chunks and a small amax, so
    # partial maxima left in the shared scratch by the first call would change the second's
    # scale if they were read.
    first = torch.randn(4096, 8192, device="cuda", generator=g)
    first[100, 200] = 3.0e4
    second = torch.randn(1000, 272, device="cuda", generator=g) * 0.01
    for x in (first.to(torch.bfloat16), second.to(torch.bfloat16)):
        q0, sf0, s0 = _with_workspace(x)
        q1, sf1, s1 = _without_allocation(x)
        s_ref = 6 * 448 / x.abs().max().to(dtype=torch.float32)
        assert s1.view(torch.int32).item() == s0.view(torch.int32).item()
        assert s1.view(torch.int32).item() == s_ref.view(torch.int32).item()
        assert torch.equal(q1, q0) and torch.equal(sf1, sf0)


def test_noalloc_refuses_inputs_beyond_its_scratch():
    too_many = (1 << 30) + 16
    fake = 0x10000  # never dereferenced: the size check comes first
    assert capi.quantize_auto_scale_noalloc(fake, too_many, fake, fake, fake, _stream()) == 7
