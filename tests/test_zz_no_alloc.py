"""Allocation-free gated-attention backward, called through its exported C symbol.

The entry point ``eb_gated_attention_bwd_noalloc`` serves callers that may
not allocate device memory; it keeps its scratch in a fixed device array.
This file is collected last on purpose. Two calls in a row with different
shapes (so the second sees the first call's leftover scratch) must match the
regular backward entry point within the bf16 tolerance of the other tests.
"""
import ctypes

import pytest
import torch

from exploration_b200.ops import _native

pytestmark = pytest.mark.gpu

ATOL, RTOL = 3e-2, 5e-2


def entry_point():
    _native.load(required=True)        # makes sure torch's libraries are resident
    lib = ctypes.CDLL(str(_native.so_path()))
    fn = lib.eb_gated_attention_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 13 + [ctypes.c_int] * 6 + [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int]
    return fn


def status_reader():
    lib = ctypes.CDLL(str(_native.so_path()))
    fn = lib.eb_gated_attention_bwd_noalloc_status
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int), ctypes.c_char_p,
                   ctypes.c_int]
    return fn


def wait_record(device):
    """(site, cta) of a bounded wait of the allocation-free kernels that gave up; (0, 0) when none did."""
    site, cta = ctypes.c_int(-1), ctypes.c_int(-1)
    message = ctypes.create_string_buffer(256)
    status = status_reader()(device, ctypes.byref(site), ctypes.byref(cta), message, len(message))
    assert status == 0, message.value.decode()
    return site.value, cta.value


def forward_case(seed, batch, queries, keys, heads, dim, block):
    ext = _native.load(required=True)
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(batch, queries, heads, dim, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(batch, keys, heads, dim, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(batch, keys, heads, dim, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.sort(torch.randint(0, keys, (batch, queries), device="cuda", generator=g), 1).values
    pos[0, 0] = -1
    pos = pos.to(torch.int32).contiguous()
    out, rc, pr, zr, lse = ext.gated_attention_fwd(q, k, v, pos, block)
    grad = torch.randn(q.shape, device="cuda", generator=g).to(torch.bfloat16)
    return ext, (grad, q, k, v, pos, out, rc, pr, zr, lse)


def call(fn, tensors, dq, dk, dv, batch, queries, keys, heads, dim, block):
    message = ctypes.create_string_buffer(256)
    ptrs = [t.data_ptr() for t in tensors] + [dq.data_ptr(), dk.data_ptr(), dv.data_ptr()]
    stream = torch.cuda.current_stream().cuda_stream
    status = fn(*ptrs, batch, queries, keys, heads, dim, block, stream, message, len(message))
    return status, message.value.decode()


def test_noalloc_backward_matches_regular_entry_point_twice(native):
    fn = entry_point()
    # One warpgroup split (block <= 64: two gradient warpgroups) and one without, at both head sizes.
    cases = [(11, 1, 300, 640, 3, 64, 16), (12, 2, 200, 520, 2, 128, 128), (13, 1, 260, 700, 2, 128, 32)]
    for seed, batch, queries, keys, heads, dim, block in cases:
        ext, tensors = forward_case(seed, batch, queries, keys, heads, dim, block)
        want = ext.gated_attention_bwd(*tensors, block)
        dq, dk, dv = (torch.full_like(t, float("nan")) for t in tensors[1:4])
        status, message = call(fn, tensors, dq, dk, dv, batch, queries, keys, heads, dim, block)
        assert status == 0, message
        torch.cuda.synchronize()
        assert wait_record(torch.cuda.current_device()) == (0, 0)
        for name, got, ref in zip(("dq", "dk", "dv"), (dq, dk, dv), want):
            torch.testing.assert_close(got.float(), ref.float(), atol=ATOL, rtol=RTOL, msg=name)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    fn = entry_point()
    empty = torch.empty(0, device="cuda")
    status, message = call(fn, [empty] * 10, empty, empty, empty, 1, 1 << 20, 1024, 4, 64, 16)
    assert status != 0 and "exceeds" in message
