"""The allocation-free dispatch-plan entry point, called through its exported C symbol.

Callers that cannot allocate device memory when they need a plan (engines
with one fixed arena, C programs without PyTorch's allocator) use
``pm_moe_plan_noalloc``; it must produce exactly the plan of the allocating
PyTorch entry point ``moe_plan``.  This file is collected last on purpose.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from placemoe_b200 import _build

    lib = ctypes.CDLL(_build._so_path(_build.KERNELS_NAME))
    fn = lib.pm_moe_plan_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p]
    lib.pm_moe_plan_noalloc_error.restype = ctypes.c_char_p
    lib.pm_moe_plan_noalloc_scratch_ints.restype = ctypes.c_int
    return lib


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _call(lib, idx, lut, w, num_slots, cap, align, outs):
    offsets, counts, row_of, row_token, row_scale = outs
    n, k = idx.numel(), idx.shape[-1]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.pm_moe_plan_noalloc(_ptr(idx), _ptr(lut), _ptr(w), n, k, num_slots, cap, align, _ptr(offsets),
                                   _ptr(counts), _ptr(row_of), _ptr(row_token), _ptr(row_scale), stream)


@pytest.mark.parametrize("use_lut", [False, True])
def test_noalloc_plan_matches_allocating_entry_point(use_lut):
    from placemoe_b200.ops import kernels

    lib = _lib()
    dev = "cuda"
    # caller-owned output buffers, sized once for the larger of the two calls
    t_max, k, slots, align = 5000, 8, 64, 128
    cap = t_max * k + slots * align
    outs = (torch.empty(slots + 1, dtype=torch.int32, device=dev), torch.empty(slots, dtype=torch.int32, device=dev),
            torch.empty(t_max * k, dtype=torch.int32, device=dev), torch.empty(cap, dtype=torch.int32, device=dev),
            torch.empty(cap, dtype=torch.float32, device=dev))
    g = torch.Generator(device=dev).manual_seed(11)
    for call, t in enumerate((5000, 1234)):  # two calls in a row; the second reuses the scratch of the first
        idx = torch.randint(0, slots, (t, k), device=dev, dtype=torch.int32, generator=g)
        lut = torch.randperm(slots, device=dev, generator=g).to(torch.int32) if use_lut else None
        w = torch.rand(t, k, device=dev, generator=g)
        rc = _call(lib, idx, lut, w, slots, cap, align, outs)
        assert rc == 0, lib.pm_moe_plan_noalloc_error()
        ref = kernels().moe_plan(idx, lut, w, slots, cap, align)
        torch.cuda.synchronize()
        offsets, counts, row_of, row_token, row_scale = outs
        end = int(ref[0][-1])
        assert torch.equal(offsets, ref[0]), f"call {call}: offsets"
        assert torch.equal(counts, ref[1]), f"call {call}: counts"
        assert torch.equal(row_of[: t * k], ref[2]), f"call {call}: row_of"
        assert torch.equal(row_token[:end], ref[3][:end]), f"call {call}: row_token"
        assert torch.equal(row_scale[:end], ref[4][:end]), f"call {call}: row_scale"


def test_noalloc_rejects_requests_beyond_scratch():
    lib = _lib()
    limit = lib.pm_moe_plan_noalloc_scratch_ints()
    slots = 1024
    n = (limit // slots + 1) * 2048  # one block more than the scratch holds
    dummy = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.pm_moe_plan_noalloc(_ptr(dummy), None, None, n, 1, slots, 16, 128, _ptr(dummy), _ptr(dummy),
                                 _ptr(dummy), _ptr(dummy), _ptr(dummy), ctypes.c_void_p(0))
    assert rc == 2
    assert b"scratch" in lib.pm_moe_plan_noalloc_error()


def test_noalloc_rejects_too_small_capacity():
    """The padded plan can end at n + num_slots * (align - 1) rows: a smaller capacity is refused before
    any launch, and the caller's buffers stay untouched."""
    lib = _lib()
    t, k, slots, align = 300, 4, 16, 128
    n = t * k
    cap = n + slots * (align - 1) - 1
    idx = torch.randint(0, slots, (t, k), device="cuda", dtype=torch.int32)
    outs = (torch.full((slots + 1,), -7, dtype=torch.int32, device="cuda"),
            torch.full((slots,), -7, dtype=torch.int32, device="cuda"),
            torch.full((n,), -7, dtype=torch.int32, device="cuda"),
            torch.full((cap,), -7, dtype=torch.int32, device="cuda"),
            torch.full((cap,), -7.0, dtype=torch.float32, device="cuda"))
    rc = _call(lib, idx, None, None, slots, cap, align, outs)
    torch.cuda.synchronize()
    assert rc == 1
    assert b"capacity" in lib.pm_moe_plan_noalloc_error()
    assert all(bool((o == -7).all()) for o in outs)
