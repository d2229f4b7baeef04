"""The bounds-checked debug build (``-DPLACEMOE_DEBUG_BOUNDS``): an index read from data that is out of
range records error 3 and the access is skipped.

Every bad index below still points inside the allocation that backs the tensor (the tensors are views of
larger buffers), so even a build without the checks would read valid memory: the tests cannot fault.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _dbg():
    from placemoe_b200 import _build

    try:
        mod = _build.load_debug_kernels()
    except ImportError:
        pytest.skip("bounds-checked debug build not present")
    assert mod.debug_bounds() is True
    return mod


def test_normal_build_has_no_index_checks():
    from placemoe_b200.ops import kernels

    assert kernels().debug_bounds() is False


def test_gather_rows_skips_and_records_bad_index():
    dbg = _dbg()
    dbg.device_error(True)
    backing = torch.randn(128, 256, device="cuda").to(torch.bfloat16)
    src = backing[:64]  # 64 rows; the bad index 71 below stays inside the 128-row allocation
    row_token = torch.tensor([0, 5, 71, 3], dtype=torch.int32, device="cuda")
    out = torch.full((4, 256), 7.0, device="cuda", dtype=torch.bfloat16)
    dbg.gather_rows(src, row_token, None, out)
    torch.cuda.synchronize()
    assert dbg.device_error(True) == 3
    assert torch.equal(out[0], src[0]) and torch.equal(out[1], src[5]) and torch.equal(out[3], src[3])
    assert bool((out[2] == 0).all())  # the bad row is skipped (written as a padding row)
    assert dbg.device_error(True) == 0  # cleared by the read


def test_fused_dispatch_rejects_bad_expert_id():
    """One-rank EP dispatch in the debug build with an expert id beyond the mapping tables: the
    assignment is dropped (position -1), the status block records a bounds error, the rest is placed."""
    from placemoe_b200.ops import p2p_status

    dbg = _dbg()
    dev = torch.device("cuda", torch.cuda.current_device())
    st = p2p_status(dev)
    st.zero_()
    e, k, t, h, slots = 8, 2, 16, 256, 8
    tab_backing = torch.zeros(2 * e, dtype=torch.int32, device=dev)  # ids up to 2e - 1 stay inside it
    dest_tab = tab_backing[:e]
    slot_backing = torch.arange(2 * e, dtype=torch.int32, device=dev) % slots
    slot_tab = slot_backing[:e]
    idx = torch.randint(0, e, (t, k), dtype=torch.int32, device=dev)
    idx[3, 1] = e + 3  # out of range
    x = torch.randn(t, h, device=dev).to(torch.bfloat16)
    w = torch.rand(t, k, device=dev)
    align, kpad = 128, 4
    cap = ((t * k + slots * (align - 1)) + align - 1) // align * align
    off_x = 1 << 16
    off_meta = off_x + cap * h * 2
    off_tab = off_meta + cap * 16
    off_back = off_tab + cap * kpad * 4
    off_dw = off_back + t * h * 2
    off_dy = off_dw + t * k * 4 + 256
    off_prim = off_dy + cap * h * 2
    total = off_prim + (cap + 1) * 4 + 16
    arena = torch.zeros(total, dtype=torch.uint8, device=dev)
    peers = torch.tensor([arena.data_ptr()], dtype=torch.int64, device=dev)
    geo = [1, 0, slots, k, h, t, cap, align, kpad, 0, 0, 256, off_x, off_meta, off_tab, off_back, off_dw, off_dy,
           off_prim]
    scratch = torch.zeros(int(dbg.ep_scratch_ints(1, slots)), dtype=torch.int32, device=dev)
    pos = torch.empty(t, k, dtype=torch.int32, device=dev)
    dst = torch.empty(t, k, dtype=torch.int32, device=dev)
    offsets = torch.empty(slots + 1, dtype=torch.int32, device=dev)
    row_scale = torch.empty(cap, dtype=torch.float32, device=dev)
    dbg.ep_dispatch(x, idx, w, dest_tab, slot_tab, peers, geo, scratch, st, 1, 2.0, pos, dst, offsets, row_scale)
    torch.cuda.synchronize()
    code, where = st.tolist()[:2]
    assert code == 3 and where == 7
    assert pos[3, 1].item() == -1
    valid = torch.ones_like(pos, dtype=torch.bool)
    valid[3, 1] = False
    assert bool((pos[valid] >= 0).all())
    st.zero_()
