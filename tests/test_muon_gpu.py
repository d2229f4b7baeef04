"""Muon's Newton-Schulz orthogonalisation on the tcgen05 GEMMs against the fp32 PyTorch iteration."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(256, 512), (1024, 256), (3, 128, 384)])
def test_newton_schulz_cuda_matches_fp32(shape):
    from placemoe_b200.ops import check_device_error
    from placemoe_b200.optim.muon import zeropower_newton_schulz

    g = torch.randn(*shape, generator=torch.Generator().manual_seed(1))
    ref = zeropower_newton_schulz(g, steps=5)  # CPU: fp32 iteration
    got = zeropower_newton_schulz(g.cuda(), steps=5).float().cpu()
    torch.cuda.synchronize()
    check_device_error()
    assert got.shape == ref.shape
    err = ((got - ref).abs().max() / ref.abs().max()).item()
    assert err < 5e-2, err  # bf16 operands over 15 chained products
