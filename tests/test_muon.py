"""Muon Newton-Schulz orthogonalisation: oracle pinned to the reference's output (CPU)
and the tensor-core bf16 kernel against it (GPU)."""

import pytest
import torch

from oracle import muon_oracle


@pytest.fixture(scope="module")
def muon_golden():
    import os
    return torch.load(os.path.join(os.path.dirname(__file__), "golden", "muon_golden.pt"))


def test_oracle_reproduces_reference_newton_schulz(muon_golden):
    for name, c in muon_golden["cases"].items():
        out = muon_oracle.newton_schulz(c["update"], muon_golden["coeffs"], muon_golden["steps"], muon_golden["eps"],
                                        muon_golden["polish"], c["polish_steps"])
        assert out.dtype == torch.bfloat16 and out.shape == c["out"].shape
        assert torch.equal(out, c["out"]), name


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["wide", "tall", "small", "square_polish"])
def test_gpu_newton_schulz_matches_reference(muon_golden, cuda_device, case):
    """bf16 products accumulate in fp32 in a different order than the reference's CPU
    bmm, so results may differ by bf16 rounding of intermediate products: the kernel must
    stay within twice the deviation of torch's own CUDA bf16 path from the same golden
    output, and within 2% of the float64 iteration's magnitude."""
    from flashcart_b200 import ops  # noqa: F401

    c = muon_golden["cases"][case]
    u = c["update"].to(cuda_device)
    ours = torch.ops.flashcart.newton_schulz(u, list(muon_golden["coeffs"]), muon_golden["steps"],
                                             list(muon_golden["polish"]), c["polish_steps"], muon_golden["eps"])
    ref = c["out"].float()
    torch_cuda = muon_oracle.newton_schulz(u, muon_golden["coeffs"], muon_golden["steps"], muon_golden["eps"],
                                           muon_golden["polish"], c["polish_steps"]).float().cpu()
    exact = muon_oracle.newton_schulz(c["update"], muon_golden["coeffs"], muon_golden["steps"], muon_golden["eps"],
                                      muon_golden["polish"], c["polish_steps"], dtype=torch.float64)
    err = (ours.float().cpu() - ref).abs().max().item()
    base = (torch_cuda - ref).abs().max().item()
    scale = exact.abs().max().item()
    assert ours.dtype == torch.bfloat16 and ours.shape == c["out"].shape
    assert err <= max(2 * base, 0.02 * scale), (err, base, scale)
    # the result is (close to) orthogonal like the reference's
    assert (ours.float().cpu() - exact.float()).abs().max().item() <= 0.1 * scale
    from flashcart_b200.ops import check_device_status
    check_device_status(cuda_device)


@pytest.mark.gpu
def test_gpu_newton_schulz_rejects_unaligned_shapes(cuda_device):
    from flashcart_b200 import ops  # noqa: F401

    with pytest.raises(NotImplementedError, match="multiples of 8"):
        torch.ops.flashcart.newton_schulz(torch.randn(1, 12, 64, device=cuda_device), [3.4445, -4.775, 2.0315], 5,
                                          [2.0, -1.5, 0.5], 0, 1e-7)
