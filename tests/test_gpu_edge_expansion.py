"""Config 2 at test size: edge expansion followed by the equivariant linear map.

The reference composition (Survey configuration 2; ``o3/irreps.py``, ``nn/radial.py``,
``nn/layers.py:84-131``, ``o3/linear.py``): moments T^l(r^), l <= 3, of edge vectors uniform
in a 5 A ball, times h = Linear(8 -> 128)(Bessel(8, r_max 5)(r) * cutoff(r)), laid out as
(E, sum_l (2l+1) 128) = (E, 2048), then o3.LinearLayer(3, 3, 128, 128) with Xavier-normal
weights and weight_scale 1. fp32 on the GPU (3xTF32 linear maps) against the float64
oracle, and the single-TF32 path against the reference's TF32 tolerance.
"""

import math

import pytest
import torch

from oracle import stf_oracle as O

pytestmark = pytest.mark.gpu


def _vectors(n, seed=0):
    g = torch.Generator().manual_seed(seed)
    d = torch.randn(n, 3, generator=g, dtype=torch.float64)
    d = d / d.norm(dim=-1, keepdim=True)
    r = 5.0 * torch.rand(n, generator=g, dtype=torch.float64) ** (1.0 / 3.0)
    v = d * r.unsqueeze(-1)
    return v[v.norm(dim=-1) >= 1e-4]


def _expand(T, h, C=128):
    blocks, off = [], 0
    for l in range(4):
        n = 2 * l + 1
        blocks.append((T[:, off:off + n].unsqueeze(-1) * h.unsqueeze(1)).reshape(T.shape[0], n * C))
        off += n
    return torch.cat(blocks, dim=-1)


def _oracle(v, w_h, scale_h, ws):
    r = v.norm(dim=-1)
    T = O.irreps(v / r.unsqueeze(-1), 3)
    k = (math.pi / 5.0) * torch.arange(1, 9, dtype=torch.float64)
    basis = math.sqrt(2.0 / 5.0) * k * torch.sinc(r.unsqueeze(-1) * k / math.pi)
    t = r / 5.0
    env = torch.clamp((1 - 28 * t ** 6 + 48 * t ** 7 - 21 * t ** 8) * (r < 5.0), 0, 1)
    h = (basis * env.unsqueeze(-1)) @ (w_h.t() * scale_h)
    return O.linear(_expand(T, h), ws, 3, 3, 128, 128, scales=[1.0] * 4)


def _ours(v, lay, lin):
    from flashcart_b200 import o3
    from flashcart_b200.nn.radial import BesselBasis, PolynomialCutoff

    dev = v.device
    r = v.norm(dim=-1)
    T = o3.Irreps(3).forward_normalized(v / r.unsqueeze(-1))
    h = lay(BesselBasis(8, 5.0).to(dev)(r) * PolynomialCutoff(5.0, 6).to(dev)(r).unsqueeze(-1))
    return lin(_expand(T, h))


def test_gpu_edge_expansion_and_linear_match_oracle(cuda_device):
    from flashcart_b200 import o3
    from flashcart_b200.nn.layers import LinearLayer

    torch.manual_seed(0)
    v64 = _vectors(20000)
    lay = LinearLayer(8, 128).to(cuda_device)
    lin = o3.LinearLayer(3, 3, 128, 128, weight_scale=1.0).to(cuda_device)
    with torch.no_grad():
        for w in lin.weight:
            torch.nn.init.xavier_normal_(w)
    ref = _oracle(v64, lay.weight.detach().double().cpu(), float(lay.scale),
                  [w.detach().double().cpu() for w in lin.weight])
    out = _ours(v64.float().to(cuda_device), lay, lin)
    err = (out.double().cpu() - ref).abs().max().item()
    assert err <= 2e-5 * ref.abs().max().item(), err
    # single-TF32 products: the reference's TF32 tolerance (tests/o3/test_linear.py:37)
    prev = (torch.backends.cuda.matmul.allow_tf32, torch.get_float32_matmul_precision())
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.set_float32_matmul_precision("high")
    try:
        fast = _ours(v64.float().to(cuda_device), lay, lin)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev[0]
        torch.set_float32_matmul_precision(prev[1])
    assert torch.allclose(fast.double().cpu(), ref, atol=3e-3, rtol=2e-3)
    from flashcart_b200.ops import check_device_status
    check_device_status(cuda_device)
