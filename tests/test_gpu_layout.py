"""Canonical weight layout (``layout='canonical'``: W1 [K, H], W2 [H, N], Y = GELU(X W1) W2),
beyond the reference's V1, which rejects it.  Canonical weights are the Linear weights
stored transposed; ``prepare_ffn`` copies them once into Linear storage, so every kernel
family must give exactly the Linear result."""
import pytest
import torch

from ffn_optim_b200 import prepare_ffn

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,k,h,n,opts", [
    (300, 136, 520, 200, {}), (700, 256, 1000, 300, {"down_impl": "streamk"}),
    (512, 256, 1024, 256, {"down_impl": "full_load_a"}), (16, 1024, 4096, 1024, {"down_impl": "streamk"}),
    (16, 1024, 4096, 1024, {"weight_format": "fp8"}), (64, 512, 1024, 512, {"activation": "silu"}),
], ids=str)
def test_canonical_equals_linear(m, k, h, n, opts):
    g = torch.Generator().manual_seed(m + k)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    w1 = (torch.randn(h, k, generator=g) * k ** -0.5).to(torch.bfloat16).cuda()
    w2 = (torch.randn(n, h, generator=g) * h ** -0.5).to(torch.bfloat16).cuda()
    lin = prepare_ffn(x, w1, w2, **opts)
    y_lin = lin.run().clone()
    lin.check()
    can = prepare_ffn(x, w1.t().contiguous(), w2.t().contiguous(), layout="canonical", **opts)
    y_can = can.run()
    can.check()
    assert torch.equal(y_can, y_lin)
    with pytest.raises(ValueError):  # shapes are checked as the Linear views
        prepare_ffn(x, w1, w2.t().contiguous(), layout="canonical", **opts)
