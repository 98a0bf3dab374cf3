"""Overlapped launches (``PreparedFFN.set_launch_overlap``, programmatic dependent launch),
beyond the reference: results must be those of serial launches, bit for bit.

The hard case is a chain of two FFNs where the second reads the first's output buffer
directly (``ffn_b200_rebind_io``): the first kernel lets its dependents launch at its start,
so the second's CTAs set up while the first is still running and must not touch global
memory before the first has completed; the next iteration's first FFN then overwrites the
buffer the second just read.  Every kernel family runs the chain: prefill tiles (basic and
Stream-K), CTA pairs, hidden-resident row blocks, decode tiles with bf16 and fp8 weights,
SwiGLU.  A plain ``run(x)`` sequence (a torch copy kernel before each launch) is checked too.
"""
import pytest
import torch

from ffn_optim_b200 import _lib, prepare_ffn

pytestmark = pytest.mark.gpu

VARIANTS = [  # (M, K=N, H, prepare_ffn options)
    (512, 512, 2048, {}),
    (512, 512, 2048, {"down_impl": "streamk"}),
    (1024, 512, 2048, {"tile": "pair256x256"}),
    (512, 256, 1024, {"down_impl": "full_load_a"}),
    (16, 1024, 4096, {"down_impl": "streamk"}),
    (16, 1024, 4096, {"down_impl": "streamk", "weight_format": "fp8"}),
    (16, 1024, 4096, {"activation": "swiglu"}),
]


def _weights(k, h, glu, g):
    w1 = (torch.randn(2 * h if glu else h, k, generator=g) * k ** -0.5).to(torch.bfloat16).cuda()
    w2 = (torch.randn(k, h, generator=g) * h ** -0.5).to(torch.bfloat16).cuda()
    return w1, w2


@pytest.mark.parametrize("m,k,h,opts", VARIANTS, ids=lambda v: str(v))
def test_overlapped_chain_matches_serial(m, k, h, opts):
    g = torch.Generator().manual_seed(m + h)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    glu = opts.get("activation") == "swiglu"
    a = prepare_ffn(x, *_weights(k, h, glu, g), **opts)
    b = prepare_ffn(x, *_weights(k, h, glu, g), **opts)
    for p in (a, b):
        p.set_wait_limit(2.0)
    lib = _lib.load()
    # B reads A's output buffer as its X (same [M, pitch] layout: N == K) and writes its own.
    assert lib.ffn_b200_rebind_io(b.handle, a.storage[4].data_ptr(), b.storage[4].data_ptr()) == _lib.OK
    a.run()
    y_ref = b.run().clone()
    ya_ref = a.storage[4].clone()
    b.check()
    for p in (a, b):
        p.set_launch_overlap(True)
    outs = []
    for _ in range(8):
        a.run()
        outs.append(b.run().clone())
    b.check()
    a.check()
    for y in outs:
        assert torch.equal(y, y_ref)
    assert torch.equal(a.storage[4], ya_ref)
    a.close()
    b.close()


def test_overlapped_runs_with_new_inputs():
    g = torch.Generator().manual_seed(5)
    m, k, h = 300, 256, 1024
    xs = [torch.randn(m, k, generator=g).to(torch.bfloat16).cuda() for _ in range(3)]
    w1, w2 = _weights(k, h, False, g)
    p = prepare_ffn(xs[0], w1, w2, down_impl="streamk")
    ref = [p.run(x).clone() for x in xs]
    p.set_launch_overlap(True)
    got = [p.run(xs[i % 3]).clone() for i in range(9)]
    p.check()
    for i, y in enumerate(got):
        assert torch.equal(y, ref[i % 3])
    p.set_launch_overlap(False)
    assert torch.equal(p.run(xs[1]), ref[1])
    p.close()
