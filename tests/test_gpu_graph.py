"""Runs captured in CUDA graphs (``PreparedFFN.capture_graph``), beyond the reference.

The launch epoch the kernel's counters and flags are compared against lives on the device
(a launch count every CTA bumps), so a captured launch replays correctly any number of
times and interleaves with eager runs.  Every kernel family replays against its eager
results, bit for bit: prefill tiles (static and claimed tile orders, Stream-K), CTA pairs,
row blocks, decode tiles with bf16 and fp8 weights, SwiGLU, and overlapped launches.
"""
import pytest
import torch

from ffn_optim_b200 import prepare_ffn

pytestmark = pytest.mark.gpu

VARIANTS = [  # (M, K, H, N, options)
    (512, 512, 2048, 512, {}),
    (512, 512, 2048, 512, {"schedule": "dynamic"}),
    (700, 256, 1000, 300, {"down_impl": "streamk"}),
    (1024, 512, 2048, 512, {"tile": "pair256x256"}),
    (512, 256, 1024, 256, {"down_impl": "full_load_a"}),
    (16, 1024, 4096, 1024, {"down_impl": "streamk"}),
    (16, 1024, 4096, 1024, {"down_impl": "streamk", "weight_format": "fp8"}),
    (16, 1024, 4096, 1024, {"activation": "swiglu"}),
    (16, 1024, 4096, 1024, {"down_impl": "streamk", "overlap": True}),
]


@pytest.mark.parametrize("m,k,h,n,opts", VARIANTS, ids=lambda v: str(v))
def test_graph_replays_match_eager(m, k, h, n, opts):
    opts = dict(opts)
    overlap = opts.pop("overlap", False)
    g = torch.Generator().manual_seed(m + h + n)
    xs = [torch.randn(m, k, generator=g).to(torch.bfloat16).cuda() for _ in range(3)]
    rows = 2 * h if opts.get("activation") == "swiglu" else h
    w1 = (torch.randn(rows, k, generator=g) * k ** -0.5).to(torch.bfloat16).cuda()
    w2 = (torch.randn(n, h, generator=g) * h ** -0.5).to(torch.bfloat16).cuda()
    p = prepare_ffn(xs[0], w1, w2, **opts)
    p.set_wait_limit(2.0)
    if overlap:
        p.set_launch_overlap(True)
    ref = [p.run(x).clone() for x in xs]
    graph = p.capture_graph(runs=2)
    for i in range(12):
        p.load_input(xs[i % 3])
        graph.replay()
        assert torch.equal(p.run().clone() if i % 4 == 3 else p._output_view().clone(), ref[i % 3])
    p.check()
    assert torch.equal(p.run(xs[1]), ref[1])
    p.check()
    del graph
    p.close()
