"""A denoising step (GPU mask rebuild for the step's keyframe offset + attention
layers) captured once in a CUDA graph and replayed: identical to eager."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_graph_capture_of_a_step_matches_eager():
    from longvideosparseattention_b200 import block_sparse_attention, build_block_mask
    T, P, H, D, W, kfi, nt = 9, 160, 2, 128, 1, 4, 40
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    mk = lambda n: (torch.randn(1, n, H, D, generator=g, device=dev) / D ** 0.25).to(torch.bfloat16)
    layers = [(mk(T * P), mk(T * P), mk(T * P)) for _ in range(3)]
    tq, tk, tv = mk(nt), mk(nt), mk(nt)
    mask = build_block_mask(T, P, W, 1, kfi, 0, True, nt, device=dev)
    outs = [torch.empty_like(layers[0][0]) for _ in layers]
    touts = [torch.empty_like(tq) for _ in layers]
    offset = {"v": 1}

    def step():
        build_block_mask(T, P, W, 1, kfi, offset["v"], True, nt, device=dev, reuse=mask)
        for (q, k, v), o, to in zip(layers, outs, touts):
            block_sparse_attention(q, k, v, mask, tq, tk, tv, out=o, text_out=to)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()  # warm-up outside capture (function attributes, allocator)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    eager = [o.clone() for o in outs]
    for o in outs:
        o.zero_()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(outs, eager):
        assert torch.equal(a, b)
