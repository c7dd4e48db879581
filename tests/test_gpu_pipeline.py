"""attention_from_host (copies overlapped with the kernel on separate
streams) returns exactly what per-layer device calls return."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_pipeline_matches_direct_calls():
    from longvideosparseattention_b200 import block_sparse_attention, build_block_mask
    from longvideosparseattention_b200.pipeline import attention_from_host
    dev = torch.device("cuda")
    T, P, H, D, nt, L = 9, 300, 4, 128, 50, 5
    g = torch.Generator().manual_seed(2)
    mk = lambda n: (torch.randn(1, n, H, D, generator=g) / D ** 0.25).bfloat16().pin_memory()
    layers = [(mk(T * P), mk(T * P), mk(T * P), mk(nt), mk(nt), mk(nt)) for _ in range(L)]
    outs = [(torch.empty(1, T * P, H, D, dtype=torch.bfloat16).pin_memory(),
             torch.empty(1, nt, H, D, dtype=torch.bfloat16).pin_memory()) for _ in range(L)]
    mask = build_block_mask(T, P, 1, 1, 4, 2, True, nt, device=dev)
    attention_from_host(layers, mask, outs, dev)
    torch.cuda.current_stream(dev).synchronize()
    for lay, (o, to) in zip(layers, outs):
        want, twant = block_sparse_attention(*[x.to(dev) for x in lay[:3]], mask, *[x.to(dev) for x in lay[3:]])
        assert torch.equal(o, want.cpu()) and torch.equal(to, twant.cpu())
