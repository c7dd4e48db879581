"""attention_from_host (copies overlapped with the kernel on separate
streams) returns exactly what per-layer device calls return, with the
kernel call built in or given as ``layer_fn`` (how a Ulysses rank streams
its host-resident shards)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("via_layer_fn", [False, True])
def test_pipeline_matches_direct_calls(via_layer_fn):
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
    fn = (lambda q, k, v, tq, tk, tv: block_sparse_attention(q, k, v, mask, tq, tk, tv)) if via_layer_fn else None
    attention_from_host(layers, mask, outs, dev, layer_fn=fn)
    torch.cuda.current_stream(dev).synchronize()
    for lay, (o, to) in zip(layers, outs):
        want, twant = block_sparse_attention(*[x.to(dev) for x in lay[:3]], mask, *[x.to(dev) for x in lay[3:]])
        assert torch.equal(o, want.cpu()) and torch.equal(to, twant.cpu())
