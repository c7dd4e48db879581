"""Seeded stand-ins for the diffusers attention modules the adapters read
(only the fields the adapters touch).  Shared by the golden-vector generator
and the tests, so both build bit-identical modules."""

import torch


class MockAttn(torch.nn.Module):
    """heads, to_q/to_k/to_v, norm_q/norm_k, to_out; optional dual-stream
    add_*_proj, norm_added_*, to_add_out."""

    def __init__(self, dim: int, heads: int, norm: str, dual: bool, seed: int):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        D = dim // heads
        self.heads = heads

        def lin(i, o):
            m = torch.nn.Linear(i, o)
            with torch.no_grad():
                m.weight.copy_(torch.randn(o, i, generator=g) / i ** 0.5)
                m.bias.copy_(0.1 * torch.randn(o, generator=g))
            return m

        def nrm():
            if norm == "rms":
                m = torch.nn.RMSNorm(D, eps=1e-6)
            else:
                m = torch.nn.LayerNorm(D, eps=1e-5)
                with torch.no_grad():
                    m.bias.copy_(0.1 * torch.randn(D, generator=g))
            with torch.no_grad():
                m.weight.copy_(1 + 0.2 * torch.randn(D, generator=g))
            return m

        self.to_q, self.to_k, self.to_v = lin(dim, dim), lin(dim, dim), lin(dim, dim)
        self.norm_q, self.norm_k = nrm(), nrm()
        self.to_out = torch.nn.ModuleList([lin(dim, dim), torch.nn.Dropout(0.0)])
        if dual:
            self.add_q_proj, self.add_k_proj, self.add_v_proj = lin(dim, dim), lin(dim, dim), lin(dim, dim)
            self.norm_added_q, self.norm_added_k = nrm(), nrm()
            self.to_add_out = lin(dim, dim)


def rope_pair(S: int, D: int, seed: int):
    """(cos, sin) [1, S, 1, D] with each pair angle in both slots of the pair."""
    g = torch.Generator().manual_seed(seed)
    ang = torch.rand(S, D // 2, generator=g) * 6.0
    return (torch.cos(ang).repeat_interleave(2, -1)[None, :, None, :],
            torch.sin(ang).repeat_interleave(2, -1)[None, :, None, :])
