"""Failure detection without a GPU fault: every wait in the attention
kernels is bounded.  A test hook makes one CTA skip its query-tile load, so
the waits on it can never complete; with a 50 ms limit the kernel must
return on its own, record LVSA_ERR_DEVICE_TIMEOUT in the device error word
(read by the host through check_device_errors), leave the other CTAs'
rows correct, and leave the context usable: the next normal launch on the
same device is correct and reports no error."""

import pytest
import torch

from oracle import lvsa_oracle as O
from tests.gpu_util import assert_close, seeded, to_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("D,fp8,kernel", [(128, False, "pair"), (128, False, "single"), (64, False, "auto"),
                                          (128, True, "auto")])
def test_expired_wait_reports_timeout_and_context_survives(D, fp8, kernel, monkeypatch):
    monkeypatch.setenv("LVSA_ATTN_KERNEL", kernel)
    from longvideosparseattention_b200 import _native as N
    from longvideosparseattention_b200 import block_sparse_attention, build_block_mask, check_device_errors
    dev = torch.device("cuda")
    T, P, H, W, kfi, off = 6, 128, 2, 1, 3, 0
    m = build_block_mask(T, P, W, 1, kfi, off, True, 0, device=dev)
    q, k = seeded((1, T * P, H, D), 1, scale=D ** -0.5), seeded((1, T * P, H, D), 2, scale=D ** -0.5)
    v = seeded((1, T * P, H, D), 3)
    check_device_errors(dev)                     # start clean
    out = torch.full_like(q, 5.0)
    block_sparse_attention(q, k, v, m, out=out, fp8=fp8, wait_timeout_us=50_000, inject_fault=1)
    torch.cuda.synchronize()                     # returns: the waits are bounded
    with pytest.raises(N.LvsaError) as e:
        check_device_errors(dev)
    assert e.value.status == N.LVSA_ERR_DEVICE_TIMEOUT
    # The stalled CTA (head 0, first query tile(s)) wrote nothing; the rest ran.
    assert (out[0, :P, 0] == 5.0).all()
    fp = O.frame_pattern(T, P, W, 1, kfi, off)
    want, _ = O.attention(to_np(q), to_np(k), to_np(v), fp)
    tol = dict(max_abs=6e-2, mean_abs=6e-3) if fp8 else {}
    assert_close(to_np(out)[:, :, 1], want[:, :, 1], what="other head", **tol)
    # Same device, normal launch: correct, no error.
    out2, _ = block_sparse_attention(q, k, v, m, fp8=fp8)
    torch.cuda.synchronize()
    check_device_errors(dev)
    assert_close(to_np(out2), want, what="after the timeout", **tol)
