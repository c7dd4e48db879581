"""Host-resident layer inputs streamed through the attention kernel.

For callers whose q/k/v live in (pinned) host memory -- activation offload
for very long videos, or a host-side orchestrator feeding the GPU layer by
layer -- ``attention_from_host`` overlaps the three stages of consecutive
layers: the host-to-device copy of layer i+1 on one stream, the attention of
layer i on the caller's stream, the device-to-host copy of layer i-1 on a
third stream.  Two device slots for inputs and for outputs are double
buffered with CUDA events, so a copy never overwrites data a kernel still
reads.  With PCIe copies shorter than the kernel (cfg2: 1.16 GB in per
layer ~ 21 ms at ~55 GB/s against ~34 ms of attention) the host-to-host time
per layer approaches the kernel time.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch

from .block_sparse import block_sparse_attention


def attention_from_host(inputs: Sequence[Sequence[Optional[torch.Tensor]]], mask,
                        outputs: Sequence[Sequence[Optional[torch.Tensor]]], device: torch.device,
                        layer_fn: Optional[Callable] = None) -> None:
    """inputs[i] = (q, k, v, text_q, text_k, text_v) pinned host tensors of
    layer i (text entries None without text); outputs[i] = (out, text_out)
    pinned host tensors the results are copied into.  Runs asynchronously on
    the current stream of ``device`` (plus two copy streams); synchronize
    that stream (or the device) before reading ``outputs``.

    ``layer_fn(q, k, v, text_q, text_k, text_v) -> (out, text_out)``
    replaces the single-GPU kernel call, e.g. a Ulysses layer over this
    rank's token shard (its collectives run on the compute stream's order;
    the copies of the neighbouring layers overlap them)."""
    n = len(inputs)
    if len(outputs) != n:
        raise ValueError("one output pair per input layer")
    compute = torch.cuda.current_stream(device)
    s_in = torch.cuda.Stream(device)
    s_out = torch.cuda.Stream(device)
    slots_in: List[Optional[List[Optional[torch.Tensor]]]] = [None, None]
    slots_out: List[Optional[Tuple[torch.Tensor, Optional[torch.Tensor]]]] = [None, None]
    in_ready = [torch.cuda.Event() for _ in range(n)]
    consumed = [torch.cuda.Event() for _ in range(n)]   # kernel i finished reading slot i % 2
    copied_out = [torch.cuda.Event() for _ in range(n)]  # out slot i % 2 is on the host again

    def stage_in(i: int) -> None:
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(consumed[i - 2])
            src = inputs[i]
            slot = slots_in[i & 1]
            if slot is None or any((a is None) != (b is None) or (a is not None and a.shape != b.shape)
                                   for a, b in zip(slot, src)):
                slot = [None if x is None else torch.empty(x.shape, dtype=x.dtype, device=device) for x in src]
                slots_in[i & 1] = slot
            for d, h in zip(slot, src):
                if h is not None:
                    d.copy_(h, non_blocking=True)
            in_ready[i].record(s_in)

    stage_in(0)
    for i in range(n):
        if i + 1 < n:
            stage_in(i + 1)
        compute.wait_event(in_ready[i])
        d = slots_in[i & 1]
        if i >= 2:
            compute.wait_event(copied_out[i - 2])  # out slot free
        o_slot = slots_out[i & 1]
        if layer_fn is not None:
            o, to = layer_fn(*d)
        else:
            o, to = block_sparse_attention(d[0], d[1], d[2], mask, d[3], d[4], d[5],
                                           out=None if o_slot is None else o_slot[0],
                                           text_out=None if o_slot is None else o_slot[1])
        slots_out[i & 1] = (o, to)
        consumed[i].record(compute)
        with torch.cuda.stream(s_out):
            s_out.wait_event(consumed[i])
            outputs[i][0].copy_(o, non_blocking=True)
            if to is not None and outputs[i][1] is not None:
                outputs[i][1].copy_(to, non_blocking=True)
            copied_out[i].record(s_out)
        # Device memory used on streams other than its allocation stream: keep
        # the caching allocator from reusing it before those uses finish.
        for x in d:
            if x is not None:
                x.record_stream(compute)
        o.record_stream(s_out)
        if to is not None:
            to.record_stream(s_out)
    # The caller's stream completes only after every output is on the host.
    for i in range(max(0, n - 2), n):
        compute.wait_event(copied_out[i])
