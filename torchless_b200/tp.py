"""Tensor-parallel set-up over torch.distributed (one process per GPU).

Each rank loads its slice of the model (``Model.from_buffer(..., tp_size,
tp_rank)``), then ``connect`` gathers every rank's exchange-buffer handle in
rank order and maps the peers' buffers, so that the decode kernel can sum
o_proj / down_proj partials over NVLink.  torch.distributed is used only to
move the 64-byte handles and for host barriers; the decode data path has no
collective library in it.
"""
from __future__ import annotations

from typing import List


def gather_handles(handle: bytes, group=None) -> List[bytes]:
    """All ranks' handles in rank order (any torch.distributed backend)."""
    import torch.distributed as dist
    out: List[bytes] = [b""] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return out


def connect(model, group=None) -> None:
    """Exchange handles and map the peers; ends with a barrier so that no rank
    launches a step before every rank has mapped every buffer."""
    import torch.distributed as dist
    model.tp_connect(gather_handles(model.tp_handle(), group))
    dist.barrier(group)


def connect_batch(batch, group=None) -> None:
    """Same for a tensor-parallel Batch (tl_batch_*): its own exchange buffers
    carry the residual and argmax exchanges of batched decoding."""
    import torch.distributed as dist
    batch.tp_connect(gather_handles(batch.tp_handle(), group))
    dist.barrier(group)
