"""Expert parallelism of the MoE block, one process per GPU (rbt_moe_ep_*).

GPU g of N owns experts [g*E/N, (g+1)*E/N) of every layer and the whole router.
The library runs the whole layer on each GPU -- routing, the push of every token's
row into the GPUs that own its experts (stores to peer memory over NVLink), the
experts, the return of the partial rows and the combine in GPU order -- with no
host synchronisation (include/rbt_moe.h).  What a process-per-GPU group needs
from the host is the connection: every rank's IPC handle of its receive/return
block, gathered in rank order.  `connect` does that over a torch.distributed
process group of the caller's (gloo suffices: the handles are 64 bytes each, and
no collective runs on the data path).  A rank that fails or never arrives makes
the gather fail after the group's timeout, which is reported as an RbtMoeError
instead of a hang.
"""
from __future__ import annotations

import torch.distributed as dist

from . import moe


def connect(ctx: "moe.MoeContext", group=None) -> None:
    """Gather every rank's handle (rank order) and connect this rank's context.
    The context must have been ep_init'ed as this process's rank of the group."""
    world = dist.get_world_size(group)
    handles = [None] * world
    try:
        dist.all_gather_object(handles, ctx.ep_handle(), group=group)
    except Exception as exc:  # a rank that raised, exited or never joined
        raise moe.RbtMoeError(f"expert parallelism: gathering the {world} ranks' handles failed: {exc}") from exc
    bad = [r for r, h in enumerate(handles) if not isinstance(h, (bytes, bytearray)) or len(h) != 64]
    if bad:
        raise moe.RbtMoeError(f"expert parallelism: ranks {bad} sent no valid handle")
    ctx.ep_connect(handles)
