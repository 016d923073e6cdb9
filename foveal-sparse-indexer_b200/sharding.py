"""Multi-GPU execution of the token-routed forward (one process per GPU, ``torch.distributed``).

Two layouts, chosen by the caller:

* **Parameter-block sharding** (large shapes, e.g. the 70B MLP): every rank holds x and all router
  parameters, runs the same deterministic router for all tokens, and computes the contraction only
  over the blocks it owns (block b belongs to rank ``b % world``, so the always-on base blocks are
  spread over ranks).  The fp32 partial outputs are summed with one collective (all-reduce, or
  reduce-scatter over token rows).  The additive stream is added once, by rank 0.  This is the only
  exchange step of the path.
* **Token splitting** (small shapes / throughput runs): each rank processes its own tokens with
  replicated weights.  Tokens are independent, so there is no collective at all.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import kernels


def shard_parameter_blocks(module, group=None) -> None:
    """Makes ``module`` (routing="token") compute only the parameter blocks of this rank."""
    if module.routing != "token":
        raise ValueError("parameter-block sharding applies to routing='token'")
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    module._shard = (rank, world, group)


def owned_blocks(num_blocks: int, rank: int, world: int):
    """Block ids owned by ``rank``: b % world == rank."""
    return list(range(rank, num_blocks, world))


def _cuda_partial(module, x2d, world: int, rank: int, additive: bool, want_routes: bool):
    kg, ku, v, packed, wq, k16, wout = module._weights()
    return kernels.token_forward(
        x2d, kg, ku, v, packed, wq, k16, wout, base_blocks=module.base_blocks, top_p=module.top_p,
        min_remote=module.min_remote_blocks, max_remote=module.max_remote_blocks,
        temperature=module.temperature, additive=additive, block_stride=world, block_offset=rank,
        out_f32=True, want_routes=want_routes)


def sharded_token_forward(module, x2d: torch.Tensor, *, want_routes: bool = False, reduce: str = "all",
                          compute_partial: Optional[Callable] = None):
    """Parameter-block-sharded forward.  Returns (y, remote_indices, remote_counts, scores); with
    ``reduce="scatter"`` y holds only this rank's contiguous slice of token rows."""
    rank, world, group = module._shard
    fn = compute_partial or _cuda_partial
    y_part, ridx, cnt, S = fn(module, x2d, world, rank, rank == 0, want_routes)
    if reduce == "all":
        dist.all_reduce(y_part, op=dist.ReduceOp.SUM, group=group)
        y = y_part
    elif reduce == "scatter":
        M = y_part.shape[0]
        if M % world:
            raise ValueError("reduce='scatter' needs the token count to divide by the world size")
        y = torch.empty(M // world, y_part.shape[1], dtype=y_part.dtype, device=y_part.device)
        dist.reduce_scatter_tensor(y, y_part, op=dist.ReduceOp.SUM, group=group)
    else:
        raise ValueError("reduce must be 'all' or 'scatter'")
    return y.to(x2d.dtype), ridx, cnt, S


def split_tokens(x2d: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Token-split layout: this rank's contiguous share of the token rows (ranks < M % world get one more)."""
    M = x2d.shape[0]
    base, extra = divmod(M, world)
    start = rank * base + min(rank, extra)
    return x2d[start:start + base + (1 if rank < extra else 0)]
