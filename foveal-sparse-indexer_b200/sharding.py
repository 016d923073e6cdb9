"""Multi-GPU execution of the token-routed forward (one process per GPU, ``torch.distributed``).

Two layouts, chosen by the caller:

* **Parameter-block sharding** (large shapes, e.g. the 70B MLP): every rank holds x and all router
  parameters, runs the same deterministic router for all tokens, and computes the contraction only
  over the blocks it owns (block b belongs to rank ``b % world``, so the always-on base blocks are
  spread over ranks).  The fp32 partial outputs are summed with a collective (all-reduce, or
  reduce-scatter over token rows).  The additive stream is added once, by rank 0.  This is the only
  exchange step of the path.  With ``chunks > 1`` the tokens are processed in chunks and the collective
  of chunk i runs (NCCL, on its own stream) while chunk i+1 is computed.
* **Token splitting** (small shapes / throughput runs): each rank processes its own tokens with
  replicated weights.  Tokens are independent, so there is no collective at all.
"""

from __future__ import annotations

import contextlib
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


def _cuda_partial(module, x2d, world: int, rank: int, additive: bool, want_routes: bool, out=None):
    kg, ku, v, packed, wq, k16, wout = module._weights()
    return kernels.token_forward(
        x2d, kg, ku, v, packed, wq, k16, wout, base_blocks=module.base_blocks, top_p=module.top_p,
        min_remote=module.min_remote_blocks, max_remote=module.max_remote_blocks,
        temperature=module.temperature, additive=additive, block_stride=world, block_offset=rank,
        out_f32=True, want_routes=want_routes, y=out)


def _comm_stream(module, device) -> torch.cuda.Stream:
    st = getattr(module, "_comm_stream_obj", None)
    if st is None or st.device != device:
        st = torch.cuda.Stream(device=device)
        module._comm_stream_obj = st
    return st


def sharded_token_forward(module, x2d: torch.Tensor, *, want_routes: bool = False, reduce: str = "all",
                          compute_partial: Optional[Callable] = None, chunks: int = 1):
    """Parameter-block-sharded forward.  Returns (y, remote_indices, remote_counts, scores); with
    ``reduce="scatter"`` y holds only this rank's contiguous slice of token rows.

    ``chunks > 1`` overlaps the collective with compute: chunk i's partial is reduced on a side stream
    while chunk i+1 is computed.  For ``reduce="scatter"`` chunk i gathers, for every rank r, the i-th
    piece of r's output slice, so that each rank's result stays one contiguous slice; this needs the
    token count to divide by ``world * chunks``.  Routes are returned only without chunking."""
    rank, world, group = module._shard
    fn = compute_partial or _cuda_partial
    if reduce not in ("all", "scatter"):
        raise ValueError("reduce must be 'all' or 'scatter'")
    M, D = x2d.shape
    if reduce == "scatter" and M % world:
        raise ValueError("reduce='scatter' needs the token count to divide by the world size")
    if chunks <= 1 or want_routes:
        y_part, ridx, cnt, S = fn(module, x2d, world, rank, rank == 0, want_routes)
        if reduce == "all":
            dist.all_reduce(y_part, op=dist.ReduceOp.SUM, group=group)
            y = y_part
        else:
            y = torch.empty(M // world, D, dtype=y_part.dtype, device=y_part.device)
            dist.reduce_scatter_tensor(y, y_part, op=dist.ReduceOp.SUM, group=group)
        return y.to(x2d.dtype), ridx, cnt, S

    if reduce == "scatter" and M % (world * chunks):
        raise ValueError("chunked reduce='scatter' needs the token count to divide by world * chunks")
    # CUDA: each chunk's collective is issued from a side stream that waits for that chunk's compute, so
    # NCCL reduces chunk i while the compute stream runs chunk i+1 (host tensors: plain sequence)
    cuda = x2d.is_cuda
    cur = torch.cuda.current_stream(x2d.device) if cuda else None
    comm = _comm_stream(module, x2d.device) if cuda else None
    if cuda:
        comm.wait_stream(cur)

    def after_compute():
        if not cuda:
            return contextlib.nullcontext()
        ev = torch.cuda.Event()
        ev.record(cur)
        comm.wait_event(ev)
        return torch.cuda.stream(comm)

    works = []
    if reduce == "all":
        y = torch.empty(M, D, dtype=torch.float32, device=x2d.device)
        bounds = [M * i // chunks for i in range(chunks + 1)]
        for i in range(chunks):
            lo, hi = bounds[i], bounds[i + 1]
            if fn is _cuda_partial:  # the kernel writes its partial straight into the output rows
                part = fn(module, x2d[lo:hi], world, rank, rank == 0, False, out=y[lo:hi])[0]
            else:
                part = fn(module, x2d[lo:hi], world, rank, rank == 0, False)[0]
                y[lo:hi].copy_(part)
                part = y[lo:hi]
            with after_compute():
                works.append(dist.all_reduce(part, op=dist.ReduceOp.SUM, group=group, async_op=True))
        for w in works:
            w.wait()
        return y.to(x2d.dtype), None, None, None

    s = M // (world * chunks)  # rows of one rank's piece of one chunk
    xv = x2d.view(world, chunks, s, D)
    y = torch.empty(M // world, D, dtype=torch.float32, device=x2d.device)
    for i in range(chunks):
        xc = xv[:, i].reshape(world * s, D)  # rank-major: piece i of every rank's slice
        part, _, _, _ = fn(module, xc, world, rank, rank == 0, False)
        with after_compute():
            out = y[i * s:(i + 1) * s]
            works.append(dist.reduce_scatter_tensor(out, part, op=dist.ReduceOp.SUM, group=group, async_op=True))
    for w in works:
        w.wait()
    return y.to(x2d.dtype), None, None, None


def split_tokens(x2d: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Token-split layout: this rank's contiguous share of the token rows (ranks < M % world get one more)."""
    M = x2d.shape[0]
    base, extra = divmod(M, world)
    start = rank * base + min(rank, extra)
    return x2d[start:start + base + (1 if rank < extra else 0)]
