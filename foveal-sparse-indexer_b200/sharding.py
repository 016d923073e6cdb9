"""Multi-GPU execution of the token-routed forward (one process per GPU, ``torch.distributed``).

Layouts, chosen by the caller:

* **Parameter-block sharding** (the 8B / 70B MLP shapes): every rank computes the contraction only over
  the blocks it owns (block b belongs to rank ``b % world``, so the always-on base blocks are spread over
  ranks) for all tokens, and the partial outputs are summed by one collective (reduce-scatter over token
  rows, or all-reduce).  Partials are bf16 for a bf16 model (half the NVLink bytes of fp32).
  The routing is split over the ranks as well: each rank routes only its share of the tokens
  (``fp_route_tokens``), one all-gather of the routes (block ids and counts, 4·(K_max + 1) bytes per
  token) gives every rank all of them, and each rank's contraction runs from the given routes
  (``fp_pattention_routed_fwd``).  The additive stream of a token is added by the rank that routed it.
  With ``chunks > 1`` the tokens are processed in chunks and the reduce-scatter of chunk i (NCCL, on its
  own stream) runs while chunk i+1 is computed.  Routes are deterministic per token, so the result
  equals the single-GPU forward's (the bf16 partial sums round differently).
* **Token-partitioned input** (``sharded_forward_slices`` / ``sharded_forward_host``): each rank starts
  from its own slice of the batch; an all-gather brings every slice's rows of a chunk to every rank.
* **Token splitting**: each rank processes its own tokens with replicated weights; no collective.
"""

from __future__ import annotations

import contextlib
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import kernels


def shard_parameter_blocks(module, group=None, partial_dtype: Optional[torch.dtype] = None,
                           shard_routing: bool = True, peer_reduce: bool = False) -> None:
    """Makes ``module`` (routing="token") compute only the parameter blocks of this rank.

    ``partial_dtype``: dtype of the partial outputs that the collective sums (default: the module's
    dtype, so a bf16 model moves bf16 partials, half the bytes of fp32; the reduction of N bf16 partials
    stays well inside the 2e-2 relative bar of bf16 outputs).  ``torch.float32`` keeps fp32 partials.
    ``shard_routing``: route only this rank's share of the tokens and all-gather the routes (when the
    token count divides by the world size); False routes every token on every rank.
    ``peer_reduce``: replace the reduce-scatter of the unchunked, split-routing forward by the peer-memory
    one (the contraction stores each row's partial straight into the owning rank's receive buffer over
    NVLink; see :class:`PeerReduce`).  The buffers are set up by the first such forward, on every rank of
    the group at once; :func:`release_peer_buffers` frees them."""
    if module.routing != "token":
        raise ValueError("parameter-block sharding applies to routing='token'")
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    module._shard = (rank, world, group)
    pd = partial_dtype or module.k_gate.dtype
    if pd not in (torch.float32, torch.bfloat16):
        raise ValueError("partial_dtype must be torch.float32 or torch.bfloat16")
    module._shard_partial_dtype = pd
    module._shard_routing = bool(shard_routing)
    module._peer_reduce = bool(peer_reduce)
    if not peer_reduce:
        release_peer_buffers(module)


def peer_layout(world: int, rows: int, D: int, esize: int, cap: int) -> dict:
    """Byte layout of one rank's peer buffer (see :class:`PeerReduce`): ``slot`` bytes per (parity, writer)
    partial slot starting at ``slots`` (slots back to back: the combine kernel reads slot w at w * rows * D
    elements), the route tables at ``routes`` (per parity ``route_par`` bytes: ids then counts at
    ``ids_bytes``, each rounded up to 256 bytes), ``total`` bytes in all."""
    al = lambda n: (n + 255) // 256 * 256  # noqa: E731
    slot = rows * D * esize
    ids_bytes = al(world * rows * cap * 4)
    route_par = ids_bytes + al(world * rows * 4)
    slots = kernels.PEER_FLAG_BYTES
    routes = slots + 2 * world * slot
    return {"slot": slot, "slots": slots, "ids_bytes": ids_bytes, "route_par": route_par, "routes": routes,
            "total": routes + 2 * route_par}


class PeerReduce:
    """Receive buffers of the peer-memory reduce-scatter and route exchange, one per rank, mapped into every
    rank of the group through CUDA IPC.  Buffer of rank w: 256 bytes of flags (word v: the last epoch whose
    partial rank v finished storing here; word 32 + v: the last epoch whose routes rank v stored here),
    then 2 parities x world slots x ``rows`` x D partials, then 2 parities of the route table of all
    world x ``rows`` tokens (ids [world*rows, cap] int32, counts [world*rows] int32).  Call e uses parity
    e % 2; each call's epoch is one more than the last, on every rank."""

    ROUTE_FLAGS = 128  # byte offset of the route flags

    def __init__(self, group, rank: int, world: int, rows: int, D: int, dtype: torch.dtype, cap: int, device):
        self.group, self.rank, self.world, self.rows, self.D, self.dtype, self.cap = (group, rank, world, rows, D,
                                                                                     dtype, cap)
        lay = peer_layout(world, rows, D, torch.empty((), dtype=dtype).element_size(), cap)
        self.slot, self.ids_bytes, self.route_par, self.route_base = (lay["slot"], lay["ids_bytes"],
                                                                      lay["route_par"], lay["routes"])
        nbytes = lay["total"]
        self.addr = None
        self.base, handle = kernels.peer_alloc(nbytes)
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        addr, ok = [], True
        for w in range(world):
            if w == rank:
                addr.append(self.base)
                continue
            try:
                addr.append(kernels.peer_open(handles[w]))
            except RuntimeError:
                ok = False
                break
        # every rank learns whether every mapping succeeded, so that all of them use the peer path or none
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
        if int(flag.item()) == 0:
            for w, a in enumerate(addr):
                if w != rank:
                    kernels.peer_close(a)
            kernels.peer_free(self.base)
            raise RuntimeError("peer-memory reduce-scatter: a rank could not map another rank's buffer")
        self.addr = addr
        self.epoch = 0
        self.err = torch.zeros(256, dtype=torch.uint8, device=device)
        self.err_wait = torch.zeros(256, dtype=torch.uint8, device=device)
        # additive-stream contexts of all rows: this rank's rows written per call, the others stay zero
        self.ctx_full = torch.zeros(world * rows, 16, dtype=torch.float32, device=device)

    def fits(self, rows: int, D: int, dtype: torch.dtype, cap: int) -> bool:
        return rows == self.rows and D == self.D and dtype == self.dtype and cap == self.cap

    def slots(self, parity: int):
        """This rank's receive slot on every rank (device addresses)."""
        return [a + kernels.PEER_FLAG_BYTES + (parity * self.world + self.rank) * self.slot for a in self.addr]

    def flags(self):
        """This rank's output flag word on every rank."""
        return [a + 4 * self.rank for a in self.addr]

    def route_flags(self):
        return [a + self.ROUTE_FLAGS + 4 * self.rank for a in self.addr]

    def recv(self, parity: int) -> int:
        """This rank's own slots of one parity."""
        return self.base + kernels.PEER_FLAG_BYTES + parity * self.world * self.slot

    def route_ids(self, parity: int, addr: Optional[int] = None) -> int:
        return (self.base if addr is None else addr) + self.route_base + parity * self.route_par

    def route_counts(self, parity: int, addr: Optional[int] = None) -> int:
        return self.route_ids(parity, addr) + self.ids_bytes

    def close(self) -> None:
        """Collective: every rank unmaps the others' buffers, then frees its own."""
        if self.addr is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for w, a in enumerate(self.addr):
            if w != self.rank:
                kernels.peer_close(a)
        dist.barrier(group=self.group)
        kernels.peer_free(self.base)
        self.addr = None


def release_peer_buffers(module) -> None:
    """Frees the module's peer-memory receive buffers (collective over the shard group)."""
    pr = getattr(module, "_peer_state", None)
    if pr is not None:
        pr.close()
        module._peer_state = None


def _peer_state(module, rows: int, D: int, dtype: torch.dtype, cap: int, device) -> Optional[PeerReduce]:
    """The module's receive buffers for ``rows`` rows per rank (collective when they are (re)built); None,
    with peer_reduce switched off on every rank, when the buffers cannot be mapped."""
    rank, world, group = module._shard
    pr = getattr(module, "_peer_state", None)
    if pr is None or not pr.fits(rows, D, dtype, cap):
        release_peer_buffers(module)
        try:
            pr = PeerReduce(group, rank, world, rows, D, dtype, cap, device)
        except RuntimeError:
            module._peer_reduce = False
            return None
        module._peer_state = pr
    return pr


def _peer_routed_scatter(module, x2d, xv_mine, world: int, rank: int, group, route_fn, pd):
    """Unchunked split-routing forward through peer memory: routes of this rank's rows, stored into every
    rank's route table (in place of an all-gather); the contraction of this rank's blocks from the full
    table, storing every row's partial into the owning rank's receive slot; the sum of this rank's slots.
    Returns (y, None), or (None, (ridx, cnt, ctx)) with the routes all-gathered by NCCL when the shape takes
    a split contraction (decode-size batches) or the buffers cannot be mapped: the caller then reduces with
    the collective (every rank takes the same branch: same shapes)."""
    M, D = x2d.shape
    s = M // world
    kg, ku, v, packed, _, _, wout = module._weights()
    cap = max(int(module.max_remote_blocks), 1)
    ok = (kernels.peer_reduce_supported(x2d.dtype, M, D, kg.shape[0] // 64, cap, world) and s % 4 == 0)
    pr = _peer_state(module, s, D, pd, cap, x2d.device) if ok else None
    if pr is None:
        return None, _gather_routes(module, xv_mine, group, world, rank, route_fn)
    epoch = pr.epoch + 1
    par = epoch & 1
    if getattr(module, "_peer_routes", True):
        ridx, cnt, ctx = route_fn(module, xv_mine)
        kernels.peer_put(ridx.to(torch.int32), [pr.route_ids(par, a) + rank * s * cap * 4 for a in pr.addr])
        kernels.peer_put(cnt.to(torch.int32), [pr.route_counts(par, a) + rank * s * 4 for a in pr.addr])
        kernels.peer_signal(pr.route_flags(), epoch, x2d.device)
        pr.ctx_full[rank * s:(rank + 1) * s].copy_(ctx)
        kernels.peer_wait(pr.base + PeerReduce.ROUTE_FLAGS, world, epoch, pr.err_wait)
        routes = (pr.route_ids(par), pr.route_counts(par), pr.ctx_full)
    else:  # routes all-gathered by NCCL (module._peer_routes = False)
        routes = _gather_routes(module, xv_mine, group, world, rank, route_fn)
    kernels.routed_peer_forward(x2d, kg, ku, v, packed, wout, *routes, base_blocks=module.base_blocks,
                                block_stride=world, block_offset=rank, peer_out=pr.slots(par), peer_flags=pr.flags(),
                                rows_per_rank=s, epoch=epoch, out_f32=pd == torch.float32, capacity=cap)
    pr.epoch = epoch
    y = kernels.peer_combine(pr.recv(par), pr.base, world, s, D, in_f32=pd == torch.float32, epoch=epoch,
                             out_dtype=pd, err_ws=pr.err)
    return y, None


def owned_blocks(num_blocks: int, rank: int, world: int):
    """Block ids owned by ``rank``: b % world == rank."""
    return list(range(rank, num_blocks, world))


def _partial_dtype(module) -> torch.dtype:
    return getattr(module, "_shard_partial_dtype", None) or torch.float32


def _cuda_partial(module, x2d, world: int, rank: int, additive: bool, want_routes: bool, out=None):
    """Replicated routing: this rank's blocks for all tokens, routing every token here."""
    kg, ku, v, packed, wq, k16, wout = module._weights()
    return kernels.token_forward(
        x2d, kg, ku, v, packed, wq, k16, wout, base_blocks=module.base_blocks, top_p=module.top_p,
        min_remote=module.min_remote_blocks, max_remote=module.max_remote_blocks,
        temperature=module.temperature, additive=additive, block_stride=world, block_offset=rank,
        out_f32=_partial_dtype(module) == torch.float32, want_routes=want_routes, y=out)


def _cuda_route(module, x_mine):
    """Routes of this rank's rows: (remote_indices [s, cap] int32, remote_counts [s] int32, ctx16 [s, 16])."""
    _, _, _, _, wq, k16, _ = module._weights()
    return kernels.route_tokens(x_mine, wq, k16, base_blocks=module.base_blocks, top_p=module.top_p,
                                min_remote=module.min_remote_blocks, max_remote=module.max_remote_blocks,
                                temperature=module.temperature)


def _cuda_routed_partial(module, xc, world: int, rank: int, ridx, cnt, ctx16, out=None):
    """This rank's blocks for the rows of ``xc`` from given routes, plus the additive stream of the rows
    whose ctx16 rows are given (zeros elsewhere)."""
    kg, ku, v, packed, _, _, wout = module._weights()
    return kernels.routed_forward(xc, kg, ku, v, packed, wout, ridx, cnt, ctx16, base_blocks=module.base_blocks,
                                  block_stride=world, block_offset=rank,
                                  out_f32=_partial_dtype(module) == torch.float32, y=out)


def _gather_routes(module, x_mine, group, world: int, rank: int, route_fn):
    """Route this rank's rows and all-gather every rank's routes in rank order: (ridx [world*s, cap],
    cnt [world*s], ctx16 [world*s, 16] with this rank's rows' contexts and zeros elsewhere).  One
    collective carries ids and counts together."""
    s = x_mine.shape[0]
    ridx, cnt, ctx = route_fn(module, x_mine)
    cap = ridx.shape[1]
    mine = torch.cat([ridx.to(torch.int32), cnt.to(torch.int32)[:, None]], dim=1).contiguous()
    allr = torch.empty(world * s, cap + 1, dtype=torch.int32, device=x_mine.device)
    dist.all_gather_into_tensor(allr, mine, group=group)
    ctx_full = torch.zeros(world * s, 16, dtype=torch.float32, device=x_mine.device)
    ctx_full[rank * s:(rank + 1) * s] = ctx
    return allr[:, :cap], allr[:, cap], ctx_full


def _use_shard_routing(module, M: int, world: int, want_routes: bool, compute_partial) -> bool:
    return (getattr(module, "_shard_routing", False) and not want_routes and compute_partial is None
            and M % world == 0)


def _comm_stream(module, device) -> torch.cuda.Stream:
    st = getattr(module, "_comm_stream_obj", None)
    if st is None or st.device != device:
        st = torch.cuda.Stream(device=device)
        module._comm_stream_obj = st
    return st


def sharded_token_forward(module, x2d: torch.Tensor, *, want_routes: bool = False, reduce: str = "all",
                          compute_partial: Optional[Callable] = None, chunks: int = 1,
                          route_fn: Optional[Callable] = None, routed_fn: Optional[Callable] = None):
    """Parameter-block-sharded forward of a batch held by every rank.  Returns (y, remote_indices,
    remote_counts, scores); with ``reduce="scatter"`` y holds only this rank's contiguous slice of token
    rows.

    ``chunks > 1`` overlaps the collective with compute: chunk i's partial is reduced on a side stream
    while chunk i+1 is computed.  For ``reduce="scatter"`` chunk i gathers, for every rank r, the i-th
    piece of r's output slice, so that each rank's result stays one contiguous slice; this needs the
    token count to divide by ``world * chunks``.  Routes are returned only without chunking (and then the
    routing is replicated).  ``compute_partial`` / ``route_fn`` + ``routed_fn`` replace the CUDA kernels
    (host-side tests)."""
    rank, world, group = module._shard
    if reduce not in ("all", "scatter"):
        raise ValueError("reduce must be 'all' or 'scatter'")
    M, D = x2d.shape
    if reduce == "scatter" and M % world:
        raise ValueError("reduce='scatter' needs the token count to divide by the world size")
    chunks = 1 if want_routes else max(1, int(chunks))
    split_routes = route_fn is not None or (_use_shard_routing(module, M, world, want_routes, compute_partial)
                                            and M % (world * chunks) == 0)
    route_fn = route_fn or _cuda_route
    routed_fn = routed_fn or _cuda_routed_partial
    fn = compute_partial or _cuda_partial
    pd = _partial_dtype(module)
    rank_major = split_routes or (chunks > 1 and reduce == "scatter")
    if rank_major and M % (world * chunks):
        raise ValueError("sharding with split routing or a chunked reduce-scatter needs the token count to "
                         "divide by world * chunks")
    s = M // (world * chunks) if rank_major else 0

    def partial_of(xc, xv_mine):
        """This rank's partial for the rows of xc (rank-major pieces; xv_mine = this rank's piece)."""
        if split_routes:
            ridx, cnt, ctx = _gather_routes(module, xv_mine, group, world, rank, route_fn)
            return routed_fn(module, xc, world, rank, ridx, cnt, ctx).to(pd)
        return fn(module, xc, world, rank, rank == 0, False)[0].to(pd)

    if chunks <= 1 or want_routes:
        if split_routes:
            xv = x2d.view(world, s, D)
            routes = None
            if (reduce == "scatter" and getattr(module, "_peer_reduce", False) and x2d.is_cuda
                    and route_fn is _cuda_route and routed_fn is _cuda_routed_partial):
                y, routes = _peer_routed_scatter(module, x2d, xv[rank], world, rank, group, route_fn, pd)
                if y is not None:
                    return y.to(x2d.dtype), None, None, None
            if routes is not None:  # the peer path declined this shape: reduce with the collective
                y_part = routed_fn(module, x2d, world, rank, *routes).to(pd)
            else:
                y_part = partial_of(x2d, xv[rank])
            ridx = cnt = S = None
        else:
            y_part, ridx, cnt, S = fn(module, x2d, world, rank, rank == 0, want_routes)
            y_part = y_part.to(pd)
        if reduce == "all":
            dist.all_reduce(y_part, op=dist.ReduceOp.SUM, group=group)
            y = y_part
        else:
            y = torch.empty(M // world, D, dtype=y_part.dtype, device=y_part.device)
            dist.reduce_scatter_tensor(y, y_part, op=dist.ReduceOp.SUM, group=group)
        return y.to(x2d.dtype), ridx, cnt, S

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
    if not rank_major:
        # all-reduce with the routing replicated: contiguous token chunks, each partial written in place
        y = torch.empty(M, D, dtype=pd, device=x2d.device)
        bounds = [M * i // chunks for i in range(chunks + 1)]
        for i in range(chunks):
            lo, hi = bounds[i], bounds[i + 1]
            if fn is _cuda_partial:  # the kernel writes its partial straight into the output rows
                part = fn(module, x2d[lo:hi], world, rank, rank == 0, False, out=y[lo:hi])[0]
            else:
                y[lo:hi].copy_(fn(module, x2d[lo:hi], world, rank, rank == 0, False)[0].to(pd))
                part = y[lo:hi]
            with after_compute():
                works.append(dist.all_reduce(part, op=dist.ReduceOp.SUM, group=group, async_op=True))
        for w in works:
            w.wait()
        return y.to(x2d.dtype), None, None, None

    # chunk i holds piece i of every rank's row slice (rank-major), so that the routing of chunk i is split
    # over the ranks and, for reduce-scatter, each rank's output stays one contiguous slice
    xv = x2d.view(world, chunks, s, D)
    parts = []
    y = torch.empty(M // world, D, dtype=pd, device=x2d.device) if reduce == "scatter" else None
    for i in range(chunks):
        part = partial_of(xv[:, i].reshape(world * s, D), xv[rank, i])
        with after_compute():
            if reduce == "all":
                parts.append(part)
                works.append(dist.all_reduce(part, op=dist.ReduceOp.SUM, group=group, async_op=True))
            else:
                works.append(dist.reduce_scatter_tensor(y[i * s:(i + 1) * s], part, op=dist.ReduceOp.SUM,
                                                        group=group, async_op=True))
    for w in works:
        w.wait()
    if reduce == "all":  # back from rank-major pieces to token order
        y = torch.stack(parts).view(chunks, world, s, D).transpose(0, 1).reshape(M, D)
    return y.to(x2d.dtype), None, None, None


def sharded_forward_slices(module, x_slice: torch.Tensor, *, chunks: int = 1,
                           compute_partial: Optional[Callable] = None, route_fn: Optional[Callable] = None,
                           routed_fn: Optional[Callable] = None) -> torch.Tensor:
    """Block-sharded forward of a token batch that is partitioned over the ranks.

    Every rank passes its own contiguous slice of the batch's token rows (the same number on every rank)
    and receives the output rows of that slice.  Per chunk: an all-gather brings piece i of every rank's
    slice to every rank (NVLink, rank-major), each rank routes its own piece and the routes are
    all-gathered (or, with ``compute_partial``, every rank routes all rows), each rank computes the partial
    output of its parameter blocks over those rows, and a reduce-scatter returns to every rank the sum for
    its own piece.  Chunk i+1's all-gather is issued before chunk i's reduce-scatter, so on GPUs the
    collectives of one chunk run while another chunk computes.  No rank ever holds more than its slice of
    the input at the start: the host-to-device traffic of a job is split over the ranks' links instead of
    every rank copying the whole batch."""
    rank, world, group = module._shard
    split_routes = route_fn is not None or (getattr(module, "_shard_routing", False) and compute_partial is None)
    route_fn = route_fn or _cuda_route
    routed_fn = routed_fn or _cuda_routed_partial
    fn = compute_partial or _cuda_partial
    s_all, D = x_slice.shape
    chunks = max(1, min(int(chunks), s_all)) if s_all else 1
    if s_all % chunks:
        raise ValueError("the slice's token count must divide by the number of chunks")
    s = s_all // chunks
    pd = _partial_dtype(module)
    dev = x_slice.device
    y = torch.empty(s_all, D, dtype=pd, device=dev)
    if s_all == 0:
        return y.to(x_slice.dtype)
    gathered = [torch.empty(world * s, D, dtype=x_slice.dtype, device=dev) for _ in range(chunks)]

    def gather(i):
        return dist.all_gather_into_tensor(gathered[i], x_slice[i * s:(i + 1) * s].contiguous(), group=group,
                                           async_op=True)

    ag = [gather(0)] + ([gather(1)] if chunks > 1 else [])
    rs = []
    for i in range(chunks):
        ag[i].wait()  # the current stream waits for chunk i's rows
        if split_routes:
            ridx, cnt, ctx = _gather_routes(module, x_slice[i * s:(i + 1) * s], group, world, rank, route_fn)
            part = routed_fn(module, gathered[i], world, rank, ridx, cnt, ctx).to(pd)
        else:
            part = fn(module, gathered[i], world, rank, rank == 0, False)[0].to(pd)
        rs.append(dist.reduce_scatter_tensor(y[i * s:(i + 1) * s], part, op=dist.ReduceOp.SUM, group=group,
                                             async_op=True))
        if i + 2 < chunks:
            ag.append(gather(i + 2))
    for w in rs:
        w.wait()
    return y.to(x_slice.dtype)


def sharded_forward_host(module, x_host: torch.Tensor, out: Optional[torch.Tensor] = None, *,
                         chunks: int = 4) -> torch.Tensor:
    """:func:`sharded_forward_slices` for a slice held in host memory (pinned for the copies to overlap):
    each chunk's rows are copied to the device on a copy stream, gathered, routed (this rank's rows, routes
    all-gathered), computed and reduce-scattered, and its output rows copied back on another stream while
    later chunks run.  Returns the output slice in host memory, complete once the caller's current stream
    has been synchronised."""
    rank, world, group = module._shard
    dev = module.k_gate.device
    s_all, D = x_host.shape
    chunks = max(1, min(int(chunks), s_all)) if s_all else 1
    if s_all % chunks:
        raise ValueError("the slice's token count must divide by the number of chunks")
    s = s_all // chunks
    if out is None:
        out = torch.empty(s_all, D, dtype=x_host.dtype, pin_memory=True)
    if s_all == 0:
        return out
    split_routes = getattr(module, "_shard_routing", False)
    st = getattr(module, "_shard_host_streams", None)
    if st is None or st[0].device != dev:
        st = tuple(torch.cuda.Stream(device=dev) for _ in range(3))
        module._shard_host_streams = st
    s_in, s_ag, s_out = st
    cur = torch.cuda.current_stream(dev)
    for st_ in st:
        st_.wait_stream(cur)
    pd = _partial_dtype(module)
    # device buffers are kept across calls (per shape): every stream above waited for the caller's stream,
    # which waited for the previous call's last copy-out, so the previous call is done with them; fresh
    # allocations per call left the caching allocator with blocks held by the side streams (record_stream)
    # and measured calls that stalled in new device allocations
    key = (s_all, D, chunks, x_host.dtype, pd, world)
    bufs = getattr(module, "_shard_host_bufs", None)
    if bufs is None or bufs[0] != key or bufs[1].device != dev:
        bufs = (key, torch.empty(s_all, D, dtype=x_host.dtype, device=dev),
                torch.empty(s_all, D, dtype=pd, device=dev),
                [torch.empty(world * s, D, dtype=x_host.dtype, device=dev) for _ in range(chunks)])
        module._shard_host_bufs = bufs
    _, x_dev, y_dev, gathered = bufs
    copied = []
    with torch.cuda.stream(s_in):  # every chunk's copy-in is queued at once; each signals its own event
        for i in range(chunks):
            x_dev[i * s:(i + 1) * s].copy_(x_host[i * s:(i + 1) * s], non_blocking=True)
            copied.append(torch.cuda.Event())
            copied[-1].record(s_in)

    def gather(i):
        s_ag.wait_event(copied[i])
        with torch.cuda.stream(s_ag):  # the collective waits for chunk i's copy-in only
            return dist.all_gather_into_tensor(gathered[i], x_dev[i * s:(i + 1) * s], group=group, async_op=True)

    ag = [gather(0)] + ([gather(1)] if chunks > 1 else [])
    for i in range(chunks):
        ag[i].wait()
        if split_routes:
            ridx, cnt, ctx = _gather_routes(module, x_dev[i * s:(i + 1) * s], group, world, rank, _cuda_route)
            part = _cuda_routed_partial(module, gathered[i], world, rank, ridx, cnt, ctx)
        else:
            part = _cuda_partial(module, gathered[i], world, rank, rank == 0, False)[0]
        w = dist.reduce_scatter_tensor(y_dev[i * s:(i + 1) * s], part, op=dist.ReduceOp.SUM, group=group,
                                       async_op=True)
        with torch.cuda.stream(s_out):
            w.wait()
            yv = y_dev[i * s:(i + 1) * s]
            out[i * s:(i + 1) * s].copy_(yv if pd == x_host.dtype else yv.to(x_host.dtype), non_blocking=True)
        if i + 2 < chunks:
            ag.append(gather(i + 2))
    cur.wait_stream(s_out)
    return out


def split_tokens(x2d: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Token-split layout: this rank's contiguous share of the token rows (ranks < M % world get one more)."""
    M = x2d.shape[0]
    base, extra = divmod(M, world)
    start = rank * base + min(rank, extra)
    return x2d[start:start + base + (1 if rank < extra else 0)]
