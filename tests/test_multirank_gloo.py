"""Multi-rank host logic on CPU (gloo, world_size 2).

* Parameter-block sharding: every rank routes all tokens, computes the partial output of the blocks it
  owns (b % world == rank; the additive stream only on rank 0), and an all-reduce (or reduce-scatter)
  sums the partials, in one piece or chunk by chunk.  The partials here come from the CPU oracle restricted to the owned blocks, so the
  test checks the decomposition and the collective wiring of ``sharding.sharded_token_forward``.
* Failure detection: a rank that leaves before the collective makes the other rank's collective end
  with an error within the process-group timeout instead of hanging.
"""

from __future__ import annotations

import datetime
import os
import socket
import sys
import tempfile
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank, world, port, timeout_s=60):
    sys.path.insert(0, REPO)
    sys.path.insert(0, HERE)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _oracle_partial(module, x2d, world, rank, additive, want_routes):
    import oracle
    from conftest import configs

    w = configs.Weights(module.k_gate.detach(), module.k_up.detach(), module.v.detach(),
                        module.q_proj_16d.weight.detach(), module.block_keys_16d.detach(),
                        module.out_proj_16d.weight.detach())
    S = oracle.router_scores(x2d, w.q_proj_16d, w.block_keys_16d) / module.temperature
    r = oracle.select_blocks_noncausal(S[None], local_window_blocks=module.base_blocks, top_p=module.top_p,
                                       min_remote_blocks=module.min_remote_blocks,
                                       max_remote_blocks=module.max_remote_blocks,
                                       remote_capacity=module.max_remote_blocks)
    idx, cnt = r.remote_indices[0], r.remote_counts[0]
    M = x2d.shape[0]
    sel = torch.zeros(M, module.num_blocks, dtype=torch.bool)
    sel[:, :module.base_blocks] = True
    for t in range(M):
        sel[t, idx[t, :int(cnt[t])].long()] = True
    y = torch.zeros(M, x2d.shape[1])
    for b in range(rank, module.num_blocks, world):  # owned blocks
        toks = sel[:, b].nonzero().flatten()
        if toks.numel():
            rows = slice(b * 64, (b + 1) * 64)
            xb = x2d[toks]
            h = torch.nn.functional.silu(xb @ w.k_gate[rows].t()) * (xb @ w.k_up[rows].t())
            y.index_add_(0, toks, h @ w.v[rows])
    if additive:
        y = y + oracle.additive_stream(S, w.block_keys_16d, w.out_proj_16d)
    return y, idx, cnt, S


def _oracle_route(module, x_mine):
    """Routes of this rank's rows (oracle): (ids [s, cap], counts [s], ctx16 [s, 16])."""
    import oracle
    w = m_weights(module)
    S = oracle.router_scores(x_mine, w.q_proj_16d, w.block_keys_16d) / module.temperature
    r = oracle.select_blocks_noncausal(S[None], local_window_blocks=module.base_blocks, top_p=module.top_p,
                                       min_remote_blocks=module.min_remote_blocks,
                                       max_remote_blocks=module.max_remote_blocks,
                                       remote_capacity=module.max_remote_blocks)
    ctx = torch.softmax(S, dim=-1) @ w.block_keys_16d
    return r.remote_indices[0], r.remote_counts[0], ctx


def _oracle_routed(module, xc, world, rank, ridx, cnt, ctx16):
    """This rank's blocks from given routes (oracle) plus ctx16 . W_out^T of the given context rows."""
    w = m_weights(module)
    M = xc.shape[0]
    sel = torch.zeros(M, module.num_blocks, dtype=torch.bool)
    sel[:, :module.base_blocks] = True
    for t in range(M):
        sel[t, ridx[t, :int(cnt[t])].long()] = True
    y = torch.zeros(M, xc.shape[1])
    for b in range(rank, module.num_blocks, world):
        toks = sel[:, b].nonzero().flatten()
        if toks.numel():
            rows = slice(b * 64, (b + 1) * 64)
            xb = xc[toks]
            h = torch.nn.functional.silu(xb @ w.k_gate[rows].t()) * (xb @ w.k_up[rows].t())
            y.index_add_(0, toks, h @ w.v[rows])
    return y + ctx16 @ w.out_proj_16d.t()


def _split_routes_worker(rank, world, port, out_dir):
    """Routing split over the ranks: each rank routes its share, the routes are all-gathered, each rank's
    contraction runs from the given routes (sharded_token_forward, chunked; sharded_forward_slices)."""
    _setup(rank, world, port)
    from conftest import fsi
    import oracle

    torch.manual_seed(0)
    m = fsi.FovealPattentionMLP(hidden_dim=64, intermediate_dim=640, base_blocks=2, remote_blocks=3,
                                dtype=torch.float32, routing="token", top_p=0.7, min_remote_blocks=1,
                                max_remote_blocks=3)
    with torch.no_grad():
        m.out_proj_16d.weight.normal_(std=0.05)
    M = 8 * world
    x2d = torch.randn(M, 64)
    fsi.sharding.shard_parameter_blocks(m)
    hooks = dict(route_fn=_oracle_route, routed_fn=_oracle_routed)
    ya, _, _, _ = fsi.sharding.sharded_token_forward(m, x2d, reduce="all", **hooks)
    yac, _, _, _ = fsi.sharding.sharded_token_forward(m, x2d, reduce="all", chunks=2, **hooks)
    ys, _, _, _ = fsi.sharding.sharded_token_forward(m, x2d, reduce="scatter", chunks=4, **hooks)
    s = M // world
    yl = fsi.sharding.sharded_forward_slices(m, x2d[rank * s:(rank + 1) * s].contiguous(), chunks=2, **hooks)
    ref = oracle.token_forward(x2d, m_weights(m), base_blocks=2, top_p=0.7, min_remote_blocks=1,
                               max_remote_blocks=3)["y"]
    mine = ref[rank * s:(rank + 1) * s]
    errs = [float((ya - ref).norm() / ref.norm()), float((yac - ref).norm() / ref.norm()),
            float((ys - mine).norm() / mine.norm()), float((yl - mine).norm() / mine.norm())]
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(" ".join(str(e) for e in errs))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_split_routing_matches_full(world):
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_split_routes_worker, args=(world, port, d), nprocs=world, join=True)
        for r in range(world):
            errs = list(map(float, open(os.path.join(d, f"r{r}.txt")).read().split()))
            assert len(errs) == 4 and max(errs) < 1e-5, (r, errs)


def _shard_worker(rank, world, port, out_dir):
    _setup(rank, world, port)
    from conftest import fsi
    import oracle

    torch.manual_seed(0)
    m = fsi.FovealPattentionMLP(hidden_dim=64, intermediate_dim=640, base_blocks=2, remote_blocks=3,
                                dtype=torch.float32, routing="token", top_p=0.7, min_remote_blocks=1,
                                max_remote_blocks=3)
    with torch.no_grad():
        m.out_proj_16d.weight.normal_(std=0.05)
    x2d = torch.randn(32, 64)
    fsi.sharding.shard_parameter_blocks(m)
    assert fsi.sharding.owned_blocks(10, rank, world) == list(range(rank, 10, world))
    y, _, _, _ = fsi.sharding.sharded_token_forward(m, x2d, compute_partial=_oracle_partial)
    ys, _, _, _ = fsi.sharding.sharded_token_forward(m, x2d, compute_partial=_oracle_partial, reduce="scatter")
    # chunked: the collective of chunk i overlaps chunk i+1 on GPUs; here the decomposition and, for
    # reduce-scatter, the rank-major chunk layout that keeps each rank's rows contiguous
    yc, _, _, _ = fsi.sharding.sharded_token_forward(m, x2d, compute_partial=_oracle_partial, chunks=3)
    ysc, _, _, _ = fsi.sharding.sharded_token_forward(m, x2d, compute_partial=_oracle_partial, reduce="scatter",
                                                     chunks=4)
    ref = oracle.token_forward(x2d, m_weights(m), base_blocks=2, top_p=0.7, min_remote_blocks=1,
                               max_remote_blocks=3)["y"]
    mine = ref[rank * 16:(rank + 1) * 16]
    errs_all = [float((t - ref).norm() / ref.norm()) for t in (y, yc)]
    errs_sc = [float((t - mine).norm() / mine.norm()) for t in (ys, ysc)]
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(" ".join(str(e) for e in errs_all + errs_sc))
    dist.destroy_process_group()


def m_weights(m):
    from conftest import configs
    return configs.Weights(m.k_gate.detach(), m.k_up.detach(), m.v.detach(), m.q_proj_16d.weight.detach(),
                           m.block_keys_16d.detach(), m.out_proj_16d.weight.detach())


def test_block_sharded_forward_matches_full():
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_shard_worker, args=(2, port, d), nprocs=2, join=True)
        for r in range(2):
            errs = list(map(float, open(os.path.join(d, f"r{r}.txt")).read().split()))
            assert len(errs) == 4 and max(errs) < 1e-5, (r, errs)


def _slices_worker(rank, world, port, out_dir, partial_dtype, chunks):
    """Token-partitioned input: each rank holds only its slice of the batch; all-gather, block-sharded
    partials (oracle restricted to the owned blocks, rounded to the partial dtype as the kernel stores
    them) and reduce-scatter return this rank's output rows."""
    _setup(rank, world, port)
    from conftest import fsi
    import oracle

    torch.manual_seed(0)
    m = fsi.FovealPattentionMLP(hidden_dim=128, intermediate_dim=2048, base_blocks=4, remote_blocks=8,
                                dtype=torch.float32, routing="token", top_p=0.8, min_remote_blocks=2,
                                max_remote_blocks=8)
    with torch.no_grad():
        for p_ in (m.k_gate, m.k_up, m.v, m.q_proj_16d.weight, m.block_keys_16d):
            p_.normal_(std=0.05)
        m.out_proj_16d.weight.normal_(std=0.05)
    x2d = torch.randn(world * 24, 128)
    pd = {"fp32": torch.float32, "bf16": torch.bfloat16}[partial_dtype]
    fsi.sharding.shard_parameter_blocks(m, partial_dtype=pd)

    def partial(mod, xg, w_, r_, additive, want_routes):
        y, *rest = _oracle_partial(mod, xg, w_, r_, additive, want_routes)
        return (y.to(pd), *rest)

    mine = x2d[rank * 24:(rank + 1) * 24].contiguous()
    y = fsi.sharding.sharded_forward_slices(m, mine, chunks=chunks, compute_partial=partial)
    ref = oracle.token_forward(x2d, m_weights(m), base_blocks=4, top_p=0.8, min_remote_blocks=2,
                               max_remote_blocks=8)["y"][rank * 24:(rank + 1) * 24]
    err = float((y.float() - ref).norm() / ref.norm())
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(f"{err} {tuple(y.shape) == (24, 128)}")
    dist.destroy_process_group()


@pytest.mark.parametrize("world,partial_dtype,chunks,tol", [(2, "fp32", 3, 1e-5), (4, "fp32", 1, 1e-5),
                                                            (8, "bf16", 2, 2e-2)])
def test_token_partitioned_block_sharding(world, partial_dtype, chunks, tol):
    """sharded_forward_slices at 2, 4 and 8 ranks; at 8 ranks with bf16 partials (the bf16 model's
    default), whose sum must stay within the 2e-2 relative bar of bf16 outputs."""
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_slices_worker, args=(world, port, d, partial_dtype, chunks), nprocs=world, join=True)
        for r in range(world):
            err, shape_ok = open(os.path.join(d, f"r{r}.txt")).read().split()
            assert shape_ok == "True" and float(err) < tol, (r, err)


def _token_split_worker(rank, world, port, out_dir):
    _setup(rank, world, port)
    from conftest import fsi

    x = torch.arange(37 * 3, dtype=torch.float32).view(37, 3)
    part = fsi.sharding.split_tokens(x, rank, world)
    sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(sizes, torch.tensor([part.shape[0]]))
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(f"{int(part[0, 0]) // 3} {part.shape[0]} {sum(int(s) for s in sizes)}")
    dist.destroy_process_group()


def test_token_split_covers_all_rows():
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_token_split_worker, args=(2, port, d), nprocs=2, join=True)
        r0 = list(map(int, open(os.path.join(d, "r0.txt")).read().split()))
        r1 = list(map(int, open(os.path.join(d, "r1.txt")).read().split()))
        assert r0 == [0, 19, 37] and r1 == [19, 18, 37]


def _failure_worker(rank, world, port, out_dir):
    _setup(rank, world, port, timeout_s=5)
    if rank == 1:
        # leaves between steps, before the collective, with nothing in flight
        with open(os.path.join(out_dir, "r1.txt"), "w") as f:
            f.write("left")
        os._exit(0)
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        outcome = "completed"
    except Exception as e:  # noqa: BLE001 - any collective error is the expected outcome
        outcome = f"error:{type(e).__name__}"
    with open(os.path.join(out_dir, "r0.txt"), "w") as f:
        f.write(outcome)
    os._exit(0)


def test_lost_rank_surfaces_as_error_not_hang():
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.spawn(_failure_worker, args=(2, port, d), nprocs=2, join=False)
        deadline = time.time() + 120
        while not ctx.join(timeout=2):
            if time.time() > deadline:
                for p in ctx.processes:
                    if p.is_alive():
                        p.kill()
                pytest.fail("a rank hung instead of failing")
        assert open(os.path.join(d, "r0.txt")).read().startswith("error:")
