"""Parameter-block sharding over NCCL on 2 GPUs (skipped with fewer than 2 visible GPUs).

Each rank computes the partial output of the blocks it owns (b % 2 == rank) for all tokens; an NCCL
all-reduce (or reduce-scatter over token rows) sums the fp32 or bf16 partials, in one piece or chunk by
chunk with each chunk's collective overlapping the next chunk's compute; with the token-partitioned input
each rank starts from its own slice of the batch (device or pinned host memory), which an all-gather
brings to every rank.  The result must match the
single-GPU forward within the bf16 tolerance, and the routes must be identical on both ranks.
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

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    sys.path.insert(0, REPO)
    sys.path.insert(0, HERE)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    from conftest import configs, fsi, rel_err
    wl = configs.CONFIGS["8b"]
    w = configs.make_weights(wl)
    x = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:2048].contiguous().to(dev, torch.bfloat16)

    def module():
        m = fsi.FovealPattentionMLP(hidden_dim=wl.hidden_dim, intermediate_dim=wl.intermediate_dim,
                                    base_blocks=wl.base_blocks, remote_blocks=wl.max_remote_blocks,
                                    dtype=torch.bfloat16, routing="token", top_p=wl.top_p,
                                    min_remote_blocks=wl.min_remote_blocks, max_remote_blocks=wl.max_remote_blocks)
        m.load_state_dict({k: t.to(torch.bfloat16) for k, t in w.state_dict().items()}, strict=False)
        return m.to(dev).eval()

    rows = slice(rank * 1024, (rank + 1) * 1024)
    with torch.no_grad():
        full, info_full = module()(x, return_router_info=True)
        m = module()
        fsi.sharding.shard_parameter_blocks(m, partial_dtype=torch.float32)
        y, info = m(x, return_router_info=True)
        ys, _, _, _ = fsi.sharding.sharded_token_forward(m, x, reduce="scatter")
        # chunked: each chunk's collective overlaps the next chunk's compute
        yc, _, _, _ = fsi.sharding.sharded_token_forward(m, x, reduce="all", chunks=3)
        ysc, _, _, _ = fsi.sharding.sharded_token_forward(m, x, reduce="scatter", chunks=4)
        # bf16 partials (the bf16 model's default): half the bytes on NVLink
        mb = module()
        fsi.sharding.shard_parameter_blocks(mb)  # routing split over the ranks (the default)
        ysb, _, _, _ = fsi.sharding.sharded_token_forward(mb, x, reduce="scatter", chunks=4)
        ysa, _, _, _ = fsi.sharding.sharded_token_forward(mb, x, reduce="all", chunks=2)
        mr = module()
        fsi.sharding.shard_parameter_blocks(mr, shard_routing=False)  # every rank routes every token
        ysr, _, _, _ = fsi.sharding.sharded_token_forward(mr, x, reduce="scatter", chunks=4)
        # token-partitioned input: each rank passes only its slice (all-gather, compute, reduce-scatter),
        # from device memory and from pinned host memory
        ysl = fsi.sharding.sharded_forward_slices(mb, x[rows].contiguous(), chunks=4)
        yh = fsi.sharding.sharded_forward_host(mb, x[rows].cpu().pin_memory(), chunks=4)
        # peer-memory reduce-scatter: the contraction stores the peer's rows over NVLink; three calls cover
        # both receive parities and a reused buffer; bf16 and fp32 partials
        mp_ = module()
        fsi.sharding.shard_parameter_blocks(mp_, peer_reduce=True)
        yp = [fsi.sharding.sharded_token_forward(mp_, x, reduce="scatter")[0] for _ in range(3)]
        peer_err = fsi._lib.device_error(mp_._peer_state.err) or fsi._lib.device_error(mp_._peer_state.err_wait)
        peer_epoch = mp_._peer_state.epoch
        fsi.sharding.release_peer_buffers(mp_)
        mf = module()
        fsi.sharding.shard_parameter_blocks(mf, partial_dtype=torch.float32, peer_reduce=True)
        ypf = fsi.sharding.sharded_token_forward(mf, x, reduce="scatter")[0]
        fsi.sharding.release_peer_buffers(mf)
    torch.cuda.synchronize()
    e_all = max(rel_err(y.float(), full.float()), rel_err(yc.float(), full.float()))
    e_all = max(e_all, rel_err(ysa.float(), full.float()))
    e_sc = max(rel_err(t.float().cpu(), full[rows].float().cpu()) for t in (ys, ysc, ysb, ysr, ysl, yh, *yp, ypf))
    same_routes = bool(torch.equal(info["remote_indices"], info_full["remote_indices"]))
    peer_ok = int(peer_err == 0 and peer_epoch == 3 and torch.equal(yp[0], yp[1]) and torch.equal(yp[1], yp[2]))
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(f"{e_all} {e_sc} {int(same_routes)} {peer_ok}")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_block_sharded_forward_over_nccl_matches_single_gpu():
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.spawn(_worker, args=(2, port, d), nprocs=2, join=False)
        deadline = time.time() + 600
        while not ctx.join(timeout=5):
            if time.time() > deadline:
                for p in ctx.processes:
                    if p.is_alive():
                        p.kill()
                pytest.fail("sharded forward did not finish")
        for r in range(2):
            e_all, e_sc, same, peer_ok = open(os.path.join(d, f"r{r}.txt")).read().split()
            assert float(e_all) < 2e-2 and float(e_sc) < 2e-2 and same == "1", (r, e_all, e_sc, same)
            assert peer_ok == "1", r  # peer path: no wait ran out, three epochs, repeated calls bit-equal


def _single_rank_worker(index, port, out_dir):
    sys.path.insert(0, REPO)
    sys.path.insert(0, HERE)
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    dist.init_process_group("nccl", rank=0, world_size=1, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=120), device_id=dev)
    from conftest import configs, fsi, rel_err
    wl = configs.CONFIGS["8b"]
    w = configs.make_weights(wl)
    x = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:1024].contiguous().to(dev, torch.bfloat16)
    m = fsi.FovealPattentionMLP(hidden_dim=wl.hidden_dim, intermediate_dim=wl.intermediate_dim,
                                base_blocks=wl.base_blocks, remote_blocks=wl.max_remote_blocks,
                                dtype=torch.bfloat16, routing="token", top_p=wl.top_p,
                                min_remote_blocks=wl.min_remote_blocks, max_remote_blocks=wl.max_remote_blocks)
    m.load_state_dict({k: t.to(torch.bfloat16) for k, t in w.state_dict().items()}, strict=False)
    m = m.to(dev).eval()
    with torch.no_grad():
        full = m(x)
        fsi.sharding.shard_parameter_blocks(m, peer_reduce=True)
        ys = [fsi.sharding.sharded_token_forward(m, x, reduce="scatter")[0] for _ in range(3)]
        st = m._peer_state
        ok = (st is not None and st.epoch == 3 and fsi._lib.device_error(st.err) == 0
              and fsi._lib.device_error(st.err_wait) == 0)
        fsi.sharding.release_peer_buffers(m)
    torch.cuda.synchronize()
    e = max(rel_err(y.float(), full.float()) for y in ys)
    same = all(torch.equal(ys[0], y) for y in ys)
    with open(os.path.join(out_dir, "r0.txt"), "w") as f:
        f.write(f"{e} {int(same)} {int(ok)}")
    dist.destroy_process_group()


def test_peer_route_exchange_single_rank():
    """The peer-memory path of the sharded forward as a job of one rank (one GPU): the routes go through the
    peer route table (put, flag, wait), the contraction stores into the rank's own slot, the combine waits
    for its own flag.  Three calls (both parities) equal the unsharded forward within the bf16 bar and
    each other bit for bit; no bounded wait ran out."""
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.spawn(_single_rank_worker, args=(port, d), nprocs=1, join=False)
        deadline = time.time() + 300
        while not ctx.join(timeout=5):
            if time.time() > deadline:
                for p in ctx.processes:
                    if p.is_alive():
                        p.kill()
                pytest.fail("single-rank peer forward did not finish")
        e, same, ok = open(os.path.join(d, "r0.txt")).read().split()
        assert float(e) < 2e-2 and same == "1" and ok == "1", (e, same, ok)
