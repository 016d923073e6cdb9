"""GPU parity: the CUDA path (through the C ABI) against the golden vectors and the CPU oracle.

Bars: active-block sets and counts bit-exact.  Tokens whose reference boundary margin lies below
TIE_EPS are rounding-level near ties: they are counted (in the band, and how many of them differ) and
reported at the end of the run, not failed.  Where both sides compute bit-equal probabilities for the
tied blocks (repeated block keys, equal scores), the lower block id must win and nothing is excused.  Outputs within 1e-4 relative (fp32 configuration) or 2e-2 relative (bf16
configurations) of the fp32 reference, measured as ||y - ref|| / ||ref|| and as max|y - ref| / max|ref|.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

import oracle
from conftest import active_set_matches, serve_model, compare_routes, configs, fsi, golden, max_rel, rel_err

pytestmark = pytest.mark.gpu

TOL = {"fp32": 1e-4, "bf16": 2e-2}
DEV = "cuda"


def module_for(wl, w, routing="token", remote_blocks=None):
    m = fsi.FovealPattentionMLP(
        hidden_dim=wl.hidden_dim, intermediate_dim=wl.intermediate_dim, base_blocks=wl.base_blocks,
        remote_blocks=remote_blocks if remote_blocks is not None else wl.max_remote_blocks,
        temperature=wl.temperature, dtype=wl.torch_dtype, routing=routing, top_p=wl.top_p,
        min_remote_blocks=wl.min_remote_blocks, max_remote_blocks=wl.max_remote_blocks)
    sd = {k: t.to(wl.torch_dtype) for k, t in w.state_dict().items()}
    m.load_state_dict(sd, strict=False)
    return m.to(DEV).eval()


def check_y(y, ref, dtype, factor=1.0):
    tol = TOL[dtype] * factor
    e1, e2 = rel_err(y.float(), ref), max_rel(y.float(), ref)
    assert e1 < tol and e2 < tol, f"rel_l2 {e1:.3e}, max_rel {e2:.3e}, tol {tol}"
    return e1


def run_token(m, x2d):
    with torch.no_grad():
        y, info = m(x2d.to(DEV), return_router_info=True)
    torch.cuda.synchronize()
    return y, info


def device_error_is_clear():
    ws = fsi._lib._ws
    for buf in ws.values():
        assert fsi._lib.device_error(buf) == 0


# ------------------------------------------------------------------ router
@pytest.mark.parametrize("case", ["guard", "peaked", "wide", "nobase"])
def test_select_blocks_known_answer(case):
    g = golden("router_kat")
    base, tp, kmin, kmax, cap = g[f"{case}_params"]
    s = torch.from_numpy(g[f"{case}_scores"]).to(DEV)
    r = fsi.select_blocks(s, causal=False, local_window_blocks=int(base), top_p=float(tp),
                          min_remote_blocks=int(kmin), max_remote_blocks=int(kmax), remote_capacity=int(cap))
    B, Q, _ = s.shape
    bad, _ = compare_routes(r.remote_indices.reshape(B * Q, -1).cpu(), r.remote_counts.reshape(-1).cpu(),
                            g[f"{case}_indices"].reshape(B * Q, -1), g[f"{case}_counts"].reshape(-1))
    assert bad == 0
    assert np.array_equal(r.remote_counts.cpu().numpy(), g[f"{case}_counts"])
    assert abs(float(r.cap_rate) - float(g[f"{case}_cap_rate"])) < 1e-6
    # full capacity array, including the tail past the counts (base ids / padding), matches the oracle
    o = oracle.select_blocks_noncausal(s.cpu(), local_window_blocks=int(base), top_p=float(tp),
                                       min_remote_blocks=int(kmin), max_remote_blocks=int(kmax),
                                       remote_capacity=int(cap))
    assert torch.equal(r.remote_indices.cpu(), o.remote_indices)


def test_router_scores_match_oracle():
    for name, n in (("pr1", 512), ("8b", 256), ("70b", 128)):
        wl = configs.CONFIGS[name]
        w = configs.make_weights(wl)
        x2d = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:n].contiguous()
        ref = oracle.router_scores(x2d, w.q_proj_16d, w.block_keys_16d)
        s, q16 = fsi.kernels.router_scores(x2d.to(DEV, wl.torch_dtype), w.q_proj_16d.to(DEV, wl.torch_dtype),
                                           w.block_keys_16d.to(DEV, wl.torch_dtype), want_q16=True)
        assert rel_err(s, ref) < 1e-5, name
        qref = torch.nn.functional.rms_norm(x2d @ w.q_proj_16d.t(), (16,))
        assert rel_err(q16, qref) < 1e-5, name


# ------------------------------------------------------------------ token mode vs golden
def token_vs_golden(wl, w, x2d, g, prefix, n_out, label=None):
    m = module_for(wl, w)
    y, info = run_token(m, x2d)
    bad, ties = compare_routes(info["remote_indices"].cpu(), info["remote_counts"].cpu(),
                               g[f"{prefix}remote_indices"], g[f"{prefix}remote_counts"], g[f"{prefix}margins"],
                               label=label or f"{wl.name} golden ({x2d.shape[0]} tokens)")
    assert bad == 0, f"{bad} routes differ outside near ties ({ties} ties)"
    if n_out:
        check_y(y[:n_out].cpu(), torch.from_numpy(g[f"{prefix}y"]), wl.dtype)
    device_error_is_clear()
    return y, info


def test_token_pr1_fp32():
    wl = configs.CONFIGS["pr1"]
    w, x = configs.make_weights(wl), configs.make_x(wl)
    token_vs_golden(wl, w, x.reshape(-1, wl.hidden_dim), golden("pr1"), "tok_", 512)


@pytest.mark.parametrize("k", [8, 16, 32])
def test_token_decode(k):
    wl = [p for p in configs.decode_points() if p.max_remote_blocks == k][0]
    w, x = configs.make_weights(wl), configs.make_x(wl)
    token_vs_golden(wl, w, x.reshape(-1, wl.hidden_dim), golden("decode"), f"k{k}_", 64)


def test_token_8b_slice():
    wl = configs.CONFIGS["8b"]
    w = configs.make_weights(wl)
    xs = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:128].contiguous()
    token_vs_golden(wl, w, xs, golden("8b_slice"), "tok_", 16)


def test_token_70b_slice():
    wl = configs.CONFIGS["70b"]
    w = configs.make_weights(wl)
    xs = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:64].contiguous()
    token_vs_golden(wl, w, xs, golden("70b_slice"), "tok_", 4)


def test_token_sweep_slice():
    g = golden("sweep_slice")
    pts = configs.sweep_points()
    w = configs.make_weights(pts[0])
    xs = configs.make_x(pts[0]).reshape(-1, pts[0].hidden_dim)[:64].contiguous()
    for i, wl in enumerate(pts):
        n_out = g[f"p{i}_y"].shape[0] if f"p{i}_y" in g else 0
        token_vs_golden(wl, w, xs, g, f"p{i}_", n_out, label=f"sweep top_p {wl.top_p} K_max {wl.max_remote_blocks}")


# ------------------------------------------------------------------ pooled mode vs golden
@pytest.mark.parametrize("training", [False, True])
def test_pooled_pr1(training):
    wl = configs.CONFIGS["pr1"]
    g = golden("pr1")
    w, x = configs.make_weights(wl), configs.make_x(wl)
    m = module_for(wl, w, routing="pooled")
    m.train(training)
    with torch.no_grad():
        y, info = m(x.to(DEV), return_router_info=True)
    p = "ptrain_" if training else "peval_"
    assert set(info["active_blocks"].cpu().tolist()) == set(g[f"{p}active_blocks"].tolist())
    check_y(y.reshape(-1, wl.hidden_dim).cpu(), torch.from_numpy(g[f"{p}y"]), "fp32")


def test_pooled_decode_and_cache():
    wl = configs.decode_points()[1]
    g = golden("decode")
    w, x = configs.make_weights(wl), configs.make_x(wl)
    m = module_for(wl, w, routing="pooled", remote_blocks=16)
    with torch.no_grad():
        y, info = m(x.to(DEV), return_router_info=True)
        assert set(info["active_blocks"].cpu().tolist()) == set(g["peval_active_blocks"].tolist())
        check_y(y.reshape(-1, wl.hidden_dim).cpu(), torch.from_numpy(g["peval_y"]), "bf16")
        y2 = m(x.to(DEV))  # cache hit (decode fast path): same active set, same result
    assert torch.equal(y, y2)


def test_pooled_8b_slice():
    wl = configs.CONFIGS["8b"]
    g = golden("8b_slice")
    w = configs.make_weights(wl)
    xs = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:128].contiguous()
    m = module_for(wl, w, routing="pooled", remote_blocks=20)
    with torch.no_grad():
        y, info = m(xs.view(1, 128, -1).to(DEV), return_router_info=True)
    assert set(info["active_blocks"].cpu().tolist()) == set(g["peval_active_blocks"].tolist())
    check_y(y.reshape(-1, wl.hidden_dim)[:16].cpu(), torch.from_numpy(g["peval_y"]), "bf16")


# ------------------------------------------------------------------ full-size configurations
def full_size_check(name, n_out):
    """All tokens: routes vs the oracle; a token subsample: outputs vs the oracle."""
    wl = configs.CONFIGS[name]
    w = configs.make_weights(wl)
    x2d = configs.make_x(wl).reshape(-1, wl.hidden_dim)
    m = module_for(wl, w)
    y, info = run_token(m, x2d)
    S = oracle.router_scores(x2d, w.q_proj_16d, w.block_keys_16d) / wl.temperature
    r = oracle.select_blocks_noncausal(S[None], local_window_blocks=wl.base_blocks, top_p=wl.top_p,
                                       min_remote_blocks=wl.min_remote_blocks,
                                       max_remote_blocks=wl.max_remote_blocks,
                                       remote_capacity=wl.max_remote_blocks)
    idx, cnt = r.remote_indices[0], r.remote_counts[0]
    margins = oracle.boundary_margins(r.remote_probs_sorted[0], cnt)
    bad, ties = compare_routes(info["remote_indices"].cpu(), info["remote_counts"].cpu(), idx, cnt, margins,
                               label=f"{name} full ({x2d.shape[0]} tokens)", count_margins=r.count_margins[0])
    assert bad == 0, f"{bad} of {x2d.shape[0]} routes differ outside near ties ({ties} ties)"
    sel = torch.randperm(x2d.shape[0], generator=torch.Generator().manual_seed(7))[:n_out].sort().values
    ref = oracle.token_pattention(x2d[sel], w.k_gate, w.k_up, w.v, wl.base_blocks, idx[sel], cnt[sel])
    ref = ref + oracle.additive_stream(S[sel], w.block_keys_16d, w.out_proj_16d)
    check_y(y[sel.to(DEV)].cpu(), ref, wl.dtype)
    device_error_is_clear()
    return y


def test_full_8b_config():
    y = full_size_check("8b", 128)
    assert torch.isfinite(y).all()


def test_full_sweep_routes():
    """Every token of the sweep workload (16384 tokens, 8B shape) at all 20 (top_p, K_max) points: routes
    against the oracle, with the tie accounting of each point recorded."""
    pts = configs.sweep_points()
    w = configs.make_weights(pts[0])
    x2d = configs.make_x(pts[0]).reshape(-1, pts[0].hidden_dim)
    S = oracle.router_scores(x2d, w.q_proj_16d, w.block_keys_16d)
    for wl in pts:
        m = module_for(wl, w)
        _, info = run_token(m, x2d)
        r = oracle.select_blocks_noncausal(S[None] / wl.temperature, local_window_blocks=wl.base_blocks,
                                           top_p=wl.top_p, min_remote_blocks=wl.min_remote_blocks,
                                           max_remote_blocks=wl.max_remote_blocks,
                                           remote_capacity=wl.max_remote_blocks)
        idx, cnt = r.remote_indices[0], r.remote_counts[0]
        margins = oracle.boundary_margins(r.remote_probs_sorted[0], cnt)
        bad, ties = compare_routes(info["remote_indices"].cpu(), info["remote_counts"].cpu(), idx, cnt, margins,
                                   label=f"sweep full top_p {wl.top_p} K_max {wl.max_remote_blocks}",
                                   count_margins=r.count_margins[0])
        assert bad == 0, f"top_p {wl.top_p} K_max {wl.max_remote_blocks}: {bad} routes differ ({ties} near ties)"
    device_error_is_clear()


def test_bit_equal_ties_go_to_lower_block_ids():
    """Bit-equal probabilities at the selection boundary: the lower block id wins (stable descending
    order), in both selection kernels.

    * ``fp_select_blocks`` on scores quantised to multiples of 1/4 (many exactly equal scores per row).
    * The fused routing kernel of the token forward with block keys repeated in groups of three (every
      block of a group scores bit-identically for every token), so that most tokens' K_max boundary falls
      inside a group.
    Every token must match the oracle's stable-sort route; the test also requires that bit-equal ties
    were actually exercised."""
    g = torch.Generator().manual_seed(11)
    s = (torch.randn(1, 512, 96, generator=g) * 4).round() / 4
    r = fsi.select_blocks(s.to(DEV), causal=False, local_window_blocks=3, top_p=0.9, min_remote_blocks=2,
                          max_remote_blocks=12, remote_capacity=12)
    o = oracle.select_blocks_noncausal(s, local_window_blocks=3, top_p=0.9, min_remote_blocks=2,
                                       max_remote_blocks=12, remote_capacity=12)
    mg = oracle.boundary_margins(o.remote_probs_sorted[0], o.remote_counts[0])
    bad, _ = compare_routes(r.remote_indices[0].cpu(), r.remote_counts[0].cpu(), o.remote_indices[0],
                            o.remote_counts[0], mg, label="exact ties: fp_select_blocks (quantised scores)",
                            strict_exact=True)
    assert bad == 0
    assert int((mg == 0).sum()) > 100, "the case must exercise bit-equal ties"

    wl = configs.CONFIGS["8b"].with_(name="ties", hidden_dim=512, intermediate_dim=2048, base_blocks=2,
                                     max_remote_blocks=8, min_remote_blocks=2, top_p=0.95)
    w = configs.make_weights(wl)
    grp = torch.arange(wl.num_blocks) // 3 * 3
    w = dataclasses.replace(w, block_keys_16d=w.block_keys_16d[grp].contiguous() * 8)  # groups of 3 identical keys
    x2d = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:1024].contiguous()
    ref = oracle.token_forward(x2d, w, base_blocks=wl.base_blocks, top_p=wl.top_p,
                               min_remote_blocks=wl.min_remote_blocks, max_remote_blocks=wl.max_remote_blocks)
    sp = ref["sorted_probs"]
    mg = oracle.boundary_margins(sp, ref["remote_counts"])
    m = module_for(wl, w)
    y, info = run_token(m, x2d)
    bad, _ = compare_routes(info["remote_indices"].cpu(), info["remote_counts"].cpu(), ref["remote_indices"],
                            ref["remote_counts"], mg, label="exact ties: fused routing kernel (repeated keys)",
                            strict_exact=True)
    assert bad == 0
    assert int((mg == 0).sum()) > 100, "the case must exercise bit-equal ties"
    check_y(y.cpu(), ref["y"].reshape(x2d.shape[0], -1), "bf16")
    device_error_is_clear()


def test_full_70b_config():
    full_size_check("70b", 32)


@pytest.mark.parametrize("M", [300, 1000, 2500])
def test_mid_token_counts(M):
    """Token counts between decode and the full batch: split-K down projection (300 tokens: 48 output
    tiles, 3 splits summed in a fixed order) and one or more partial waves of tiles (1000, 2500).  Outputs
    on a token sample match the oracle, and repeated calls are bitwise identical."""
    wl = configs.CONFIGS["8b"]
    w = configs.make_weights(wl)
    x2d = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:M].contiguous()
    m = module_for(wl, w)
    y, info = run_token(m, x2d)
    y2, _ = run_token(m, x2d)
    assert torch.equal(y, y2)
    idx, cnt = info["remote_indices"].cpu(), info["remote_counts"].cpu()
    sel = torch.linspace(0, M - 1, 24).long()
    S = oracle.router_scores(x2d[sel], w.q_proj_16d, w.block_keys_16d) / wl.temperature
    ref = oracle.token_pattention(x2d[sel], w.k_gate, w.k_up, w.v, wl.base_blocks, idx[sel], cnt[sel])
    ref = ref + oracle.additive_stream(S, w.block_keys_16d, w.out_proj_16d)
    check_y(y[sel.to(DEV)].cpu(), ref, wl.dtype)
    device_error_is_clear()


def test_block_shards_sum_to_full():
    """Parameter-block sharding arithmetic on one GPU: the fp32 partials of stride-2 shards (additive
    stream on shard 0 only) sum to the unsharded forward."""
    wl = configs.CONFIGS["8b"]
    w = configs.make_weights(wl)
    x2d = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:1000].contiguous().to(DEV, torch.bfloat16)
    m = module_for(wl, w)
    kg, ku, v, packed, wq, k16, wout = m._weights()
    kw = dict(base_blocks=wl.base_blocks, top_p=wl.top_p, min_remote=wl.min_remote_blocks,
              max_remote=wl.max_remote_blocks)
    full, _, _, _ = fsi.kernels.token_forward(x2d, kg, ku, v, packed, wq, k16, wout, out_f32=True, **kw)
    parts = [fsi.kernels.token_forward(x2d, kg, ku, v, packed, wq, k16, wout, out_f32=True, block_stride=4,
                                       block_offset=r, additive=(r == 0), **kw)[0] for r in range(4)]
    assert rel_err(sum(parts).cpu(), full.cpu()) < 1e-5


@pytest.mark.parametrize("M", [1, 5, 40, 64])
def test_decode_sizes_split_and_shards(M):
    """Batches of at most 64 tokens at the 8B shape: each gate/up tile's contraction is split over D in
    four work units summed in split order by the last to arrive, and the down projection contracts over
    the touched blocks only.  Outputs match the oracle, repeated calls are bitwise identical (the split
    sum does not depend on arrival order), and stride-4 block shards sum to the unsharded forward."""
    wl = configs.CONFIGS["8b"]
    w = configs.make_weights(wl)
    x2d = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:M].contiguous()
    m = module_for(wl, w)
    y, info = run_token(m, x2d)
    y2, _ = run_token(m, x2d)
    assert torch.equal(y, y2)
    idx, cnt = info["remote_indices"].cpu(), info["remote_counts"].cpu()
    S = oracle.router_scores(x2d, w.q_proj_16d, w.block_keys_16d) / wl.temperature
    ref = oracle.token_pattention(x2d, w.k_gate, w.k_up, w.v, wl.base_blocks, idx, cnt)
    ref = ref + oracle.additive_stream(S, w.block_keys_16d, w.out_proj_16d)
    check_y(y.cpu(), ref, wl.dtype)
    kg, ku, v, packed, wq, k16, wout = m._weights()
    kw = dict(base_blocks=wl.base_blocks, top_p=wl.top_p, min_remote=wl.min_remote_blocks,
              max_remote=wl.max_remote_blocks)
    xd = x2d.to(DEV, torch.bfloat16)
    full, _, _, _ = fsi.kernels.token_forward(xd, kg, ku, v, packed, wq, k16, wout, out_f32=True, **kw)
    parts = [fsi.kernels.token_forward(xd, kg, ku, v, packed, wq, k16, wout, out_f32=True, block_stride=4,
                                       block_offset=r, additive=(r == 0), **kw)[0] for r in range(4)]
    assert rel_err(sum(parts).cpu(), full.cpu()) < 1e-5
    device_error_is_clear()


@pytest.mark.parametrize("M", [2048, 1000])
def test_peer_output_single_rank(M):
    """The peer-memory reduce-scatter's kernels on one GPU (a job of one rank): the contraction stores its
    rows into the rank's own receive slot (2048 rows: TMA tile stores from the pair kernel's epilogue; 1000
    rows, not a multiple of 32: plain stores), the flag kernel raises the rank's flag and the combine
    waits for it and copies the slot out.  Equal bit for bit to the routed forward writing y directly, over
    two calls (both receive parities).  Decode-size batches decline (split contraction)."""
    wl = configs.CONFIGS["8b"]
    w = configs.make_weights(wl)
    x2d = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:M].contiguous().to(DEV, torch.bfloat16)
    m = module_for(wl, w)
    kg, ku, v, packed, wq, k16, wout = m._weights()
    kw = dict(base_blocks=wl.base_blocks, top_p=wl.top_p, min_remote=wl.min_remote_blocks,
              max_remote=wl.max_remote_blocks)
    ridx, cnt, ctx = fsi.kernels.route_tokens(x2d, wq, k16, **kw)
    ref = fsi.kernels.routed_forward(x2d, kg, ku, v, packed, wout, ridx, cnt, ctx, base_blocks=wl.base_blocks)
    D = wl.hidden_dim
    slot = M * D * 2
    base, _ = fsi.kernels.peer_alloc(fsi.kernels.PEER_FLAG_BYTES + 2 * slot)
    err_ws = torch.zeros(256, dtype=torch.uint8, device=DEV)
    try:
        for epoch in (1, 2):
            recv = base + fsi.kernels.PEER_FLAG_BYTES + (epoch & 1) * slot
            ok = fsi.kernels.routed_peer_forward(x2d, kg, ku, v, packed, wout, ridx, cnt, ctx,
                                                 base_blocks=wl.base_blocks, block_stride=1, block_offset=0,
                                                 peer_out=[recv], peer_flags=[base], rows_per_rank=M, epoch=epoch)
            assert ok
            y = fsi.kernels.peer_combine(recv, base, 1, M, D, in_f32=False, epoch=epoch, out_dtype=torch.bfloat16,
                                         err_ws=err_ws)
            torch.cuda.synchronize()
            assert torch.equal(y, ref), epoch
            assert fsi._lib.device_error(err_ws) == 0
        xs = x2d[:64].contiguous()
        r2, c2, x2 = fsi.kernels.route_tokens(xs, wq, k16, **kw)
        assert not fsi.kernels.routed_peer_forward(xs, kg, ku, v, packed, wout, r2, c2, x2,
                                                   base_blocks=wl.base_blocks, block_stride=1, block_offset=0,
                                                   peer_out=[base + fsi.kernels.PEER_FLAG_BYTES], peer_flags=[base],
                                                   rows_per_rank=64, epoch=3)
    finally:
        torch.cuda.synchronize()
        fsi.kernels.peer_free(base)
    device_error_is_clear()


def test_split_routing_entry_points():
    """The token-routed forward split in two (fp_route_tokens, then fp_pattention_routed_fwd from the given
    routes): the routes equal the fused forward's, four stride-4 shards from the given routes (additive
    stream from shard 0's context rows only) sum to the fused forward, and one unsharded call equals it."""
    wl = configs.CONFIGS["8b"]
    w = configs.make_weights(wl)
    x2d = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:1000].contiguous().to(DEV, torch.bfloat16)
    m = module_for(wl, w)
    kg, ku, v, packed, wq, k16, wout = m._weights()
    kw = dict(base_blocks=wl.base_blocks, top_p=wl.top_p, min_remote=wl.min_remote_blocks,
              max_remote=wl.max_remote_blocks)
    full, ridx0, cnt0, _ = fsi.kernels.token_forward(x2d, kg, ku, v, packed, wq, k16, wout, out_f32=True,
                                                     want_routes=True, **kw)
    ridx, cnt, ctx = fsi.kernels.route_tokens(x2d, wq, k16, **kw)
    assert torch.equal(cnt, cnt0)
    bad, _ = compare_routes(ridx.cpu(), cnt.cpu(), ridx0.cpu(), cnt0.cpu())
    assert bad == 0
    one = fsi.kernels.routed_forward(x2d, kg, ku, v, packed, wout, ridx, cnt, ctx, base_blocks=wl.base_blocks,
                                     out_f32=True)
    assert rel_err(one.cpu(), full.cpu()) < 1e-6
    zero = torch.zeros_like(ctx)
    parts = [fsi.kernels.routed_forward(x2d, kg, ku, v, packed, wout, ridx, cnt, ctx if r == 0 else zero,
                                        base_blocks=wl.base_blocks, block_stride=4, block_offset=r, out_f32=True)
             for r in range(4)]
    assert rel_err(sum(parts).cpu(), full.cpu()) < 1e-5
    device_error_is_clear()


def test_all_blocks_active_equals_dense():
    wl = configs.CONFIGS["8b"].with_(hidden_dim=1024, intermediate_dim=2048)
    w = configs.make_weights(wl)
    x2d = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:300].contiguous()
    m = module_for(wl, w, routing="pooled", remote_blocks=wl.num_blocks - wl.base_blocks)
    active = torch.arange(wl.num_blocks, dtype=torch.int32, device=DEV)
    kg, ku, v, packed, *_ = m._weights()
    y = fsi.kernels.pooled_forward(x2d.to(DEV, torch.bfloat16), kg, ku, v, packed, active)
    check_y(y.cpu(), oracle.dense_swiglu(x2d, w), "bf16")


def test_forward_host_matches_forward():
    """Chunked host-buffer forward (copies overlapped with compute) equals the device forward."""
    wl = configs.CONFIGS["8b"]
    w = configs.make_weights(wl)
    x2d = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:5000].contiguous().to(torch.bfloat16)
    m = module_for(wl, w)
    xh = x2d.pin_memory()
    with torch.no_grad():
        ref = m(x2d.to(DEV))
        ys = [m.forward_host(xh, chunk_tokens=c) for c in (1024, 4096)]  # 9 and 3 chunks, 2 compute streams
        # two pipelined batches in flight at once (the second's copy-in overlaps the first's last chunks)
        xa, xb = x2d[:2500].contiguous().pin_memory(), x2d[2500:].contiguous().pin_memory()
        oa, da = m.forward_host_async(xa, chunk_tokens=1024)
        ob, db = m.forward_host_async(xb, chunk_tokens=1024)
        da.synchronize()
        db.synchronize()
        ys.append(torch.cat([oa, ob]))
    torch.cuda.synchronize()
    for y in ys:
        assert y.device.type == "cpu" and y.shape == ref.shape
        assert rel_err(y.float(), ref.float().cpu()) < 1e-3


# ------------------------------------------------------------------ offline router calibration
def test_block_energy_kernel_matches_reference():
    """Teacher block energies of the calibration on the gate/up tensor-core kernel (fp32 epilogue
    reduction) against the reference's dense SwiGLU energies."""
    g = golden("calib")
    wl = configs.calib_workload()
    w, x = configs.make_weights(wl), configs.make_x(wl)
    m = module_for(wl, w)
    E = m._teacher_block_energy(x.reshape(-1, wl.hidden_dim).to(DEV).float())
    ref = torch.from_numpy(g["teacher"])
    assert rel_err(E.cpu(), ref) < 1e-5 and max_rel(E.cpu(), ref) < 1e-4


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_calibrate_offline_svd_matches_reference(dtype):
    """FovealPattentionMLP.calibrate_offline_svd on the GPU against the reference's run: explained
    variance, initial KL, the calibrated router's scores (invariant to singular-vector signs) and the
    calibrated active set; bf16 modules store the calibrated router in bf16."""
    g = golden("calib")
    base_wl = configs.calib_workload()  # bf16-rounded values, also held exactly by the fp32 module
    wl = base_wl.with_(dtype=dtype)
    w, x = configs.make_weights(base_wl), configs.make_x(base_wl)
    m = module_for(wl, w, routing="pooled", remote_blocks=g.meta["remote_blocks"])
    x2d = x.reshape(-1, wl.hidden_dim)
    info = m.calibrate_offline_svd(x2d.to(DEV), ridge_lambda=g.meta["ridge_lambda"])
    assert abs(info["top16_explained_variance"] - float(g["explained"])) <= 1e-4 * float(g["explained"])
    assert abs(info["initial_kl_divergence"] - float(g["kl"])) <= 1e-3 * float(g["kl"])
    S = oracle.router_scores(x2d, m.q_proj_16d.weight.detach().float().cpu(), m.block_keys_16d.detach().float().cpu())
    # the fitted keys are ill-conditioned at this weight scale (near-uniform teacher targets, scores
    # ~1e-4), so fp32 GPU (cuSOLVER SVD, cuBLAS) and CPU runs agree to ~4e-4 relative
    assert rel_err(S, torch.from_numpy(g["scores"])) < (2e-2 if dtype == "bf16" else 2e-3)
    assert active_set_matches(info["calib_active_blocks"], g["scores"], g.meta["base_blocks"],
                              g.meta["remote_blocks"], 1e-3)
    assert m._cached_active_blocks.tolist() == info["calib_active_blocks"]


# ------------------------------------------------------------------ training (pooled routing) backward
@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_training_backward_matches_reference(dtype):
    """Training-mode forward on the kernels and its backward (fused SwiGLU backward kernel, GEMMs over the
    active rows, additive-stream / router chain rule) against the reference module's autograd."""
    g = golden("train")
    base_wl = configs.train_workload()
    wl = base_wl.with_(dtype=dtype)
    w, x = configs.make_weights(base_wl), configs.make_x(base_wl)
    m = module_for(wl, w, routing="pooled", remote_blocks=base_wl.max_remote_blocks).train()
    xg = x.to(DEV, wl.torch_dtype).requires_grad_(True)
    y, info = m(xg, return_router_info=True)
    assert torch.equal(info["active_blocks"].cpu().to(torch.int32), torch.from_numpy(g["active"]))
    (y.float() * torch.from_numpy(g["dy"]).to(DEV)).sum().backward()
    tol = 1e-4 if dtype == "fp32" else 3e-2
    assert rel_err(y.float().cpu(), torch.from_numpy(g["y"])) < tol
    got = {"x": xg.grad, "k_gate": m.k_gate.grad, "k_up": m.k_up.grad, "v": m.v.grad,
           "q_proj_16d": m.q_proj_16d.weight.grad, "block_keys_16d": m.block_keys_16d.grad,
           "out_proj_16d": m.out_proj_16d.weight.grad}
    for name, t in got.items():
        assert t is not None, name
        assert rel_err(t.float().cpu(), torch.from_numpy(g[f"grad_{name}"])) < tol, name


# ------------------------------------------------------------------ whole-model serving
@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_sparsified_model_prefill_and_decode(dtype):
    """Model surgery + decode serving (foveal_pattention.py:355-387; eval cache :278-288, :309-325): a tiny
    Llama whose MLPs are replaced by ``sparsify_model_with_foveal_pattention``, prefilled on a 48-token
    prompt (each layer routes once on its pooled query and caches the active set) and decoded for 8 steps
    on the reference's tokens, against the reference's own run of the same model."""
    g = golden("serve")
    cfgd = g.meta
    tdt = torch.float32 if dtype == "fp32" else torch.bfloat16
    m = serve_model(cfgd)
    fsi.sparsify_model_with_foveal_pattention(m, base_blocks=cfgd["base_blocks"], remote_blocks=cfgd["remote_blocks"])
    m = m.to(DEV, tdt).eval()
    tol = 1e-3 if dtype == "fp32" else 8e-2
    with torch.no_grad():
        out = m(torch.from_numpy(g["prompt"]).to(DEV), use_cache=True)
        assert rel_err(out.logits[0].float().cpu(), torch.from_numpy(g["prefill_logits"])) < tol
        for layer, ref_active in zip(m.model.layers, g["active"]):
            assert set(layer.mlp._cached_active_blocks.tolist()) == set(ref_active.tolist())
        past = out.past_key_values
        for i, tok in enumerate(g["decode_tokens"].tolist()):
            o = m(torch.tensor([[tok]], device=DEV), past_key_values=past, use_cache=True)
            past = o.past_key_values
            lg = o.logits[0, -1].float().cpu()
            assert rel_err(lg, torch.from_numpy(g["decode_logits"][i])) < tol, i
            if dtype == "fp32":
                assert int(lg.argmax()) == int(g["decode_logits"][i].argmax())


# ------------------------------------------------------------------ edge cases
@pytest.mark.parametrize("M", [1, 7, 129, 300])
def test_ragged_token_counts(M):
    wl = configs.CONFIGS["8b"].with_(hidden_dim=512, intermediate_dim=1024, base_blocks=2,
                                     max_remote_blocks=5, min_remote_blocks=2)
    w = configs.make_weights(wl)
    x2d = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:M].contiguous()
    m = module_for(wl, w)
    y, info = run_token(m, x2d)
    ref = oracle.token_forward(x2d, w, base_blocks=wl.base_blocks, top_p=wl.top_p,
                               min_remote_blocks=wl.min_remote_blocks, max_remote_blocks=wl.max_remote_blocks)
    bad, _ = compare_routes(info["remote_indices"].cpu(), info["remote_counts"].cpu(), ref["remote_indices"],
                            ref["remote_counts"], oracle.boundary_margins(ref["sorted_probs"], ref["remote_counts"]))
    assert bad == 0
    check_y(y.cpu(), ref["y"].reshape(M, -1), "bf16")


def test_no_base_blocks_and_capacity_past_available():
    """base=0, and K_max larger than the number of remote blocks (counts clamp to `available`)."""
    for base, kmax in ((0, 6), (3, 40)):
        wl = configs.CONFIGS["8b"].with_(hidden_dim=256, intermediate_dim=2048, base_blocks=base,
                                         max_remote_blocks=kmax, min_remote_blocks=2, top_p=0.95)
        w = configs.make_weights(wl)
        x2d = configs.make_x(wl).reshape(-1, wl.hidden_dim)[:200].contiguous()
        m = module_for(wl, w)
        y, info = run_token(m, x2d)
        ref = oracle.token_forward(x2d, w, base_blocks=base, top_p=wl.top_p, min_remote_blocks=2,
                                   max_remote_blocks=kmax)
        mg = oracle.boundary_margins(ref["sorted_probs"], ref["remote_counts"])
        bad, _ = compare_routes(info["remote_indices"].cpu(), info["remote_counts"].cpu(), ref["remote_indices"],
                                ref["remote_counts"], mg)
        assert bad == 0
        assert int(info["remote_counts"].max()) <= min(kmax, wl.num_blocks - base)
        check_y(y.cpu(), ref["y"].reshape(200, -1), "bf16")


def test_empty_input():
    wl = configs.CONFIGS["pr1"]
    w = configs.make_weights(wl)
    m = module_for(wl, w)
    with torch.no_grad():
        y = m(torch.zeros(0, wl.hidden_dim, device=DEV))
    assert y.shape == (0, wl.hidden_dim)


# ------------------------------------------------------------------ reference API behaviour
class _DenseMLP(torch.nn.Module):
    def __init__(self, hidden_dim=256, intermediate_dim=512):
        super().__init__()
        self.gate_proj = torch.nn.Linear(hidden_dim, intermediate_dim, bias=False)
        self.up_proj = torch.nn.Linear(hidden_dim, intermediate_dim, bias=False)
        self.down_proj = torch.nn.Linear(intermediate_dim, hidden_dim, bias=False)


def test_reference_module_tests_on_gpu():
    """tests/test_foveal_pattention.py:27-44, :69-96 and :99-124 of the reference, on the GPU."""
    torch.manual_seed(0)
    dense = _DenseMLP().to(DEV)
    patt = fsi.FovealPattentionMLP.from_dense_mlp(dense, block_size=64, base_blocks=2, remote_blocks=4)
    assert patt.num_blocks == 8 and patt.total_active_blocks == 6
    x = torch.randn(2, 16, 256, device=DEV)
    patt.train()
    out, info = patt(x, return_router_info=True)
    assert out.shape == (2, 16, 256) and "scores" in info and "active_blocks" in info
    out.sum().backward()  # the reference's gradient check (:86-92)
    assert patt.q_proj_16d.weight.grad is not None and patt.block_keys_16d.grad is not None
    assert patt.out_proj_16d.weight.grad is not None
    patt0 = fsi.FovealPattentionMLP.from_dense_mlp(dense, block_size=64, base_blocks=0, remote_blocks=4).eval()
    with torch.no_grad():
        out, info = patt0(x, return_router_info=True)
        assert out.shape == (2, 16, 256) and len(info["active_blocks"]) == 4
        patt0.clear_cache()
        assert patt0(torch.randn(2, 1, 256, device=DEV)).shape == (2, 1, 256)
    # dense equivalence when every block is active (fp32, CUDA-core path)
    full = fsi.FovealPattentionMLP.from_dense_mlp(dense, block_size=64, base_blocks=8, remote_blocks=0).eval()
    with torch.no_grad():
        y = full(x)
        ref = dense.down_proj(torch.nn.functional.silu(dense.gate_proj(x)) * dense.up_proj(x))
    assert rel_err(y.cpu(), ref.cpu()) < 1e-5


def test_errors_are_loud():
    wl = configs.CONFIGS["pr1"]
    w = configs.make_weights(wl)
    m = module_for(wl, w)
    with pytest.raises(RuntimeError):
        m(torch.zeros(4, wl.hidden_dim))  # CPU input: no fallback
    with pytest.raises(fsi.FovealKernelError):
        fsi.kernels.select(torch.zeros(4, 2000, device=DEV), base_blocks=0, top_p=0.5, min_remote=0,
                           max_remote=4, capacity=4)  # NB > 1024 unsupported
    with pytest.raises(NotImplementedError):
        fsi.select_blocks(torch.zeros(1, 4, 8, device=DEV), causal=True)
