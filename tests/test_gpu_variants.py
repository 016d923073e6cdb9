"""GPU parity of the layers that share the router: BlockSparseLinear and FovealTokenformerLinear / FFN.

* the modules against the reference's own outputs (tests/golden/variants.npz): fp32 within 1e-4
  relative (CUDA-core path), bf16 within 2e-2 relative (tcgen05 path) of the fp32 reference run on the
  same bf16-rounded values; union sizes and routes exactly;
* the building blocks (pooled block keys, cosine scores, the inference selection rule, the union)
  against the CPU oracle on seeded inputs, including the edge cases: no remote columns, a count one
  past the available blocks, an empty union;
* the tensor-core contractions at larger, ragged shapes (token counts that are not multiples of the
  tile, output widths that are not multiples of 256, partial unions) against the oracle.
"""

from __future__ import annotations

import pytest
import torch

import oracle
from conftest import VARIANT_NAMES, compare_routes, fsi, golden, rel_err, tf_kwargs, variant_setup

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
TOL = {"fp32": 1e-4, "bf16": 2e-2}
DT = {"fp32": torch.float32, "bf16": torch.bfloat16}
kernels = fsi.kernels


def _module(name, dt):
    case, p, x = variant_setup(name, dt)
    cls = {"bsl": fsi.BlockSparseLinear, "tf": fsi.FovealTokenformerLinear,
           "ffn": fsi.FovealTokenformerFFN}[case["kind"]]
    m = cls(**fsi.configs.variant_kwargs(case))
    m.load_state_dict(p)
    m = m.to(DEV, DT[dt])
    return case, m, x.to(DEV, DT[dt]), p


@pytest.mark.parametrize("dt", ["fp32", "bf16"])
@pytest.mark.parametrize("name", VARIANT_NAMES)
def test_variant_module_matches_reference(name, dt):
    g = golden("variants")
    pre = f"{name}_{dt}_"
    case, m, x, _ = _module(name, dt)
    m.eval()
    with torch.no_grad():
        y, aux = m(x, compute_teacher_loss=(dt == "fp32"))
    torch.cuda.synchronize()
    assert rel_err(y.float().cpu(), torch.from_numpy(g[pre + "eval_out"])) < TOL[dt]
    if dt == "fp32":
        d_ref = float(g[pre + "distill"])
        assert abs(float(aux["distill_loss"]) - d_ref) <= 1e-4 * max(1.0, abs(d_ref))
    if case["kind"] == "bsl":
        assert aux["route"] is None
        assert aux["active_blocks_union"] == int(g[pre + "eval_union"])
        assert abs(aux["mean_active_blocks"] - float(g[pre + "eval_mean_active"])) < 1e-6
        m.train()
        with torch.no_grad():
            y, aux = m(x)
        assert rel_err(y.float().cpu(), torch.from_numpy(g[pre + "train_out"])) < TOL[dt]
        assert aux["active_blocks_union"] == int(g[pre + "train_union"])
        r = aux["route"]
        bad, _ = compare_routes(r.remote_indices.reshape(-1, r.remote_indices.shape[-1]).cpu(),
                                r.remote_counts.reshape(-1).cpu(),
                                g[pre + "train_idx"].reshape(-1, r.remote_indices.shape[-1]),
                                g[pre + "train_cnt"].reshape(-1))
        assert bad == 0
    elif case["kind"] == "tf":
        assert aux["active_param_tokens_union"] == int(g[pre + "eval_union"])
        assert abs(aux["mean_active_param_tokens"] - float(g[pre + "eval_mean_active"])) < 1e-3
        r = aux["route"]
        cap = r.remote_indices.shape[-1]
        bad, _ = compare_routes(r.remote_indices.reshape(-1, cap).cpu(), r.remote_counts.reshape(-1).cpu(),
                                g[pre + "eval_idx"].reshape(-1, cap), g[pre + "eval_cnt"].reshape(-1))
        assert bad == 0
    else:
        for f in ("fc1", "fc2"):
            assert aux[f + "_aux"]["active_param_tokens_union"] == int(g[f"{pre}{f}_union"])


@pytest.mark.parametrize("dt", ["fp32", "bf16"])
def test_block_keys_and_cosine_scores_kernels(dt):
    g = torch.Generator().manual_seed(5)
    P = torch.randn(640, 384, generator=g)
    wk, wv, wq = (torch.randn(16, 384, generator=g) * 384 ** -0.5 for _ in range(3))
    x = torch.randn(333, 384, generator=g)
    if dt == "bf16":
        P, wk, wv, wq, x = (t.to(torch.bfloat16).float() for t in (P, wk, wv, wq, x))
    kb_ref, vb_ref = oracle.param_blocks_16d(P, wk, wv)
    td = DT[dt]
    kb, vb = kernels.param_blocks_16d(P.to(DEV, td), wk.to(DEV, td), wv.to(DEV, td))
    assert rel_err(kb.cpu(), kb_ref) < 1e-5 and rel_err(vb.cpu(), vb_ref) < 1e-5
    s_ref = oracle.cosine_block_scores(x, wq, kb_ref)
    s, _ = kernels.cosine_block_scores(x.to(DEV, td), wq.to(DEV, td), kb_ref.to(DEV))
    assert rel_err(s.cpu(), s_ref) < 1e-5


@pytest.mark.parametrize("NB,base,top_p,kmax", [(48, 2, 0.2, 6), (40, 3, 0.9, 64), (9, 3, 1.5, 8), (5, 5, 0.5, 4),
                                                (200, 4, 0.6, 56)])
def test_inference_selection_and_union(NB, base, top_p, kmax):
    """select_remote_top_p and union_blocks against the oracle: a binding top-p, K_max above the available
    blocks, a target above 1 (count = available + 1, as in the reference), no remote column at all."""
    g = torch.Generator().manual_seed(NB)
    scores = torch.randn(257, NB, generator=g) * 3.0
    sd = scores.to(DEV)
    idx, cnt, stats = kernels.select_remote_top_p(sd, base_blocks=base, top_p=top_p, max_remote=kmax, want_stats=True)
    blocks, n_active = kernels.union_blocks(idx, cnt, NB, base)
    torch.cuda.synchronize()
    if NB > base:
        ref_idx, ref_cnt = oracle.fast_remote_route(scores, base, top_p, kmax)
        # the reference's count (block_matmul.py:190-193) is not clamped to the available blocks
        rem = torch.softmax(scores[:, base:], dim=-1).sort(dim=-1, descending=True, stable=True).values.cumsum(-1)
        ref_needed = ((rem < top_p).sum(-1) + 1).clamp(0, kmax)
        assert torch.equal(cnt.cpu().long(), ref_needed)
        bad, _ = compare_routes(idx.cpu().long(), cnt.cpu().clamp(max=idx.shape[1]), ref_idx,
                                ref_cnt.clamp(max=idx.shape[1]))
        assert bad == 0
        assert abs(float(stats[1]) - float(ref_needed.sum())) < 0.5
        ref_union = oracle.union_blocks(base, ref_idx, ref_cnt, NB)
    else:
        assert int(cnt.abs().sum()) == 0
        ref_union = torch.arange(NB, dtype=torch.int32)
    n = int(n_active)
    assert n == ref_union.numel()
    assert torch.equal(blocks[:n].cpu(), ref_union)
    rest = torch.tensor(sorted(set(range(NB)) - set(ref_union.tolist())), dtype=torch.int32)
    assert torch.equal(blocks[n:].cpu(), rest)


def _bsl_case(M, D_in, out_features, base, kmax, top_p, bias, dt, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, D_in, generator=g)
    W = torch.randn(out_features, D_in, generator=g) * D_in ** -0.5
    b = torch.randn(out_features, generator=g) * 0.05 if bias else None
    wq, wk, wv = (torch.randn(16, D_in, generator=g) * D_in ** -0.5 for _ in range(3))
    wo = torch.randn(out_features, 16, generator=g) * 0.05
    if dt == "bf16":
        x, W, wq, wk, wv, wo = (t.to(torch.bfloat16).float() for t in (x, W, wq, wk, wv, wo))
        b = b.to(torch.bfloat16).float() if b is not None else None
    return x, W, b, wq, wk, wv, wo


@pytest.mark.parametrize("M,D_in,out_features,kmax,top_p,bias", [
    (600, 1024, 4096, 8, 0.8, True),     # ragged token count, partial union
    (130, 512, 1536, 24, 0.95, False),   # output width not a multiple of 256
    (1, 256, 8192, 4, 0.5, True),        # one token: a sparse union (tensor path, most tiles skipped)
    (64, 1024, 4096, 8, 0.8, True),      # decode-sized batch: the contraction is split over D_in (split-K)
    (1, 1024, 14336, 8, 0.8, False),     # one token at the 8B width: a 10-block bound, split-K over 3 tiles
])
def test_block_sparse_linear_tensor_path(M, D_in, out_features, kmax, top_p, bias):
    x, W, b, wq, wk, wv, wo = _bsl_case(M, D_in, out_features, 2, kmax, top_p, bias, "bf16", M)
    ref, active, idx, cnt, _ = oracle.block_sparse_linear(
        x, W, b, wq, wk, wv, wo, block_size=64, base_blocks=2, top_p=top_p, min_remote_blocks=0,
        max_remote_blocks=kmax, remote_capacity=kmax, fast_rule=False)
    m = fsi.BlockSparseLinear(D_in, out_features, base_blocks=2, top_p=top_p, max_remote_blocks=kmax,
                              remote_capacity=kmax, bias=bias)
    sd = {"weight": W, "indexer.q_proj.weight": wq, "indexer.k_proj.weight": torch.zeros(16, D_in),
          "indexer.v_proj.weight": torch.zeros(16, D_in), "indexer.out_proj.weight": wo,
          "weight_to_k.weight": wk, "weight_to_v.weight": wv}
    if bias:
        sd["bias"] = b
    m.load_state_dict(sd)
    m = m.to(DEV, torch.bfloat16).train()
    with torch.no_grad():
        y, aux = m(x.to(DEV, torch.bfloat16))
    torch.cuda.synchronize()
    assert aux["active_blocks_union"] == active.numel()
    assert rel_err(y.float().cpu(), ref) < 2e-2
    # inactive columns hold the additive stream only
    if active.numel() < out_features // 64:
        mask = torch.ones(out_features // 64, dtype=torch.bool)
        mask[active.long()] = False
        cols = (mask.nonzero().view(-1, 1) * 64 + torch.arange(64)).flatten()
        assert rel_err(y.float().cpu()[:, cols], ref[:, cols]) < 2e-2


@pytest.mark.parametrize("M,D_in,out_features,nact", [
    (600, 1024, 4096, 40),   # two token tiles: CTA-pair kernel, runs of consecutive blocks and gaps
    (64, 1024, 14336, 200),  # decode-sized: one-SM kernel split over D_in, four-block runs as one box
    (1, 4096, 14336, 12),    # one token, a sparse union
    (300, 512, 1536, 24),    # every block, output width not a multiple of 256
])
def test_blocked_weight_matches_row_major(M, D_in, out_features, nact):
    """The blocked weight copy (fp_pack_blocked_weight) gives the row-major weight's results bit for bit
    (same k-block order and MMA shapes); the layout itself is checked tile by tile."""
    g = torch.Generator().manual_seed(M + nact)
    NB = out_features // 64
    W = (torch.randn(out_features, D_in, generator=g) * D_in ** -0.5).to(DEV, torch.bfloat16)
    x = torch.randn(M, D_in, generator=g).to(DEV, torch.bfloat16)
    b = (torch.randn(out_features, generator=g) * 0.05).to(DEV, torch.bfloat16)
    ctx = torch.randn(M, 16, generator=g).to(DEV)
    wo = (torch.randn(out_features, 16, generator=g) * 0.05).to(DEV, torch.bfloat16)
    act = torch.randperm(NB, generator=g)[:nact].sort().values
    rest = torch.tensor(sorted(set(range(NB)) - set(act.tolist())), dtype=torch.int64)
    blocks = torch.cat([act, rest]).int().to(DEV)
    n_active = torch.tensor([nact], dtype=torch.int32, device=DEV)
    Wb = kernels.pack_blocked_weight(W)
    tiles = Wb.view(D_in // 64, NB, 64, 64)
    for kb, j in ((0, 0), (D_in // 64 - 1, NB - 1), (1, NB // 2)):
        assert torch.equal(tiles[kb, j], W[j * 64:(j + 1) * 64, kb * 64:(kb + 1) * 64])
    ma = nact  # the host-side bound of the union: exact here
    y0 = kernels.block_sparse_linear(x, W, b, blocks, n_active, ctx, wo, max_active=ma)
    y1 = kernels.block_sparse_linear(x, W, b, blocks, n_active, ctx, wo, max_active=ma, weight_blocked=Wb)
    ref = x.float() @ W.float().t() + b.float() + ctx @ wo.float().t()
    inactive = torch.ones(NB, dtype=torch.bool)
    inactive[act] = False
    cols = (inactive.nonzero().view(-1, 1) * 64 + torch.arange(64)).flatten().to(DEV)
    ref[:, cols] = ctx @ wo.float()[cols].t()
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)
    assert rel_err(y1.float(), ref) < 2e-2


def test_module_blocked_weight_copy():
    """BlockSparseLinear.use_blocked_weight: eval-mode outputs equal the row-major weight's bit for bit, and
    the copy follows an in-place weight update."""
    x, W, b, wq, wk, wv, wo = _bsl_case(64, 1024, 4096, 2, 8, 0.8, True, "bf16", 64)
    m = fsi.BlockSparseLinear(1024, 4096, base_blocks=2, top_p=0.8, max_remote_blocks=8, remote_capacity=8, bias=True)
    sd = {"weight": W, "bias": b, "indexer.q_proj.weight": wq, "indexer.k_proj.weight": torch.zeros(16, 1024),
          "indexer.v_proj.weight": torch.zeros(16, 1024), "indexer.out_proj.weight": wo,
          "weight_to_k.weight": wk, "weight_to_v.weight": wv}
    m.load_state_dict(sd)
    m = m.to(DEV, torch.bfloat16).eval()
    xd = x.to(DEV, torch.bfloat16)
    with torch.no_grad():
        y0, _ = m(xd)
        m.use_blocked_weight(True)
        y1, _ = m(xd)
        assert m._blocked is not None
        assert torch.equal(y0, y1)
        m.weight.mul_(0.5)  # in-place update (version counter): the copy is rebuilt on the next call
        m.refresh_block_cache()
        y3, _ = m(xd)
        m.use_blocked_weight(False)
        y2, _ = m(xd)
    torch.cuda.synchronize()
    assert torch.equal(y2, y3) and not torch.equal(y1, y3)


@pytest.mark.parametrize("M,D_in,D_out,Np,kmax,activation", [
    (300, 512, 768, 4096, 8, "softmax"),
    (129, 256, 256, 2048, 16, "gelu_l2"),
    (2, 1024, 512, 8192, 4, "softmax"),
])
def test_tokenformer_tensor_path(M, D_in, D_out, Np, kmax, activation):
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, D_in, generator=g)
    kp = torch.randn(Np, D_in, generator=g) * D_in ** -0.5
    vp = torch.randn(Np, D_out, generator=g) * D_out ** -0.5
    wq, wk, wv = (torch.randn(16, D_in, generator=g) * D_in ** -0.5 for _ in range(3))
    wo = torch.randn(D_out, 16, generator=g) * 0.05
    x, kp, vp, wq, wk, wv, wo = (t.to(torch.bfloat16).float() for t in (x, kp, vp, wq, wk, wv, wo))
    ref, active, _, _, _ = oracle.tokenformer_linear(x, kp, vp, wq, wk, wv, wo, block_size=64, base_blocks=2, top_p=0.9,
                                                     min_remote_blocks=0, max_remote_blocks=kmax,
                                                     remote_capacity=kmax, activation=activation)
    m = fsi.FovealTokenformerLinear(D_in, D_out, num_param_tokens=Np, base_blocks=2, top_p=0.9,
                                    max_remote_blocks=kmax, remote_capacity=kmax, activation=activation)
    m.load_state_dict({"k_param": kp, "v_param": vp, "indexer.q_proj.weight": wq, "indexer.k_proj.weight": wk,
                       "indexer.v_proj.weight": wv, "indexer.out_proj.weight": wo})
    m = m.to(DEV, torch.bfloat16).eval()
    with torch.no_grad():
        y, aux = m(x.to(DEV, torch.bfloat16).unsqueeze(0))
    torch.cuda.synchronize()
    assert aux["active_param_tokens_union"] == active.numel() * 64
    assert rel_err(y[0].float().cpu(), ref) < 2e-2


@pytest.mark.parametrize("dt", ["fp32", "bf16"])
def test_empty_union(dt):
    """No base block and top_p = 0: no token selects anything.  The reference then attends over no
    parameter token (Tokenformer: zeros) / computes no output block (BlockSparseLinear: zeros), and the
    output is the additive stream alone."""
    td = DT[dt]
    g = torch.Generator().manual_seed(3)
    D_in, D_out, Np, M = 128, 256, 512, 70
    x = torch.randn(M, D_in, generator=g)
    kp = torch.randn(Np, D_in, generator=g) * D_in ** -0.5
    vp = torch.randn(Np, D_out, generator=g) * D_out ** -0.5
    wq, wk, wv = (torch.randn(16, D_in, generator=g) * D_in ** -0.5 for _ in range(3))
    wo = torch.randn(D_out, 16, generator=g) * 0.05
    if dt == "bf16":
        x, kp, vp, wq, wk, wv, wo = (t.to(torch.bfloat16).float() for t in (x, kp, vp, wq, wk, wv, wo))
    ref, active, _, _, _ = oracle.tokenformer_linear(x, kp, vp, wq, wk, wv, wo, block_size=64, base_blocks=0, top_p=0.0,
                                                     min_remote_blocks=0, max_remote_blocks=4, remote_capacity=4,
                                                     activation="softmax")
    assert active.numel() == 0
    m = fsi.FovealTokenformerLinear(D_in, D_out, num_param_tokens=Np, base_blocks=0, top_p=0.0)
    m.load_state_dict({"k_param": kp, "v_param": vp, "indexer.q_proj.weight": wq, "indexer.k_proj.weight": wk,
                       "indexer.v_proj.weight": wv, "indexer.out_proj.weight": wo})
    m = m.to(DEV, td).eval()
    with torch.no_grad():
        y, aux = m(x.to(DEV, td).unsqueeze(0))
    assert aux["active_param_tokens_union"] == 0
    assert rel_err(y[0].float().cpu(), ref) < TOL[dt]
    # BlockSparseLinear with the same router output: every column inactive
    W = torch.randn(Np, D_in, generator=g) * D_in ** -0.5
    if dt == "bf16":
        W = W.to(torch.bfloat16).float()
    wo_b = wo.repeat(2, 1)  # [Np, 16]: BlockSparseLinear's output width is Np here
    ref_b, active_b, _, _, _ = oracle.block_sparse_linear(x, W, None, wq, wk, wv, wo_b, block_size=64, base_blocks=0,
                                                         top_p=0.0, min_remote_blocks=0, max_remote_blocks=4,
                                                         remote_capacity=4, fast_rule=False)
    assert active_b.numel() == 0
    b = fsi.BlockSparseLinear(D_in, Np, base_blocks=0, top_p=0.0, max_remote_blocks=4, remote_capacity=4)
    b.load_state_dict({"weight": W, "indexer.q_proj.weight": wq, "indexer.k_proj.weight": wk,
                       "indexer.v_proj.weight": wv, "indexer.out_proj.weight": wo_b,
                       "weight_to_k.weight": wk, "weight_to_v.weight": wv})
    b = b.to(DEV, td).train()
    with torch.no_grad():
        yb, auxb = b(x.to(DEV, td))
    assert auxb["active_blocks_union"] == 0
    assert rel_err(yb.float().cpu(), ref_b) < TOL[dt]


def test_backward_raises():
    """The layers are forward-only: a training graph through them fails loudly."""
    m = fsi.FovealTokenformerLinear(64, 64, num_param_tokens=256).to(DEV).train()
    y, _ = m(torch.randn(1, 4, 64, device=DEV))
    with pytest.raises(NotImplementedError):
        y.sum().backward()


@pytest.mark.parametrize("activation", ["softmax", "gelu_l2"])
def test_bf16_cuda_core_fallback(activation):
    """bf16 layers whose widths the tensor-core path does not tile (D_in % 64 != 0) run on CUDA cores with
    fp32 scores in the workspace; same parity bar."""
    g = torch.Generator().manual_seed(11)
    M, D_in, D_out, Np = 37, 136, 200, 512
    x = torch.randn(M, D_in, generator=g)
    kp = torch.randn(Np, D_in, generator=g) * D_in ** -0.5
    vp = torch.randn(Np, D_out, generator=g) * D_out ** -0.5
    wq, wk, wv = (torch.randn(16, D_in, generator=g) * D_in ** -0.5 for _ in range(3))
    wo = torch.randn(D_out, 16, generator=g) * 0.05
    x, kp, vp, wq, wk, wv, wo = (t.to(torch.bfloat16).float() for t in (x, kp, vp, wq, wk, wv, wo))
    ref, active, _, _, _ = oracle.tokenformer_linear(x, kp, vp, wq, wk, wv, wo, block_size=64, base_blocks=1, top_p=0.9,
                                                     min_remote_blocks=0, max_remote_blocks=3, remote_capacity=3,
                                                     activation=activation)
    m = fsi.FovealTokenformerLinear(D_in, D_out, num_param_tokens=Np, base_blocks=1, top_p=0.9, max_remote_blocks=3,
                                    remote_capacity=3, activation=activation)
    m.load_state_dict({"k_param": kp, "v_param": vp, "indexer.q_proj.weight": wq, "indexer.k_proj.weight": wk,
                       "indexer.v_proj.weight": wv, "indexer.out_proj.weight": wo})
    m = m.to(DEV, torch.bfloat16).eval()
    with torch.no_grad():
        y, aux = m(x.to(DEV, torch.bfloat16).unsqueeze(0))
    assert aux["active_param_tokens_union"] == active.numel() * 64
    assert rel_err(y[0].float().cpu(), ref) < 2e-2
    # BlockSparseLinear with the same odd input width
    W = (torch.randn(Np, D_in, generator=g) * D_in ** -0.5).to(torch.bfloat16).float()
    wo_b = (torch.randn(Np, 16, generator=g) * 0.05).to(torch.bfloat16).float()
    ref_b, active_b, _, _, _ = oracle.block_sparse_linear(x, W, None, wq, wk, wv, wo_b, block_size=64, base_blocks=1,
                                                         top_p=0.9, min_remote_blocks=0, max_remote_blocks=3,
                                                         remote_capacity=3, fast_rule=True)
    b = fsi.BlockSparseLinear(D_in, Np, base_blocks=1, top_p=0.9, max_remote_blocks=3, remote_capacity=3)
    b.load_state_dict({"weight": W, "indexer.q_proj.weight": wq, "indexer.k_proj.weight": wk,
                       "indexer.v_proj.weight": wv, "indexer.out_proj.weight": wo_b,
                       "weight_to_k.weight": wk, "weight_to_v.weight": wv})
    b = b.to(DEV, torch.bfloat16).eval()
    with torch.no_grad():
        yb, auxb = b(x.to(DEV, torch.bfloat16))
    assert auxb["active_blocks_union"] == active_b.numel()
    assert rel_err(yb.float().cpu(), ref_b) < 2e-2
