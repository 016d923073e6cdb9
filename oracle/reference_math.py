"""CPU restatement of the reference's Foveal Pattention MLP forward (test infrastructure only).

Every function cites the reference file:line it restates.  All arithmetic is fp32 PyTorch on the CPU,
with the same operator sequence as the reference, so that on the same inputs the results match the
reference bit for bit where the reference is deterministic.  Two deliberate differences:

* ``select_blocks`` sorts with ``stable=True``.  The reference calls ``Tensor.sort`` with the default
  ``stable=False`` (core.py:107); a stable descending sort breaks probability ties toward the lower
  block id, which is the documented tie rule of the CUDA router.
* ``token_pattention`` accumulates the per-token output block by block (grouping tokens that share a
  block) instead of one gathered matmul per token (pattention_triton.py:280-311).  The sum is the same
  and only the fp32 summation order differs (relative differences ~1e-7).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch
import torch.nn.functional as F

__all__ = [
    "masked_softmax",
    "select_blocks_noncausal",
    "OracleRoute",
    "router_scores",
    "additive_stream",
    "token_pattention",
    "token_pattention_per_token",
    "token_forward",
    "pooled_eval_active",
    "pooled_train_active",
    "pooled_pattention",
    "pooled_forward",
    "boundary_margins",
    "dense_swiglu",
    "pattention",
    "PATTENTION_ACTIVATIONS",
    "teacher_block_energy",
    "calibrate_offline_svd",
    "param_blocks_16d",
    "cosine_block_scores",
    "union_blocks",
    "fast_remote_route",
    "fast_rule_counts",
    "block_sparse_linear",
    "tokenformer_linear",
]


def masked_softmax(scores: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """core.py:36-43 — fp32 softmax that zeroes masked entries; denominator clamped at 1e-20."""
    safe = scores.float().masked_fill(~mask, -float("inf"))
    row_max = safe.amax(dim=-1, keepdim=True)
    row_max = torch.where(torch.isfinite(row_max), row_max, torch.zeros_like(row_max))
    numer = torch.exp(safe - row_max) * mask
    denom = numer.sum(dim=-1, keepdim=True).clamp_min(1e-20)
    return (numer / denom).to(scores.dtype)


@dataclass
class OracleRoute:
    """Fields of the reference ``Route`` (core.py:23-33) for the non-causal branch."""

    remote_indices: torch.Tensor   # [B, Q, capacity] int32, sorted by descending probability
    remote_counts: torch.Tensor    # [B, Q] int32
    base_indices: Optional[torch.Tensor]
    base_counts: Optional[torch.Tensor]
    block_scores: torch.Tensor
    cap_rate: torch.Tensor
    mean_remote_blocks: torch.Tensor
    base_only_rate: torch.Tensor
    remote_probs_sorted: torch.Tensor  # [B, Q, NB] fp32, the sorted probabilities (for margins)
    # [B, Q] fp64: distance of the top-p target from the nearest cumulative mass that decides the count
    # (inf where the K_min / K_max clamps make the count insensitive to it); a tiny value marks a token
    # whose count depends on the last bits of its probabilities
    count_margins: Optional[torch.Tensor] = None


def select_blocks_noncausal(
    block_scores: torch.Tensor,
    *,
    local_window_blocks: int = 0,
    top_p: float = 0.95,
    min_remote_blocks: int = 0,
    max_remote_blocks: int = 16,
    remote_capacity: int = 16,
    stable: bool = True,
) -> OracleRoute:
    """core.py:46-160, non-causal branch (core.py:90-99), with base blocks [0, local_window_blocks).

    Steps (reference line numbers): softmax over all blocks (:101-102), base ("local") mass (:104),
    remote probabilities with base entries set to -1 (:105), descending sort (:107), clamp and
    fp32 cumulative sum (:108-109; torch's CPU cumsum accumulates in fp64 and rounds each prefix to
    fp32), ``needed = #(cum < target) + (target > 0)`` (:111-115), clamp to [K_min, min(avail, K_max)]
    (:116-119), first ``capacity`` sorted ids (:121-123), base ids (:137-140) and statistics
    (:145-159).
    """
    batch, query_blocks, total_blocks = block_scores.shape
    device = block_scores.device
    top_p_t = torch.as_tensor(top_p, device=device, dtype=torch.float32)
    min_remote_t = torch.as_tensor(min_remote_blocks, device=device, dtype=torch.int64)
    max_remote_t = torch.as_tensor(max_remote_blocks, device=device, dtype=torch.int64)
    pb = torch.arange(total_blocks, device=device)

    complete = torch.ones((query_blocks, total_blocks), dtype=torch.bool, device=device)
    if local_window_blocks > 0:
        local_complete = (pb.view(1, total_blocks) < local_window_blocks).expand(query_blocks, -1)
        remote = (pb.view(1, total_blocks) >= local_window_blocks).expand(query_blocks, -1)
    else:
        local_complete = torch.zeros_like(complete)
        remote = complete

    probs = masked_softmax(block_scores, complete[None].expand(batch, -1, -1))
    local_mass = (probs * local_complete[None]).sum(dim=-1)
    remote_probs = probs.masked_fill(~remote[None], -1.0)
    sorted_prob, sorted_idx = remote_probs.sort(dim=-1, descending=True, stable=stable)
    sorted_prob = sorted_prob.clamp_min(0.0)
    cumulative = sorted_prob.cumsum(dim=-1)

    target = (top_p_t - local_mass).clamp_min(0.0)
    available = remote.sum(dim=-1).view(1, query_blocks).expand(batch, -1)
    needed = (cumulative < target[..., None]).sum(dim=-1) + (target > 0).long()
    needed = torch.where(available > 0, needed, torch.zeros_like(needed))
    needed = torch.where(available > 0, torch.maximum(needed, min_remote_t), needed)
    counts = torch.minimum(needed, available)
    counts = torch.minimum(counts, max_remote_t)

    # count boundary (test instrumentation, not part of the reference's result): with c = #(cum < target)
    # the count moves by one when cum[c-1] or cum[c] crosses the target; it cannot move when every count
    # in needed-1 .. needed+1 is clamped to the same value
    n_sorted = cumulative.shape[-1]
    c = (cumulative < target[..., None]).sum(dim=-1)
    lo = cumulative.gather(-1, (c - 1).clamp(0, n_sorted - 1)[..., None])[..., 0].double()
    hi = cumulative.gather(-1, c.clamp(0, n_sorted - 1)[..., None])[..., 0].double()
    tgt = target.double()
    cm = torch.minimum(torch.where(c > 0, tgt - lo, torch.full_like(tgt, float("inf"))),
                       torch.where(c < n_sorted, hi - tgt, torch.full_like(tgt, float("inf"))))
    cap_n = torch.minimum(available, max_remote_t.expand_as(available))

    def clamp_count(n):
        return torch.minimum(torch.maximum(n, min_remote_t), cap_n)

    frozen = (clamp_count(needed - 1) == clamp_count(needed)) & (clamp_count(needed + 1) == clamp_count(needed))
    cm = torch.where(frozen | (target <= 0), torch.full_like(cm, float("inf")), cm)

    indices = sorted_idx[..., :remote_capacity].to(torch.int32)
    if indices.shape[-1] < remote_capacity:
        indices = F.pad(indices, (0, remote_capacity - indices.shape[-1]))

    if local_window_blocks > 0:
        base_indices = torch.arange(local_window_blocks, device=device, dtype=torch.int32)
        base_indices = base_indices[None, None, :].expand(batch, query_blocks, -1)
        base_counts = torch.full((batch, query_blocks), local_window_blocks, device=device,
                                 dtype=torch.int32)
    else:
        base_indices = None
        base_counts = None

    cap_rate = torch.where(
        max_remote_t > 0,
        (counts >= max_remote_t).float().mean(),
        counts.new_zeros((), dtype=torch.float32),
    )
    return OracleRoute(
        remote_indices=indices,
        remote_counts=counts.to(torch.int32),
        base_indices=base_indices,
        base_counts=base_counts,
        block_scores=block_scores,
        cap_rate=cap_rate,
        mean_remote_blocks=counts.float().mean(),
        base_only_rate=(counts == 0).float().mean(),
        remote_probs_sorted=sorted_prob,
        count_margins=cm,
    )


def router_scores(x2d: torch.Tensor, q_proj_16d: torch.Tensor, block_keys_16d: torch.Tensor) -> torch.Tensor:
    """foveal_pattention.py:257-262 — ``rms_norm(x W_q^T) K_16^T / sqrt(16)`` (block keys not normalised)."""
    index_dim = q_proj_16d.shape[0]
    q_16 = F.rms_norm(F.linear(x2d, q_proj_16d), (index_dim,))
    return torch.matmul(q_16, block_keys_16d.t()) / math.sqrt(index_dim)


def additive_stream(scores_over_t: torch.Tensor, block_keys_16d: torch.Tensor,
                    out_proj_16d: torch.Tensor) -> torch.Tensor:
    """foveal_pattention.py:338-342 — ``out_proj_16d(softmax(S / T) K_16)``; the argument is S / T."""
    soft = F.softmax(scores_over_t, dim=-1)
    context_16d = torch.matmul(soft, block_keys_16d)
    return F.linear(context_16d, out_proj_16d)


def _active_lists(base: int, remote_indices: torch.Tensor, remote_counts: torch.Tensor):
    M = remote_indices.shape[0]
    out = []
    for t in range(M):
        c = int(remote_counts[t])
        rem = remote_indices[t, :c].to(torch.int64)
        out.append(torch.cat([torch.arange(base, dtype=torch.int64), rem]))
    return out


def token_pattention_per_token(x2d, k_gate, k_up, v, base, remote_indices, remote_counts,
                               block_size: int = 64) -> torch.Tensor:
    """pattention_triton.py:280-311 applied token by token (``activation="swiglu"``): gather the
    active rows, ``silu(x K_g^T) * (x K_u^T)``, then ``@ V``.  Slow; used on small token counts."""
    offsets = torch.arange(block_size)
    y = torch.empty(x2d.shape[0], v.shape[1], dtype=torch.float32)
    for t, active in enumerate(_active_lists(base, remote_indices, remote_counts)):
        idx = (active.view(-1, 1) * block_size + offsets).flatten()
        g = torch.matmul(x2d[t:t + 1], k_gate[idx].t())
        u = torch.matmul(x2d[t:t + 1], k_up[idx].t())
        y[t] = torch.matmul(F.silu(g) * u, v[idx])[0]
    return y


def token_pattention(x2d, k_gate, k_up, v, base, remote_indices, remote_counts,
                     block_size: int = 64) -> torch.Tensor:
    """Same sum as :func:`token_pattention_per_token`, grouped by block (each block's weights are
    read once for all tokens that selected it)."""
    M, D = x2d.shape
    NB = k_gate.shape[0] // block_size
    sel = torch.zeros(M, NB, dtype=torch.bool)
    sel[:, :base] = True
    for t in range(M):
        c = int(remote_counts[t])
        if c:
            sel[t, remote_indices[t, :c].long()] = True
    y = torch.zeros(M, v.shape[1], dtype=torch.float32)
    for b in range(NB):
        toks = sel[:, b].nonzero().flatten()
        if toks.numel() == 0:
            continue
        rows = slice(b * block_size, (b + 1) * block_size)
        xb = x2d[toks]
        h = F.silu(xb @ k_gate[rows].t()) * (xb @ k_up[rows].t())
        y.index_add_(0, toks, h @ v[rows])
    return y


def token_forward(x, w, *, base_blocks, top_p, min_remote_blocks, max_remote_blocks,
                  temperature: float = 1.0, additive: bool = True, per_token: bool = False,
                  stable: bool = True) -> Dict[str, torch.Tensor]:
    """Per-token routed forward (the north-star composition of reference functions):
    ``S = compute_router_scores(x) / T`` -> ``select_blocks(S, causal=False, base)`` -> gated
    Pattention over base ∪ selected (pattention_triton.py:280-311) -> ``+ additive_stream(S)``."""
    D = x.shape[-1]
    x2d = x.reshape(-1, D).float()
    S = router_scores(x2d, w.q_proj_16d, w.block_keys_16d) / temperature
    r = select_blocks_noncausal(S[None], local_window_blocks=base_blocks, top_p=top_p,
                                min_remote_blocks=min_remote_blocks,
                                max_remote_blocks=max_remote_blocks,
                                remote_capacity=max_remote_blocks, stable=stable)
    idx, cnt = r.remote_indices[0], r.remote_counts[0]
    fn = token_pattention_per_token if per_token else token_pattention
    y = fn(x2d, w.k_gate, w.k_up, w.v, base_blocks, idx, cnt)
    if additive:
        y = y + additive_stream(S, w.block_keys_16d, w.out_proj_16d)
    return {"y": y.reshape(x.shape), "scores": S, "remote_indices": idx, "remote_counts": cnt,
            "sorted_probs": r.remote_probs_sorted[0]}


def _pooled_active(mean_scores: torch.Tensor, base: int, remote: int) -> torch.Tensor:
    """foveal_pattention.py:296-303 / :314-321 — top-k over the remote part, base ids first."""
    _, top_remote = torch.topk(mean_scores[base:], k=remote)
    if base > 0:
        return torch.cat([torch.arange(base, dtype=torch.int32), (top_remote + base).to(torch.int32)])
    return top_remote.to(torch.int32)


def pooled_eval_active(x2d, w, base, remote) -> torch.Tensor:
    """foveal_pattention.py:310-321 — pooled query ``rms_norm(W_q mean_t(x))``, scores without the
    1/sqrt(16) scale, top-k."""
    index_dim = w.q_proj_16d.shape[0]
    q_16 = F.rms_norm(F.linear(x2d.mean(dim=0, keepdim=True), w.q_proj_16d), (index_dim,))
    mean_scores = torch.matmul(q_16, w.block_keys_16d.t()).squeeze(0)
    return _pooled_active(mean_scores, base, remote)


def pooled_train_active(scores: torch.Tensor, base, remote) -> torch.Tensor:
    """foveal_pattention.py:294-303 — top-k over the token-mean of per-token scores."""
    return _pooled_active(scores.mean(dim=0), base, remote)


def pooled_pattention(x2d, w, active: torch.Tensor, block_size: int = 64) -> torch.Tensor:
    """foveal_pattention.py:115-122 and :329-335 — gather the active rows, then
    ``F.linear(silu(F.linear(x, kg)) * F.linear(x, ku), v^T)``."""
    offs = torch.arange(block_size, dtype=torch.int64)
    idx = (active.view(-1, 1).to(torch.int64) * block_size + offs).flatten()
    kg, ku, v = w.k_gate[idx], w.k_up[idx], w.v[idx]
    act = F.silu(F.linear(x2d, kg)) * F.linear(x2d, ku)
    return F.linear(act, v.t())


def pooled_forward(x, w, *, base_blocks, remote_blocks, training: bool = False,
                   temperature: float = 1.0) -> Dict[str, torch.Tensor]:
    """foveal_pattention.py:264-352 for a fresh module (no cached active set): eval routes on the
    pooled query; training routes on the token-mean of per-token scores and adds the additive
    stream."""
    D = x.shape[-1]
    x2d = x.reshape(-1, D).float()
    scores = router_scores(x2d, w.q_proj_16d, w.block_keys_16d)
    if training:
        active = pooled_train_active(scores, base_blocks, remote_blocks)
    else:
        active = pooled_eval_active(x2d, w, base_blocks, remote_blocks)
    y = pooled_pattention(x2d, w, active)
    if training:
        y = y + additive_stream(scores / temperature, w.block_keys_16d, w.out_proj_16d)
    return {"y": y.reshape(x.shape), "active_blocks": active, "scores": scores}


def boundary_margins(sorted_probs: torch.Tensor, counts: torch.Tensor) -> torch.Tensor:
    """Per token, the fp32 gap between the last selected and the first unselected remote probability
    (``p[count-1] - p[count]``); a tiny gap marks a near tie whose order depends on rounding."""
    M, n = sorted_probs.shape
    c = counts.long().clamp(1, n - 1)
    ar = torch.arange(M)
    return sorted_probs[ar, c - 1] - sorted_probs[ar, c]


PATTENTION_ACTIVATIONS = ("swiglu", "silu", "gelu", "relu", "relu2")


def pattention(x, k_gate, v, k_up=None, active_blocks=None, activation: str = "swiglu",
               block_n: int = 64) -> torch.Tensor:
    """Function-level Pattention with one shared active-block list (pattention_triton.py:280-311, the
    semantics of ``triton_pattention``, :204-277): gather the active blocks' rows, g = x K_gate^T,
    act = silu(g) * (x K_up^T) for "swiglu", silu(g) / gelu(g) (erf form) / relu(g) / relu(g)^2
    otherwise, out = act V; fp32 on the CPU."""
    if activation not in PATTENTION_ACTIVATIONS:
        raise ValueError(f"unknown activation {activation!r}")
    shape = x.shape
    x2d = x.reshape(-1, shape[-1]).float()
    kg, v = k_gate.float(), v.float()
    ku = None if k_up is None else k_up.float()
    if active_blocks is not None:
        idx = (active_blocks.long().view(-1, 1) * block_n + torch.arange(block_n)).flatten()
        kg, v = kg[idx], v[idx]
        ku = None if ku is None else ku[idx]
    g = x2d @ kg.t()
    if activation == "swiglu":
        if ku is None:
            raise ValueError("k_up is required for swiglu")
        act = F.silu(g) * (x2d @ ku.t())
    elif activation == "silu":
        act = F.silu(g)
    elif activation == "gelu":
        act = F.gelu(g)
    elif activation == "relu":
        act = F.relu(g)
    else:
        act = F.relu(g) ** 2
    return (act @ v).reshape(*shape[:-1], v.shape[-1])


def dense_swiglu(x2d, w) -> torch.Tensor:
    """Dense SwiGLU with the reparameterised weights (foveal_pattention.py:162-169):
    ``(silu(x W_gate^T) * (x W_up^T)) W_down^T`` with ``W_down^T = v``."""
    return torch.matmul(F.silu(x2d @ w.k_gate.t()) * (x2d @ w.k_up.t()), w.v)


def teacher_block_energy(x2d, k_gate, k_up, v, block_size: int = 64) -> torch.Tensor:
    """Dense SwiGLU block activation energy of the offline calibration (foveal_pattention.py:205-216):
    ``E[t, b] = mean_{j in b} |silu(x_t k_gate_j) * (x_t k_up_j)| * ||v_b||_F``, [M, NB]."""
    A = F.silu(x2d @ k_gate.t()) * (x2d @ k_up.t())
    nb = k_gate.shape[0] // block_size
    out = []
    for b in range(nb):
        rows = slice(b * block_size, (b + 1) * block_size)
        out.append(A[:, rows].abs().mean(dim=-1) * v[rows].norm())
    return torch.stack(out, dim=-1)


def calibrate_offline_svd(x2d, w, *, base_blocks: int, remote_blocks: int, temperature: float = 1.0,
                          ridge_lambda: float = 1e-2, index_dim: int = 16, block_size: int = 64):
    """Offline SVD + ridge calibration of the 16-D router (foveal_pattention.py:175-255).  Returns
    ``(q_proj [16, D], block_keys [NB, 16], info)``; info holds the reference's returned figures plus
    ``scores`` (the calibrated router scores of the calibration tokens, invariant to the sign of each
    singular vector) and ``mean_scores``."""
    X = x2d.float()
    _, S, Vh = torch.linalg.svd(X, full_matrices=False)                   # :195
    if Vh.shape[0] < index_dim:                                           # :196-198
        pad = torch.randn(index_dim - Vh.shape[0], X.shape[1])
        Vh = torch.cat([Vh, pad], dim=0)
    V16 = Vh[:index_dim, :].T                                             # :199
    Z = F.rms_norm(X @ V16, (index_dim,))                                  # :203
    teacher = teacher_block_energy(X, w.k_gate.float(), w.k_up.float(), w.v.float(), block_size)  # :206-216
    target = F.softmax(teacher / temperature, dim=-1)                     # :217
    reg = ridge_lambda * torch.eye(index_dim)                             # :220
    block_keys = torch.linalg.solve(Z.T @ Z + reg, Z.T @ target).T        # :221
    scores = (Z @ block_keys.T) / math.sqrt(index_dim)                    # :225
    student = F.softmax(scores / temperature, dim=-1)                      # :226
    kl = F.kl_div(student.log(), target, reduction="batchmean").item()    # :227
    mean_scores = scores.mean(dim=0)                                       # :230
    _, top = torch.topk(mean_scores[base_blocks:], k=remote_blocks)       # :231
    active = torch.cat([torch.arange(base_blocks, dtype=torch.int32), (top + base_blocks).to(torch.int32)])
    total_var = (S ** 2).sum().item()                                      # :242-244
    top_var = (S[:index_dim] ** 2).sum().item()
    info = {"top16_explained_variance": top_var / max(total_var, 1e-12), "initial_kl_divergence": kl,
            "calib_active_blocks": active, "scores": scores, "mean_scores": mean_scores, "teacher": teacher}
    return V16.T.contiguous(), block_keys, info


# ------------------------------------------------------------------------------------------------
# Variants sharing the router: BlockSparseLinear (block_matmul.py) and FovealTokenformerLinear
# (tokenformer.py).  Both route every token with the 16-D indexer, take the UNION of the selected
# blocks over the whole call, and run one dense contraction over that union.
# ------------------------------------------------------------------------------------------------

def param_blocks_16d(P: torch.Tensor, k_proj: torch.Tensor, v_proj: torch.Tensor, block_size: int = 64):
    """Pooled 16-D key and value per block of ``block_size`` rows of ``P`` [N, D]:
    ``k_b = normalize(mean_{rows of b} rms_norm(P W_k^T))``, ``v_b = mean_{rows of b} P W_v^T``.
    FovealIndexer.compute_kv_blocks_16d (core.py:225-252) and BlockSparseLinear.get_block_keys_and_values
    (block_matmul.py:107-127) are the same formula with different projection weights."""
    n, d = P.shape
    nb = n // block_size
    k_elem = F.rms_norm(P @ k_proj.t(), (k_proj.shape[0],))
    v_elem = P @ v_proj.t()
    k_blocks = k_elem.view(nb, block_size, -1).mean(dim=1)
    v_blocks = v_elem.view(nb, block_size, -1).mean(dim=1)
    return F.normalize(k_blocks.float(), dim=-1), v_blocks


def cosine_block_scores(x2d: torch.Tensor, q_proj: torch.Tensor, k_blocks: torch.Tensor) -> torch.Tensor:
    """``normalize(rms_norm(x W_q^T)) . normalize(k_blocks)^T / sqrt(16)``: compute_query_16d
    (core.py:214-223) followed by FovealIndexer.compute_block_scores (core.py:254-266)."""
    q = F.rms_norm(x2d @ q_proj.t(), (q_proj.shape[0],))
    qn = F.normalize(q.float(), dim=-1)
    kn = F.normalize(k_blocks.float(), dim=-1)
    return (qn @ kn.t()) / math.sqrt(q_proj.shape[0])


def union_blocks(base: int, remote_indices: torch.Tensor, remote_counts: torch.Tensor, num_blocks: int,
                 index_offset: int = 0) -> torch.Tensor:
    """Ascending ids of ``[0, base)`` united with every token's selected remote blocks
    (block_matmul.py:206-217 ``torch.where(active_block_mask)``; tokenformer.py:176-181
    ``torch.unique`` after the base blocks)."""
    mask = torch.zeros(num_blocks, dtype=torch.bool)
    mask[:base] = True
    cap = remote_indices.shape[-1]
    idx = remote_indices.reshape(-1, cap).long() + index_offset
    cnt = remote_counts.reshape(-1).long()
    valid = torch.arange(cap).view(1, -1) < cnt.view(-1, 1)
    sel = idx[valid]
    sel = sel[sel >= base]
    if sel.numel():
        mask[sel] = True
    return torch.where(mask)[0].to(torch.int32)


def fast_remote_route(scores: torch.Tensor, base: int, top_p: float, max_remote: int):
    """BlockSparseLinear's inference selection (block_matmul.py:185-201): softmax over the remote
    columns only, ``needed = clamp(#(cumsum < top_p) + 1, 0, K_max)`` leading blocks by descending
    probability (ties to the lower id).  This is select_blocks (core.py:46-160) on the remote columns
    with no base blocks and K_min = 0, returned with block ids offset back by ``base``."""
    rem = scores[:, base:]
    n_rem = rem.shape[1]
    r = select_blocks_noncausal(rem[None], local_window_blocks=0, top_p=top_p, min_remote_blocks=0,
                                max_remote_blocks=max_remote, remote_capacity=min(max_remote, n_rem))
    return r.remote_indices[0].long() + base, r.remote_counts[0]


def fast_rule_counts(scores: torch.Tensor, base: int, top_p: float, max_remote: int) -> torch.Tensor:
    """The inference rule's per-token count as the reference computes it (block_matmul.py:188-193):
    ``clamp(#(cumsum of the sorted remote softmax < top_p) + 1, 0, K_max)``, not clamped to the available
    blocks (so it can exceed them by one when the mass never reaches top_p)."""
    probs = F.softmax(scores[:, base:], dim=-1)
    cum = probs.sort(dim=-1, descending=True, stable=True).values.cumsum(dim=-1)
    return torch.clamp((cum < top_p).sum(dim=-1) + 1, 0, max_remote)


def block_sparse_linear(x2d, weight, bias, q_proj, weight_to_k, weight_to_v, out_proj, *, block_size: int,
                        base_blocks: int, top_p: float, min_remote_blocks: int, max_remote_blocks: int,
                        remote_capacity: int, fast_rule: bool, use_additive_stream: bool = True):
    """BlockSparseLinear.forward (block_matmul.py:129-282) without the teacher loss.  ``fast_rule``:
    the eval/no-grad selection (:185-201); otherwise FovealIndexer.route (:202-217).  Returns
    ``(out [M, out_features], active ids, remote_indices, remote_counts, scores)``."""
    nb = weight.shape[0] // block_size
    base = min(base_blocks, nb)
    k_blocks, v_blocks = param_blocks_16d(weight, weight_to_k, weight_to_v, block_size)   # :108-127
    scores = cosine_block_scores(x2d, q_proj, k_blocks)                                    # :176
    if fast_rule:
        idx, cnt = fast_remote_route(scores, base, top_p, max_remote_blocks)
        active = union_blocks(base, idx, cnt, nb)
    else:
        r = select_blocks_noncausal(scores[None], local_window_blocks=base, top_p=top_p,
                                    min_remote_blocks=min_remote_blocks, max_remote_blocks=max_remote_blocks,
                                    remote_capacity=remote_capacity)
        idx, cnt = r.remote_indices[0], r.remote_counts[0]
        active = union_blocks(base, idx, cnt, nb)
    chan = (active.long().view(-1, 1) * block_size + torch.arange(block_size)).flatten()   # :234-236
    out = torch.zeros(x2d.shape[0], weight.shape[0])
    out[:, chan] = x2d @ weight[chan].t()                                                   # :238-243
    if bias is not None:                                                                   # :245-247
        out[:, chan] = out[:, chan] + bias[chan]
    if use_additive_stream:                                                                # :250-254
        probs = F.softmax(scores, dim=-1)
        out = out + (probs @ v_blocks) @ out_proj.t()
    return out, active, idx, cnt, scores


def tokenformer_linear(x2d, k_param, v_param, q_proj, k_proj, v_proj, out_proj, *, block_size: int,
                       base_blocks: int, top_p: float, min_remote_blocks: int, max_remote_blocks: int,
                       remote_capacity: int, activation: str, use_additive_stream: bool = True):
    """FovealTokenformerLinear.forward (tokenformer.py:132-228) without the teacher loss: route with
    FovealIndexer.route (:163), union of the selected blocks (:171-181), then
    ``act(x K_act^T) V_act`` with ``act`` = softmax(s / sqrt(D_in)) or gelu(normalize(s)) (:101-110),
    plus the additive stream (:197-203).  Returns ``(out, active ids, remote_indices, remote_counts,
    scores)``."""
    nb = k_param.shape[0] // block_size
    k_blocks, v_blocks = param_blocks_16d(k_param, k_proj, v_proj, block_size)             # :150-155
    scores = cosine_block_scores(x2d, q_proj, k_blocks)                                    # :160
    r = select_blocks_noncausal(scores[None], local_window_blocks=base_blocks, top_p=top_p,
                                min_remote_blocks=min_remote_blocks, max_remote_blocks=max_remote_blocks,
                                remote_capacity=remote_capacity)
    idx, cnt = r.remote_indices[0], r.remote_counts[0]
    active = union_blocks(base_blocks, idx, cnt, nb)
    rows = (active.long().view(-1, 1) * block_size + torch.arange(block_size)).flatten()
    raw = x2d @ k_param[rows].t()                                                          # :186
    if activation == "softmax":
        w = F.softmax(raw / math.sqrt(x2d.shape[1]), dim=-1)
    elif activation == "gelu_l2":
        w = F.gelu(F.normalize(raw, p=2, dim=-1))
    else:
        raise ValueError(activation)
    out = w @ v_param[rows]                                                                 # :188
    if use_additive_stream:
        probs = F.softmax(scores, dim=-1)
        out = out + (probs @ v_blocks) @ out_proj.t()
    return out, active, idx, cnt, scores
