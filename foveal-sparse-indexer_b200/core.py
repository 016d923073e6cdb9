"""Router core: ``Route``, ``select_blocks``, ``masked_softmax`` and ``FovealIndexer``.

Mirrors ``foveal_indexer/core.py`` of the reference for the parts on the Pattention MLP hot path and
on the layers that share its router (BlockSparseLinear, FovealTokenformerLinear): the non-causal
top-p selection with base-block reservation (core.py:46-160, branch :90-99), the normalised 16-D
query (core.py:214-223), the pooled 16-D block keys / values (core.py:225-252) and the cosine block
scores (core.py:254-266), all computed by the CUDA library.  The causal routing branch and the
indexer's own attention additive stream belong to the reference's attention path and raise
``NotImplementedError``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
from torch import Tensor, nn

from . import kernels
from ._lib import require_cuda


@dataclass
class Route:
    """Routing decisions (same fields as the reference ``Route``, core.py:23-33)."""

    remote_indices: Tensor        # (B, Q, remote_capacity) int32, descending probability, ties -> lower id
    remote_counts: Tensor         # (B, Q) int32
    base_indices: Optional[Tensor]  # (B, Q, base) int32
    base_counts: Optional[Tensor]   # (B, Q) int32
    block_scores: Tensor          # (B, Q, total_blocks)
    cap_rate: Tensor              # fraction of rows with count >= K_max
    mean_remote_blocks: Tensor
    base_only_rate: Tensor        # fraction of rows with count == 0


def masked_softmax(scores: Tensor, mask: Tensor) -> Tensor:
    """Softmax that zeroes masked entries (core.py:36-43).  CUDA tensors only."""
    require_cuda(scores, mask)
    safe = scores.float().masked_fill(~mask, -float("inf"))
    row_max = safe.amax(dim=-1, keepdim=True)
    row_max = torch.where(torch.isfinite(row_max), row_max, torch.zeros_like(row_max))
    numer = torch.exp(safe - row_max) * mask
    denom = numer.sum(dim=-1, keepdim=True).clamp_min(1e-20)
    return (numer / denom).to(scores.dtype)


def _scalar(v, kind):
    if isinstance(v, Tensor):
        if v.numel() != 1:
            raise NotImplementedError("per-row top_p / K_min / K_max tensors are not supported; pass scalars")
        v = v.item()
    return kind(v)


def select_blocks(
    block_scores: Tensor,
    *,
    causal: bool = True,
    block_size: int = 64,
    local_window_blocks: int = 0,
    top_p: float | Tensor = 0.95,
    min_remote_blocks: int | Tensor = 0,
    max_remote_blocks: int | Tensor = 16,
    remote_capacity: int = 16,
) -> Route:
    """Adaptive top-p mass routing over block scores (core.py:46-160), on the GPU.

    Only the non-causal branch (parameter blocks: base blocks are ``[0, local_window_blocks)``) is
    implemented; ``causal=True`` (the reference default, used by its attention path) raises.
    """
    if causal:
        raise NotImplementedError("select_blocks(causal=True) is the reference's attention routing; "
                                  "this library implements the non-causal parameter-block branch")
    B, Q, NB = block_scores.shape
    require_cuda(block_scores)
    tp = _scalar(top_p, float)
    kmin = _scalar(min_remote_blocks, int)
    kmax = _scalar(max_remote_blocks, int)
    cap = int(remote_capacity)
    if cap <= 0:
        raise ValueError("remote_capacity must be positive")
    idx, cnt, _, stats = kernels.select(block_scores.detach().reshape(B * Q, NB), base_blocks=local_window_blocks,
                                        top_p=tp, min_remote=kmin, max_remote=kmax, capacity=cap,
                                        want_stats=True)
    dev = block_scores.device
    M = max(B * Q, 1)
    if local_window_blocks > 0:
        base_indices = torch.arange(local_window_blocks, device=dev, dtype=torch.int32)[None, None, :].expand(B, Q, -1)
        base_counts = torch.full((B, Q), local_window_blocks, device=dev, dtype=torch.int32)
    else:
        base_indices = base_counts = None
    cap_rate = stats[0] / M if kmax > 0 else torch.zeros((), device=dev)
    return Route(
        remote_indices=idx.view(B, Q, cap),
        remote_counts=cnt.view(B, Q),
        base_indices=base_indices,
        base_counts=base_counts,
        block_scores=block_scores,
        cap_rate=cap_rate,
        mean_remote_blocks=stats[1] / M,
        base_only_rate=stats[2] / M,
    )


class FovealIndexer(nn.Module):
    """16-dimensional foveal indexer (core.py:163-353), hot-path subset.

    Same constructor, parameter names and initialisation as the reference.  ``compute_query_16d``
    and ``route`` run on the GPU; the attention-only members raise ``NotImplementedError``.
    """

    def __init__(self, hidden_size: int, index_dim: int = 16, block_size: int = 64,
                 local_window_blocks: int = 8, top_p: float = 0.95, min_remote_blocks: int = 0,
                 max_remote_blocks: int = 16, remote_capacity: int = 16, causal: bool = True,
                 use_additive_stream: bool = True, distill_temperature: float = 1.0):
        super().__init__()
        if index_dim != 16:
            raise ValueError("the CUDA router is specialised for index_dim = 16")
        self.hidden_size = hidden_size
        self.index_dim = index_dim
        self.block_size = block_size
        self.local_window_blocks = local_window_blocks
        self.top_p = top_p
        self.min_remote_blocks = min_remote_blocks
        self.max_remote_blocks = max_remote_blocks
        self.remote_capacity = remote_capacity
        self.causal = causal
        self.use_additive_stream = use_additive_stream
        self.distill_temperature = distill_temperature
        self.q_proj = nn.Linear(hidden_size, index_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, index_dim, bias=False)
        self.v_proj = nn.Linear(hidden_size, index_dim, bias=False)
        self.out_proj = nn.Linear(index_dim, hidden_size, bias=False)
        nn.init.normal_(self.q_proj.weight, std=hidden_size ** -0.5)
        nn.init.normal_(self.k_proj.weight, std=hidden_size ** -0.5)
        nn.init.normal_(self.v_proj.weight, std=hidden_size ** -0.5)
        nn.init.normal_(self.out_proj.weight, std=1e-3)

    def compute_query_16d(self, x: Tensor) -> Tensor:
        """``rms_norm(q_proj(x))`` (core.py:214-223) -> (..., 16) in x's dtype."""
        shape = x.shape
        x2d = x.reshape(-1, shape[-1])
        dummy_keys = torch.zeros(1, 16, dtype=x.dtype, device=x.device)
        _, q16 = kernels.router_scores(x2d, self.q_proj.weight.detach(), dummy_keys, want_q16=True)
        return q16.to(x.dtype).reshape(*shape[:-1], 16)

    def route(self, block_scores: Tensor, top_p: Optional[float] = None,
              max_remote_blocks: Optional[int] = None, min_remote_blocks: Optional[int] = None) -> Route:
        """Adaptive top-p routing (core.py:268-286); non-causal indexers only."""
        return select_blocks(
            block_scores.detach(), causal=self.causal, block_size=self.block_size,
            local_window_blocks=self.local_window_blocks,
            top_p=self.top_p if top_p is None else top_p,
            min_remote_blocks=self.min_remote_blocks if min_remote_blocks is None else min_remote_blocks,
            max_remote_blocks=self.max_remote_blocks if max_remote_blocks is None else max_remote_blocks,
            remote_capacity=self.remote_capacity)

    def compute_kv_blocks_16d(self, x: Tensor):
        """Pooled 16-D key (L2-normalised) and value per block of ``block_size`` rows (core.py:225-252).

        x: (B, N, D) or (N, D) with N % block_size == 0 -> (k_blocks, v_blocks), each (B, N / bs, 16) in
        x's dtype (one ``fp_param_blocks_16d`` call per batch row)."""
        if self.block_size != 64:
            raise NotImplementedError("the CUDA kernels pool blocks of 64 rows")
        if x.ndim == 2:
            x = x.unsqueeze(0)
        if x.shape[1] % self.block_size != 0:
            raise ValueError(f"Element length {x.shape[1]} must be divisible by block_size={self.block_size}")
        ks, vs = [], []
        for b in range(x.shape[0]):
            kb, vb = kernels.param_blocks_16d(x[b], self.k_proj.weight, self.v_proj.weight)
            ks.append(kb)
            vs.append(vb)
        return torch.stack(ks).to(x.dtype), torch.stack(vs).to(x.dtype)

    def compute_block_scores(self, q_blocks: Tensor, k_blocks: Tensor) -> Tensor:
        """``normalize(q) . normalize(k)^T / sqrt(16)`` (core.py:254-266): (B, Q, 16) x (B, NB, 16) ->
        (B, Q, NB) fp32.  Runs the cosine-score kernel with the queries as inputs and an identity
        projection (its rms_norm before the L2 normalisation does not change the direction)."""
        require_cuda(q_blocks, k_blocks)
        B, Q, _ = q_blocks.shape
        eye = torch.eye(16, dtype=q_blocks.dtype, device=q_blocks.device)
        out = []
        for b in range(B):
            kb = k_blocks[b if k_blocks.shape[0] > 1 else 0]
            s, _ = kernels.cosine_block_scores(q_blocks[b], eye, kb)
            out.append(s)
        return torch.stack(out)

    def additive_stream(self, block_scores: Tensor, v_blocks: Tensor) -> Tensor:
        raise NotImplementedError("the indexer's attention additive stream is not part of this library; "
                                  "the Pattention MLP's additive stream is fused into its forward")

    def distillation_loss(self, student_scores: Tensor, teacher_block_mass: Tensor,
                          valid_mask: Optional[Tensor] = None) -> Tensor:
        """Cross-entropy of the student block distribution against the teacher block mass
        (core.py:310-353), non-causal indexers: ``mean_q -sum_b target * log_softmax(s / T)`` with the
        teacher mass clamped at 0 and normalised (uniform where it sums to ~0).  A scalar training loss
        on [B, Q, NB] tensors, computed with torch on the scores' device."""
        require_cuda(student_scores, teacher_block_mass)
        if valid_mask is None:
            if self.causal:
                raise NotImplementedError("causal distillation masks belong to the reference's attention path")
            valid_mask = torch.ones_like(student_scores, dtype=torch.bool)
        masked = student_scores.masked_fill(~valid_mask, -float("inf"))
        log_student = torch.log_softmax(masked.float() / self.distill_temperature, dim=-1)
        log_student = torch.where(valid_mask, log_student, torch.zeros_like(log_student))
        teacher = teacher_block_mass.float().clamp_min(0.0).masked_fill(~valid_mask, 0.0)
        denom = teacher.sum(dim=-1, keepdim=True)
        uniform = valid_mask.float() / valid_mask.float().sum(dim=-1, keepdim=True).clamp_min(1.0)
        target = torch.where(denom > 1e-12, teacher / denom.clamp_min(1e-12), uniform)
        kl = -(target.detach() * log_student).sum(dim=-1)
        has_valid = valid_mask.any(dim=-1)
        if bool(has_valid.any()):
            return kl[has_valid].mean()
        return student_scores.sum() * 0.0
