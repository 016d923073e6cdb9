"""BlockSparseLinear: a linear projection whose 64-column output blocks are chosen per call by the 16-D
foveal router, on the CUDA library (mirrors ``foveal_indexer/block_matmul.py:25-282``).

Same constructor, parameter names, initialisation, ``state_dict`` keys and ``(out, aux)`` result as the
reference; the aux statistics (union size, mean active blocks, sparsity) are 0-d device tensors instead
of Python numbers, so a forward never waits for the GPU (``int()`` / ``float()`` read them).  A forward is: pooled 16-D block keys / values of the weight (cached in eval), cosine block
scores of the tokens, the selection (the inference rule of block_matmul.py:185-201 in eval without
autograd, ``FovealIndexer.route`` otherwise), the union of the selected blocks, and one contraction over
that union with the bias and the 16-D additive stream in its epilogue (tcgen05 tensor cores for bf16).
The layer is forward-only: a backward through it raises.
"""

from __future__ import annotations

import math
from typing import Any, Dict, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from . import kernels
from .core import FovealIndexer


class _NoBackward(torch.autograd.Function):
    """Attaches a backward that raises, so a training graph through the kernels fails loudly."""

    @staticmethod
    def forward(ctx, y, *inputs):
        return y

    @staticmethod
    def backward(ctx, *grads):
        raise NotImplementedError("BlockSparseLinear / FovealTokenformerLinear run forward-only kernels; "
                                  "their backward is not part of this library")


def forward_only(y: Tensor, module: nn.Module, x: Tensor) -> Tensor:
    if torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in module.parameters())):
        return _NoBackward.apply(y, x, *[p for p in module.parameters() if p.requires_grad])
    return y


def additive_context(scores: Tensor, v_blocks: Tensor) -> Tensor:
    """softmax(S) . v_blocks per token (block_matmul.py:251-252, tokenformer.py:199-201): fp32 [M, 16],
    from the selection kernel's context-only mode with temperature 1."""
    _, _, ctx, _ = kernels.select(scores, base_blocks=0, top_p=1.0, min_remote=0, max_remote=0, capacity=0,
                                  block_keys=v_blocks, want_routes=False)
    return ctx


class BlockSparseLinear(nn.Module):
    """Linear projection (in_features -> out_features) with blockwise dynamic sparsity
    (block_matmul.py:25-282)."""

    def __init__(self, in_features: int, out_features: int, block_size: int = 64, base_blocks: int = 2,
                 index_dim: int = 16, top_p: float = 0.95, min_remote_blocks: int = 0, max_remote_blocks: int = 8,
                 remote_capacity: int = 8, use_additive_stream: bool = True, bias: bool = False):
        super().__init__()
        if out_features % block_size != 0:
            raise ValueError(f"out_features ({out_features}) must be divisible by block_size ({block_size})")
        if block_size != 64:
            raise NotImplementedError("the CUDA kernels use 64-column blocks")
        self.in_features = in_features
        self.out_features = out_features
        self.block_size = block_size
        self.num_blocks = out_features // block_size
        self.base_blocks = min(base_blocks, self.num_blocks)
        self.use_additive_stream = use_additive_stream
        self.weight = nn.Parameter(torch.empty(out_features, in_features))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features))
        else:
            self.register_parameter("bias", None)
        self.reset_parameters()
        self.indexer = FovealIndexer(hidden_size=in_features, index_dim=index_dim, block_size=block_size,
                                     local_window_blocks=self.base_blocks, top_p=top_p,
                                     min_remote_blocks=min_remote_blocks, max_remote_blocks=max_remote_blocks,
                                     remote_capacity=remote_capacity, causal=False,
                                     use_additive_stream=use_additive_stream)
        self.weight_to_k = nn.Linear(in_features, index_dim, bias=False)
        self.weight_to_v = nn.Linear(in_features, index_dim, bias=False)
        self.indexer.out_proj = nn.Linear(index_dim, out_features, bias=False)
        nn.init.normal_(self.weight_to_k.weight, std=in_features ** -0.5)
        nn.init.normal_(self.weight_to_v.weight, std=in_features ** -0.5)
        nn.init.normal_(self.indexer.out_proj.weight, std=1e-3)
        self._cached_kp: Optional[Tensor] = None
        self._cached_vp: Optional[Tensor] = None
        self._blocked_on = False
        self._blocked: Optional[Tensor] = None
        self._blocked_key = None

    def use_blocked_weight(self, enable: bool = True) -> "BlockSparseLinear":
        """Keep a 64 x 64 blocked copy of the bf16 weight for the eval-mode tensor-core contraction
        (``fp_pack_blocked_weight``): each selected block at one k-block is one contiguous 8 KB run instead of
        64 row pieces of 128 bytes (measured ~8 % faster at 64 tokens on the 4096 -> 14336 shape, unchanged
        at 1 and 16384 tokens), at the cost of a second copy of the weight in device memory.  Results are
        bit-identical.  Rebuilt when the weight changes."""
        self._blocked_on = bool(enable)
        if not enable:
            self._blocked, self._blocked_key = None, None
        return self

    def _blocked_weight(self) -> Optional[Tensor]:
        w = self.weight
        if (not self._blocked_on or self.training or w.dtype != torch.bfloat16 or not w.is_cuda
                or self.in_features % 64):
            return None
        key = (w.data_ptr(), w._version, tuple(w.shape))
        if self._blocked_key != key:
            self._blocked = kernels.pack_blocked_weight(w.detach())
            self._blocked_key = key
        return self._blocked

    def reset_parameters(self) -> None:
        """block_matmul.py:101-106."""
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            fan_in, _ = nn.init._calculate_fan_in_and_fan_out(self.weight)
            bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
            nn.init.uniform_(self.bias, -bound, bound)

    def _blocks_16d(self) -> Tuple[Tensor, Tensor]:
        """fp32 (k_blocks [NB, 16] normalised, v_blocks [NB, 16]) of the weight (``fp_param_blocks_16d``)."""
        return kernels.param_blocks_16d(self.weight, self.weight_to_k.weight, self.weight_to_v.weight)

    def get_block_keys_and_values(self) -> Tuple[Tensor, Tensor]:
        """16-D key and value of every weight block, (1, NB, 16) each in the weight's dtype
        (block_matmul.py:107-127)."""
        kb, vb = self._blocks_16d()
        return kb.to(self.weight.dtype).unsqueeze(0), vb.to(self.weight.dtype).unsqueeze(0)

    def refresh_block_cache(self) -> None:
        """block_matmul.py:95-99."""
        with torch.no_grad():
            self._cached_kp, self._cached_vp = self._blocks_16d()

    def forward_kernels(self, x2d: Tensor, fast: bool, batch_shape=None) -> Dict[str, Any]:
        """The routed forward of [M, in_features] tokens as one stream of kernel launches, without any host
        synchronisation: ``fast`` selects the inference rule (block_matmul.py:185-201) instead of
        FovealIndexer.route.  Returns the device tensors (out, scores, route or (idx, cnt, stats),
        blocks, n_active, ctx16)."""
        M, NB, base = x2d.shape[0], self.num_blocks, self.base_blocks
        dev = x2d.device
        # 1-2. block keys / values (cached in eval, :160-167) and the queries' cosine scores (:170-176)
        if not self.training and self._cached_kp is not None:
            kb, vb = self._cached_kp, self._cached_vp
        else:
            kb, vb = self._blocks_16d()
            if not self.training:
                self._cached_kp, self._cached_vp = kb, vb
        scores, _ = kernels.cosine_block_scores(x2d, self.indexer.q_proj.weight, kb)
        # 3-4. selection and union of the selected blocks
        route, stats = None, None
        if fast:
            if NB - base > 0:
                idx, cnt, stats = kernels.select_remote_top_p(scores, base_blocks=base, top_p=self.indexer.top_p,
                                                              max_remote=self.indexer.max_remote_blocks,
                                                              want_stats=True)
            else:
                idx = torch.zeros(M, 1, dtype=torch.int32, device=dev)
                cnt = torch.zeros(M, dtype=torch.int32, device=dev)
        else:
            route = self.indexer.route(scores.view(*(batch_shape or (1, M)), NB))
            idx, cnt = route.remote_indices, route.remote_counts
        blocks, n_active = kernels.union_blocks(idx, cnt, NB, base)
        # 5-6. contraction over the union (+ bias) with the additive stream in the epilogue
        ctx16 = additive_context(scores, vb) if self.use_additive_stream else None
        max_active = min(NB, base + M * idx.shape[-1])  # host-side bound of the union
        out2d = kernels.block_sparse_linear(x2d, self.weight, self.bias, blocks, n_active, ctx16,
                                            self.indexer.out_proj.weight, max_active=max_active,
                                            weight_blocked=self._blocked_weight())
        return {"out": out2d, "scores": scores, "route": route, "stats": stats, "blocks": blocks,
                "n_active": n_active, "ctx16": ctx16}

    def forward(self, x: Tensor, compute_teacher_loss: bool = False) -> Tuple[Tensor, Dict[str, Any]]:
        orig_ndim = x.ndim
        if orig_ndim == 2:
            x = x.unsqueeze(1)
        batch, seq_len, in_feat = x.shape
        dev = x.device
        x_in = x
        x2d = x.reshape(-1, in_feat).to(self.weight.dtype)
        M, NB, base = x2d.shape[0], self.num_blocks, self.base_blocks
        fast = not self.training and not torch.is_grad_enabled()
        r = self.forward_kernels(x2d, fast, (batch, seq_len))
        route, scores, ctx16, n_active = r["route"], r["scores"], r["ctx16"], r["n_active"]
        # the aux statistics stay on the device (0-d tensors): the forward never waits for the GPU
        if route is not None:
            mean_remote = route.mean_remote_blocks
        elif r["stats"] is not None:
            mean_remote = r["stats"][1] / max(M, 1)
        else:
            mean_remote = torch.zeros((), dtype=torch.float32, device=dev)
        out = r["out"].view(batch, seq_len, self.out_features)
        additive_out = None
        if ctx16 is not None:
            # the additive term alone, for the aux dict (the output already contains it)
            additive_out = (ctx16 @ self.indexer.out_proj.weight.detach().float().t()).to(out.dtype)
            additive_out = additive_out.view(batch, seq_len, self.out_features)
        out = forward_only(out, self, x_in)
        if orig_ndim == 2:
            out = out.squeeze(1)
        num_active = n_active.reshape(())
        mean_active = base + mean_remote
        aux: Dict[str, Any] = {
            "route": route,
            "additive_out": additive_out,
            "active_blocks_union": num_active,
            "mean_active_blocks": mean_active,
            "total_blocks": NB,
            "sparsity": 1.0 - mean_active / NB,
            "distill_loss": torch.tensor(0.0, device=dev),
        }
        if compute_teacher_loss:  # :262-280: dense output -> block L2 energies -> softmax target
            with torch.no_grad():
                all_blocks = torch.arange(NB, dtype=torch.int32, device=dev)
                n_all = torch.full((1,), NB, dtype=torch.int32, device=dev)
                dense = kernels.block_sparse_linear(x2d, self.weight, self.bias, all_blocks, n_all)
                energy = dense.float().view(batch, seq_len, NB, self.block_size).norm(p=2, dim=-1)
                teacher_mass = F.softmax(energy, dim=-1)
            aux["distill_loss"] = self.indexer.distillation_loss(scores.view(batch, seq_len, NB), teacher_mass)
        return out, aux
