"""Foveal Tokenformer layers on the CUDA library (mirrors ``foveal_indexer/tokenformer.py:26-283``).

``FovealTokenformerLinear`` replaces a linear projection by attention from the input tokens to learnable
parameter tokens (K_P, V_P), restricted to the union of the 64-token parameter blocks the call's
tokens select with the 16-D foveal router.  Same constructor, parameter names, initialisation,
``state_dict`` keys and ``(out, aux)`` result as the reference (the aux counts are 0-d device tensors, so
the forward never waits for the GPU).  A forward is: pooled 16-D keys / values
of the parameter blocks (cached in eval), cosine block scores, ``FovealIndexer.route``, the union of the
selected blocks, then ``act(x K_act^T) V_act`` (two tensor-core contractions for bf16 around a row
activation kernel) with the 16-D additive stream in the second contraction's epilogue.  Forward-only.
"""

from __future__ import annotations

import math
from typing import Any, Dict, Literal, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from . import kernels
from .block_matmul import additive_context, forward_only
from .core import FovealIndexer


class FovealTokenformerLinear(nn.Module):
    """Token-parameter attention layer with foveal block selection (tokenformer.py:26-228)."""

    def __init__(self, in_features: int, out_features: int, num_param_tokens: int = 512, param_block_size: int = 64,
                 base_blocks: int = 2, index_dim: int = 16, top_p: float = 0.95, min_remote_blocks: int = 0,
                 max_remote_blocks: int = 4, remote_capacity: int = 4,
                 activation: Literal["softmax", "gelu_l2"] = "softmax", use_additive_stream: bool = True):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.num_param_tokens = num_param_tokens
        self.param_block_size = param_block_size
        self.base_blocks = base_blocks
        self.activation = activation
        self.use_additive_stream = use_additive_stream
        if num_param_tokens % param_block_size != 0:
            raise ValueError(f"num_param_tokens ({num_param_tokens}) must be divisible by "
                             f"param_block_size ({param_block_size})")
        if param_block_size != 64:
            raise NotImplementedError("the CUDA kernels use 64-token parameter blocks")
        if activation not in kernels.ACTIVATIONS:
            raise ValueError(f"Unknown activation: {activation}")
        self.num_blocks = num_param_tokens // param_block_size
        assert base_blocks <= self.num_blocks, "base_blocks cannot exceed total parameter blocks"
        self.k_param = nn.Parameter(torch.empty(num_param_tokens, in_features))
        self.v_param = nn.Parameter(torch.empty(num_param_tokens, out_features))
        nn.init.normal_(self.k_param, std=in_features ** -0.5)
        nn.init.normal_(self.v_param, std=out_features ** -0.5)
        self.indexer = FovealIndexer(hidden_size=in_features, index_dim=index_dim, block_size=param_block_size,
                                     local_window_blocks=base_blocks, top_p=top_p,
                                     min_remote_blocks=min_remote_blocks, max_remote_blocks=max_remote_blocks,
                                     remote_capacity=remote_capacity, causal=False,
                                     use_additive_stream=use_additive_stream)
        self.indexer.out_proj = nn.Linear(index_dim, out_features, bias=False)
        nn.init.normal_(self.indexer.out_proj.weight, std=1e-3)
        self._cached_kp: Optional[Tensor] = None
        self._cached_vp: Optional[Tensor] = None
        self._vt_cache: Optional[Tuple[Tuple, Tensor]] = None

    def _blocks_16d(self) -> Tuple[Tensor, Tensor]:
        return kernels.param_blocks_16d(self.k_param, self.indexer.k_proj.weight, self.indexer.v_proj.weight)

    def refresh_param_cache(self) -> None:
        """tokenformer.py:96-99."""
        with torch.no_grad():
            self._cached_kp, self._cached_vp = self._blocks_16d()

    def _v_param_t(self) -> Optional[Tensor]:
        """v_param transposed [D_out, Np] for the tensor-core contraction (bf16), rebuilt when v_param
        changes."""
        v = self.v_param
        if v.dtype != torch.bfloat16:
            return None
        key = (v.data_ptr(), v._version, v.shape)
        if self._vt_cache is None or self._vt_cache[0] != key:
            self._vt_cache = (key, kernels.transpose(v.detach()))
        return self._vt_cache[1]

    def _activate_scores(self, scores: Tensor) -> Tensor:
        """tokenformer.py:101-110 (used by the dense teacher)."""
        if self.activation == "softmax":
            return F.softmax(scores / math.sqrt(self.in_features), dim=-1)
        return F.gelu(F.normalize(scores, p=2, dim=-1))

    def compute_dense_teacher(self, x: Tensor) -> Tuple[Tensor, Tensor]:
        """Dense attention over every parameter token and its block mass (tokenformer.py:112-130), the
        distillation target.  A training aid: plain torch on the parameters' device, outside the
        routed kernel path."""
        raw = torch.matmul(x, self.k_param.t())
        attn = self._activate_scores(raw)
        dense_out = torch.matmul(attn, self.v_param)
        batch, seq_len, _ = x.shape
        block_mass = attn.clamp_min(0.0).view(batch, seq_len, self.num_blocks, self.param_block_size).sum(dim=-1)
        return dense_out, block_mass

    def forward_kernels(self, x2d: Tensor, batch_shape=None) -> Dict[str, Any]:
        """The routed forward of [M, in_features] tokens as one stream of kernel launches, without any host
        synchronisation.  Returns the device tensors (out, scores, route, blocks, n_active, ctx16)."""
        M, NB = x2d.shape[0], self.num_blocks
        # 1-3. block keys / values (cached in eval, :146-155), cosine scores (:160)
        if not self.training and self._cached_kp is not None:
            kb, vb = self._cached_kp, self._cached_vp
        else:
            kb, vb = self._blocks_16d()
            if not self.training:
                self._cached_kp, self._cached_vp = kb, vb
        scores, _ = kernels.cosine_block_scores(x2d, self.indexer.q_proj.weight, kb)
        # 4. route every token (:163), union of the selected blocks (:171-181)
        route = self.indexer.route(scores.view(*(batch_shape or (1, M)), NB))
        blocks, n_active = kernels.union_blocks(route.remote_indices, route.remote_counts, NB, self.base_blocks)
        # 5-6. act(x K_act^T) V_act with the additive stream in the epilogue (:183-203)
        ctx16 = additive_context(scores, vb) if self.use_additive_stream else None
        out2d = kernels.tokenformer(x2d, self.k_param, self.v_param, self._v_param_t(), self.activation, blocks,
                                    n_active, ctx16, self.indexer.out_proj.weight)
        return {"out": out2d, "scores": scores, "route": route, "blocks": blocks, "n_active": n_active, "ctx16": ctx16}

    def forward(self, x: Tensor, compute_teacher_loss: bool = False) -> Tuple[Tensor, Dict[str, Any]]:
        batch, seq_len, _ = x.shape
        dev = x.device
        x2d = x.reshape(-1, self.in_features).to(self.k_param.dtype)
        NB, bs = self.num_blocks, self.param_block_size
        r = self.forward_kernels(x2d, (batch, seq_len))
        route, scores, ctx16, n_active = r["route"], r["scores"], r["ctx16"], r["n_active"]
        out = r["out"].view(batch, seq_len, self.out_features)
        additive_out = None
        if ctx16 is not None:
            additive_out = (ctx16 @ self.indexer.out_proj.weight.detach().float().t()).to(out.dtype)
            additive_out = additive_out.view(batch, seq_len, self.out_features)
        out = forward_only(out, self, x)
        base_param_count = self.base_blocks * bs
        aux: Dict[str, Any] = {
            "route": route,
            "additive_out": additive_out,
            # device 0-d tensors: the forward never waits for the GPU to fill the aux dict
            "active_param_tokens_union": n_active.reshape(()) * bs,
            "mean_active_param_tokens": base_param_count + route.mean_remote_blocks * bs,
            "total_param_tokens": self.num_param_tokens,
            "distill_loss": torch.tensor(0.0, device=dev),
        }
        if compute_teacher_loss:  # :214-218
            with torch.no_grad():
                _, teacher_mass = self.compute_dense_teacher(x.to(self.k_param.dtype))
            aux["distill_loss"] = self.indexer.distillation_loss(scores.view(batch, seq_len, NB), teacher_mass)
        return out, aux


class FovealTokenformerFFN(nn.Module):
    """Feed-forward block of two Tokenformer layers (tokenformer.py:231-283): fc1 with the gelu_l2
    activation, fc2 with softmax."""

    def __init__(self, hidden_size: int, intermediate_size: int, num_param_tokens: int = 512,
                 param_block_size: int = 64, base_blocks: int = 2, index_dim: int = 16, top_p: float = 0.95,
                 max_remote_blocks: int = 4):
        super().__init__()
        self.fc1 = FovealTokenformerLinear(in_features=hidden_size, out_features=intermediate_size,
                                           num_param_tokens=num_param_tokens, param_block_size=param_block_size,
                                           base_blocks=base_blocks, index_dim=index_dim, top_p=top_p,
                                           max_remote_blocks=max_remote_blocks, activation="gelu_l2")
        self.fc2 = FovealTokenformerLinear(in_features=intermediate_size, out_features=hidden_size,
                                           num_param_tokens=num_param_tokens, param_block_size=param_block_size,
                                           base_blocks=base_blocks, index_dim=index_dim, top_p=top_p,
                                           max_remote_blocks=max_remote_blocks, activation="softmax")

    def forward_kernels(self, x2d: Tensor) -> Tensor:
        """Both layers as one stream of kernel launches without host synchronisation: [M, hidden] ->
        [M, hidden]."""
        h = self.fc1.forward_kernels(x2d)["out"]
        return self.fc2.forward_kernels(h)["out"]

    def forward(self, x: Tensor, compute_teacher_loss: bool = False) -> Tuple[Tensor, Dict[str, Any]]:
        h, aux1 = self.fc1(x, compute_teacher_loss=compute_teacher_loss)
        out, aux2 = self.fc2(h, compute_teacher_loss=compute_teacher_loss)
        return out, {"fc1_aux": aux1, "fc2_aux": aux2, "distill_loss": aux1["distill_loss"] + aux2["distill_loss"]}
