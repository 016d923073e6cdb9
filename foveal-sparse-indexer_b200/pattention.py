"""Function-level Pattention on the CUDA library (mirrors ``foveal_indexer/pattention_triton.py``).

* ``triton_fused_swiglu(g, u)`` / ``TritonFusedSwiGLUFunction`` (:30-104): h = silu(g) * u with its
  backward, on the elementwise kernels ``fp_swiglu_fwd`` / ``fp_swiglu_bwd``.
* ``triton_pattention(x, k_gate, v, k_up=None, active_blocks=None, activation="swiglu", block_n=64)``
  (:204-277, semantics of ``_pytorch_pattention_fallback`` :280-311): one active-block list shared by
  every token, the five activations of the reference (``swiglu``, ``silu``, ``gelu``, ``relu``,
  ``relu2``), the non-gated form (``k_up=None``) and an output width ``D_out = v.shape[1]`` of its own.
  bf16 with widths that are multiples of 64 runs on the tcgen05 gate/up and down kernels (activation in
  the gate/up epilogue); fp32 and other widths on the CUDA-core kernel.  GELU is the erf form, as in the
  reference's PyTorch path (its Triton kernel's ``sin``-based approximation, :184-186, is not
  reproduced).
* ``TritonSwiGLUPattentionMLP`` (:314-375) and ``convert_llm_mlp_to_pattention`` (:378-395): the drop-in
  MLP module and the model conversion helper, with the reference's constructor, parameters,
  initialisation and ``from_dense_mlp``.

Differences from the reference, all loud: CPU tensors raise instead of falling back to PyTorch
(:225-227); an unknown activation or SwiGLU without ``k_up`` raises ``ValueError`` (the reference's
Triton path silently picks SwiGLU or a zero up projection); ``block_n`` must be 64 (the kernels' block);
``triton_pattention`` is forward-only (as the reference's fused kernel, which has no backward).
"""

from __future__ import annotations

import weakref
from collections import OrderedDict
from typing import Optional

import torch
from torch import Tensor, nn

from . import kernels
from ._lib import require_cuda

ACTIVATIONS = tuple(kernels.PATTENTION_ACTIVATIONS)


class TritonFusedSwiGLUFunction(torch.autograd.Function):
    """h = silu(g) * u with the fused backward (pattention_triton.py:79-96)."""

    @staticmethod
    def forward(ctx, g, u):
        ctx.save_for_backward(g, u)
        return kernels.swiglu_fwd(g, u)

    @staticmethod
    def backward(ctx, dh):
        g, u = ctx.saved_tensors
        dg, du, _ = kernels.swiglu_bwd(dh, g, u, want_h=False)
        return dg, du


def triton_fused_swiglu(g: Tensor, u: Tensor) -> Tensor:
    """SwiGLU of two pre-activation tensors (pattention_triton.py:98-104), differentiable."""
    require_cuda(g, u)
    return TritonFusedSwiGLUFunction.apply(g, u)


class _NoBackward(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, *inputs):
        return y

    @staticmethod
    def backward(ctx, *grads):
        raise NotImplementedError("triton_pattention is forward-only (like the reference's fused kernel); "
                                  "train through FovealPattentionMLP's pooled training path instead")


# Packed tensor-core layouts of recently used weight triples.  An entry is valid while the very tensor
# objects it was built from are alive and unmodified (weak references plus the tensors' version counters),
# so a new tensor that happens to reuse a freed address never hits a stale entry.
_PACK_CACHE: "OrderedDict[tuple, tuple]" = OrderedDict()
_PACK_CACHE_SIZE = 8


def _packed_for(k_gate: Tensor, k_up: Optional[Tensor], v: Tensor, dtype: torch.dtype):
    if dtype != torch.bfloat16:
        return None
    ts = (k_gate, k_up, v)
    key = tuple((id(t), t.data_ptr(), t._version, tuple(t.shape), t.dtype) if t is not None else None for t in ts)
    hit = _PACK_CACHE.get(key)
    if hit is not None:
        refs, packed = hit
        if all((r is None and t is None) or (r is not None and r() is t) for r, t in zip(refs, ts)):
            _PACK_CACHE.move_to_end(key)
            return packed
        del _PACK_CACHE[key]
    packed = kernels.pack_pattention_weights(k_gate.detach().to(dtype), None if k_up is None else k_up.detach().to(dtype),
                                             v.detach().to(dtype))
    _PACK_CACHE[key] = (tuple(None if t is None else weakref.ref(t) for t in ts), packed)
    while len(_PACK_CACHE) > _PACK_CACHE_SIZE:
        _PACK_CACHE.popitem(last=False)
    return packed


def _check_args(x, k_gate, v, k_up, activation, block_n):
    if block_n != 64:
        raise ValueError("the kernels use 64-token parameter blocks (block_n=64)")
    act = activation.lower()
    if act not in ACTIVATIONS:
        raise ValueError(f"unknown activation {activation!r}; expected one of {ACTIVATIONS}")
    if act == "swiglu" and k_up is None:
        raise ValueError("k_up is required for activation='swiglu'")
    if k_gate.dim() != 2 or v.dim() != 2 or k_gate.shape[0] != v.shape[0] or k_gate.shape[1] != x.shape[-1]:
        raise ValueError(f"shapes: x [..., K], k_gate [N_p, K], v [N_p, D_out]; got x {tuple(x.shape)}, "
                         f"k_gate {tuple(k_gate.shape)}, v {tuple(v.shape)}")
    if k_up is not None and k_up.shape != k_gate.shape:
        raise ValueError("k_up must have k_gate's shape")
    if k_gate.shape[0] % block_n:
        raise ValueError("the number of parameter tokens must be a multiple of block_n")
    return act


def triton_pattention(x: Tensor, k_gate: Tensor, v: Tensor, k_up: Optional[Tensor] = None,
                      active_blocks: Optional[Tensor] = None, activation: str = "swiglu", block_n: int = 64,
                      _packed=None) -> Tensor:
    """Pattention with one shared active-block list (pattention_triton.py:204-311):
    ``act(x K_gate[A]^T [, x K_up[A]^T]) V[A]`` over the rows A of ``active_blocks`` (all blocks when
    None).  x [..., K] -> [..., D_out] in x's dtype."""
    act = _check_args(x, k_gate, v, k_up, activation, block_n)
    require_cuda(x, k_gate, v, k_up, active_blocks if isinstance(active_blocks, Tensor) else None)
    if active_blocks is not None and not isinstance(active_blocks, Tensor):
        active_blocks = torch.as_tensor(active_blocks, dtype=torch.int32, device=x.device)
    shape = x.shape
    x2d = x.reshape(-1, shape[-1])
    packed = _packed if _packed is not None else _packed_for(k_gate, k_up if act == "swiglu" else None, v, x.dtype)
    y = kernels.pattention_forward(x2d.detach(), k_gate, k_up if act == "swiglu" else None, v, packed, active_blocks,
                                   act)
    y = y.reshape(*shape[:-1], v.shape[-1])
    params = [t for t in (x, k_gate, k_up, v) if t is not None and t.requires_grad]
    if torch.is_grad_enabled() and params:
        y = _NoBackward.apply(y, *params)
    return y


pattention = triton_pattention


class TritonSwiGLUPattentionMLP(nn.Module):
    """Drop-in SwiGLU MLP as non-softmax parameter attention (pattention_triton.py:314-375): parameters
    k_gate, k_up, v [num_param_tokens, hidden_dim]; ``forward(x, active_blocks=None)``."""

    def __init__(self, hidden_dim: int = 2048, num_param_tokens: int = 6144, block_size: int = 64,
                 activation: str = "swiglu", dtype: torch.dtype = torch.bfloat16):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.num_param_tokens = num_param_tokens
        self.block_size = block_size
        self.activation = activation
        self.num_blocks = num_param_tokens // block_size
        self.k_gate = nn.Parameter(torch.empty(num_param_tokens, hidden_dim, dtype=dtype))
        self.k_up = nn.Parameter(torch.empty(num_param_tokens, hidden_dim, dtype=dtype))
        self.v = nn.Parameter(torch.empty(num_param_tokens, hidden_dim, dtype=dtype))
        nn.init.normal_(self.k_gate, std=hidden_dim ** -0.5)
        nn.init.normal_(self.k_up, std=hidden_dim ** -0.5)
        nn.init.normal_(self.v, std=num_param_tokens ** -0.5)
        self._packed_w = None
        self._packed_key = None

    @classmethod
    def from_dense_mlp(cls, dense_mlp: nn.Module, block_size: int = 64) -> "TritonSwiGLUPattentionMLP":
        """Exact reparameterisation of a dense SwiGLU MLP (pattention_triton.py:348-368)."""
        hidden_dim = dense_mlp.gate_proj.in_features
        intermediate_dim = dense_mlp.gate_proj.out_features
        dtype = dense_mlp.gate_proj.weight.dtype
        device = dense_mlp.gate_proj.weight.device
        mlp = cls(hidden_dim=hidden_dim, num_param_tokens=intermediate_dim, block_size=block_size,
                  activation="swiglu", dtype=dtype).to(device)
        with torch.no_grad():
            mlp.k_gate.copy_(dense_mlp.gate_proj.weight)
            mlp.k_up.copy_(dense_mlp.up_proj.weight)
            mlp.v.copy_(dense_mlp.down_proj.weight.t())
        return mlp

    def _packed(self):
        gated = self.activation.lower() == "swiglu"
        key = tuple((p.data_ptr(), p._version) for p in (self.k_gate, self.k_up, self.v)) + (gated, self.v.dtype)
        if self._packed_key != key:
            self._packed_w = kernels.pack_pattention_weights(self.k_gate.detach(),
                                                             self.k_up.detach() if gated else None, self.v.detach())
            self._packed_key = key
        return self._packed_w

    def forward(self, x: Tensor, active_blocks: Optional[Tensor] = None) -> Tensor:
        xx = x.to(self.k_gate.dtype) if x.dtype != self.k_gate.dtype else x
        y = triton_pattention(xx, self.k_gate, self.v, k_up=self.k_up, active_blocks=active_blocks,
                              activation=self.activation, block_n=self.block_size,
                              _packed=self._packed() if xx.dtype == torch.bfloat16 else None)
        return y


def convert_llm_mlp_to_pattention(model: nn.Module, layers: Optional[list] = None, block_size: int = 64,
                                  activation: str = "swiglu") -> nn.Module:
    """Replaces the dense MLPs of a causal LM's decoder layers by ``TritonSwiGLUPattentionMLP``
    (pattention_triton.py:378-395).  As in the reference, the converted modules are SwiGLU
    (``activation`` is accepted for signature compatibility)."""
    model_layers = getattr(model, "model", model).layers
    targets = layers if layers is not None else list(range(len(model_layers)))
    for idx in targets:
        if hasattr(model_layers[idx], "mlp") and not isinstance(model_layers[idx].mlp, TritonSwiGLUPattentionMLP):
            model_layers[idx].mlp = TritonSwiGLUPattentionMLP.from_dense_mlp(model_layers[idx].mlp,
                                                                            block_size=block_size)
    return model
