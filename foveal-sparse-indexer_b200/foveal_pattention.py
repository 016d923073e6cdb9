"""``FovealPattentionMLP``: drop-in replacement of the reference module, forward on B200 kernels.

Mirrors ``foveal_indexer/foveal_pattention.py`` of the reference: same constructor arguments,
parameter names / shapes / ``state_dict`` keys (k_gate, k_up, v, q_proj_16d.weight, block_keys_16d,
out_proj_16d.weight, offsets), ``forward(x, return_router_info)``, ``from_dense_mlp``,
``set_active_blocks``, ``clear_cache`` and ``sparsify_model_with_foveal_pattention``.

Routing modes:

* ``routing="pooled"`` (default) reproduces the reference forward (foveal_pattention.py:264-352):
  eval routes once on the pooled query and caches the active set (decode reuses it); training routes
  on the token-mean of per-token scores and adds the 16-D additive stream.
* ``routing="token"`` is per-token adaptive routing: ``select_blocks`` (core.py:46-160, non-causal,
  base blocks reserved) with ``top_p`` / ``min_remote_blocks`` / ``max_remote_blocks``, the gated
  contraction over each token's own blocks (pattention_triton.py:280-311) and the additive stream.

All arithmetic runs in ``libfovealpatt.so``; CPU tensors raise (no fallback).  The forward is not
differentiable: calling ``backward`` through it raises ``NotImplementedError``.
"""

from __future__ import annotations

import math

from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from . import kernels


def _chunk_plan(M: int, ch: int) -> list:
    """Chunk sizes for the host-streamed forward: ``ch`` tokens in the middle, ``ch/4`` and ``ch/2``
    at both ends when the batch is long enough (a short first chunk starts compute early; a short last
    chunk shortens the final copy-out)."""
    ramp = [c for c in (ch // 4, ch // 2) if c >= 256]
    head, tail, left = [], [], M
    for c in ramp:
        if left <= 0:
            break
        head.append(min(c, left))
        left -= head[-1]
    for c in ramp:
        if left > ch + c:
            tail.insert(0, c)
            left -= c
    mid = []
    while left > 0:
        mid.append(min(ch, left))
        left -= mid[-1]
    return head + mid + tail


class _PooledTrain(torch.autograd.Function):
    """Training-mode pooled forward (foveal_pattention.py:290-342) with its backward.

    Forward on the library kernels: per-token router scores, active set = top-k of their token mean
    (no gradient through the selection, as in the reference), gated contraction over the active blocks
    plus the additive stream out_proj(softmax(S/T) K_16).  Backward: the fused SwiGLU backward kernel
    (``fp_swiglu_bwd``, replacing the reference's Triton ``_swiglu_bwd_kernel``, pattention_triton.py:49-96)
    between plain GEMMs over the gathered active rows, and the chain rule of the additive stream through
    the softmax, the 16-D scores and the RMSNorm of the query into q_proj, block_keys, out_proj and x."""

    @staticmethod
    def forward(ctx, module, x2d, k_gate, k_up, v, wq, k16, wout):
        packed = module._packed()
        scores, _ = kernels.router_scores(x2d, wq, k16)
        active, _ = kernels.pooled_route(None, wq, k16, base_blocks=module.base_blocks,
                                         remote_blocks=module.remote_blocks, mode=1, token_scores=scores,
                                         dtype=x2d.dtype, D=x2d.shape[1])
        _, _, c16, _ = kernels.select(scores, base_blocks=module.base_blocks, top_p=1.0, min_remote=0, max_remote=0,
                                      capacity=0, temperature=module.temperature, block_keys=k16, want_routes=False)
        y = kernels.pooled_forward(x2d, k_gate, k_up, v, packed, active, ctx16=c16, out_proj=wout)
        ctx.save_for_backward(x2d, k_gate, k_up, v, wq, k16, wout, scores, active)
        ctx.temperature = module.temperature
        ctx.block_size = module.block_size
        ctx.mark_non_differentiable(scores, active)
        return y, scores, active

    @staticmethod
    def backward(ctx, dy, _dscores, _dactive):
        x, kg, ku, v, wq, k16, wout, S, active = ctx.saved_tensors
        T, bs = ctx.temperature, ctx.block_size
        M, D = x.shape
        dt = x.dtype
        dy = dy.reshape(M, D).to(dt).contiguous()
        idx = (active.long()[:, None] * bs + torch.arange(bs, device=x.device)).flatten()
        kg_a, ku_a, v_a = kg.detach()[idx], ku.detach()[idx], v.detach()[idx]
        G = x @ kg_a.t()
        U = x @ ku_a.t()
        dG, dU, H = kernels.swiglu_bwd(dy @ v_a.t(), G, U)
        dx = (dG @ kg_a + dU @ ku_a).float()
        dkg = torch.zeros_like(kg).index_copy_(0, idx, (dG.t() @ x).to(kg.dtype))
        dku = torch.zeros_like(ku).index_copy_(0, idx, (dU.t() @ x).to(ku.dtype))
        dv = torch.zeros_like(v).index_copy_(0, idx, (H.t() @ dy).to(v.dtype))
        # additive stream and router (fp32, as the forward's router): S = rms_norm(x Wq^T) K16^T / 4
        xf, dyf = x.float(), dy.float()
        k16f, wqf, woutf = k16.detach().float(), wq.detach().float(), wout.detach().float()
        soft = torch.softmax(S / T, dim=-1)
        dwout = dyf.t() @ (soft @ k16f)
        dctx = dyf @ woutf
        dk16 = soft.t() @ dctx
        dsoft = dctx @ k16f.t()
        dS = soft * (dsoft - (dsoft * soft).sum(dim=-1, keepdim=True)) / T
        q = xf @ wqf.t()
        r = torch.rsqrt((q * q).mean(dim=-1, keepdim=True) + torch.finfo(torch.float32).eps)
        qn = q * r
        dqn = (dS @ k16f) * 0.25
        dk16 = dk16 + (dS.t() @ qn) * 0.25
        dq = r * (dqn - qn * (dqn * qn).mean(dim=-1, keepdim=True))
        dwq = dq.t() @ xf
        dx = dx + dq @ wqf
        return (None, dx.to(dt), dkg, dku, dv, dwq.to(wq.dtype), dk16.to(k16.dtype), dwout.to(wout.dtype))


class _ForwardOnly(torch.autograd.Function):
    """Attaches a backward that raises, so a training graph through the kernels fails loudly."""

    @staticmethod
    def forward(ctx, y, *inputs):
        return y

    @staticmethod
    def backward(ctx, *grads):
        raise NotImplementedError("backward is implemented for the training-mode pooled forward (the reference's "
                                  "training path); token routing is an inference path")


class FovealPattentionMLP(nn.Module):
    """Foveal block-sparse SwiGLU token-parameter attention (Pattention) layer."""

    def __init__(
        self,
        hidden_dim: int = 2048,
        intermediate_dim: int = 6144,
        block_size: int = 64,
        base_blocks: int = 4,
        remote_blocks: int = 20,
        index_dim: int = 16,
        temperature: float = 1.0,
        dtype: torch.dtype = torch.bfloat16,
        use_fused_kernel: bool = True,
        *,
        routing: str = "pooled",
        top_p: float = 0.9,
        min_remote_blocks: int = 0,
        max_remote_blocks: Optional[int] = None,
        device=None,
    ):
        super().__init__()
        if block_size != 64:
            raise ValueError("the kernels use 64-token parameter blocks (block_size=64)")
        if index_dim != 16:
            raise ValueError("the router is specialised for index_dim=16")
        if intermediate_dim % block_size:
            raise ValueError("intermediate_dim must be a multiple of block_size")
        if routing not in ("pooled", "token"):
            raise ValueError("routing must be 'pooled' or 'token'")
        self.hidden_dim = hidden_dim
        self.intermediate_dim = intermediate_dim
        self.block_size = block_size
        self.num_blocks = intermediate_dim // block_size
        self.base_blocks = base_blocks
        self.remote_blocks = remote_blocks
        self.total_active_blocks = base_blocks + remote_blocks
        self.active_channels = self.total_active_blocks * block_size
        self.index_dim = index_dim
        self.temperature = temperature
        self.dtype = dtype
        self.use_fused_kernel = use_fused_kernel
        self.routing = routing
        self.top_p = top_p
        self.min_remote_blocks = min_remote_blocks
        self.max_remote_blocks = remote_blocks if max_remote_blocks is None else max_remote_blocks

        fk = dict(dtype=dtype, device=device)
        self.k_gate = nn.Parameter(torch.empty(intermediate_dim, hidden_dim, **fk))
        self.k_up = nn.Parameter(torch.empty(intermediate_dim, hidden_dim, **fk))
        self.v = nn.Parameter(torch.empty(intermediate_dim, hidden_dim, **fk))
        self.q_proj_16d = nn.Linear(hidden_dim, index_dim, bias=False, **fk)
        self.block_keys_16d = nn.Parameter(torch.empty(self.num_blocks, index_dim, **fk))
        self.out_proj_16d = nn.Linear(index_dim, hidden_dim, bias=False, **fk)
        self.register_buffer("offsets", torch.arange(block_size, dtype=torch.int64, device=device))

        # Eval-mode routing cache (foveal_pattention.py:100-104).  The kernels read the active blocks in
        # place, so the cache holds the active block ids only; the gathered-weight attributes of the
        # reference are kept for compatibility and stay None.
        self._cached_kg = None
        self._cached_ku = None
        self._cached_v = None
        self._cached_active_blocks: Optional[Tensor] = None
        self._packed_w = None
        self._packed_key = None
        self._shard = None  # (rank, world, group) when parameter blocks are sharded
        self.reset_parameters()

    # ------------------------------------------------------------------ reference API
    def clear_cache(self) -> None:
        """Clears the cached active set (foveal_pattention.py:108-113)."""
        self._cached_kg = self._cached_ku = self._cached_v = None
        self._cached_active_blocks = None

    def set_active_blocks(self, active_blocks: Tensor) -> None:
        """Fixes the active block set used by eval/decode calls (foveal_pattention.py:115-122)."""
        self._cached_active_blocks = active_blocks.to(device=self.k_gate.device, dtype=torch.int32).contiguous()

    def reset_parameters(self) -> None:
        """Reference initialisation (foveal_pattention.py:124-131)."""
        std = self.hidden_dim ** -0.5
        nn.init.normal_(self.k_gate, std=std)
        nn.init.normal_(self.k_up, std=std)
        nn.init.normal_(self.v, std=std)
        nn.init.normal_(self.q_proj_16d.weight, std=std)
        nn.init.normal_(self.block_keys_16d, std=self.index_dim ** -0.5)
        nn.init.normal_(self.out_proj_16d.weight, std=1e-3)

    @classmethod
    def from_dense_mlp(cls, dense_mlp: nn.Module, block_size: int = 64, base_blocks: int = 4,
                       remote_blocks: int = 20, index_dim: int = 16, temperature: float = 1.0,
                       use_fused_kernel: bool = True, **kwargs) -> "FovealPattentionMLP":
        """Exact reparameterisation of a dense SwiGLU MLP (foveal_pattention.py:133-173):
        K_gate = W_gate, K_up = W_up, V = W_down^T, additive stream initialised to zero."""
        hidden_dim = dense_mlp.gate_proj.in_features
        intermediate_dim = dense_mlp.gate_proj.out_features
        dtype = dense_mlp.gate_proj.weight.dtype
        device = dense_mlp.gate_proj.weight.device
        m = cls(hidden_dim=hidden_dim, intermediate_dim=intermediate_dim, block_size=block_size,
                base_blocks=base_blocks, remote_blocks=remote_blocks, index_dim=index_dim,
                temperature=temperature, dtype=dtype, use_fused_kernel=use_fused_kernel, **kwargs).to(device)
        with torch.no_grad():
            m.k_gate = nn.Parameter(dense_mlp.gate_proj.weight.data)
            m.k_up = nn.Parameter(dense_mlp.up_proj.weight.data)
            m.v = nn.Parameter(dense_mlp.down_proj.weight.data.t().contiguous())
            nn.init.zeros_(m.out_proj_16d.weight)
        return m

    @torch.no_grad()
    def calibrate_offline_svd(self, features: Tensor, ridge_lambda: float = 1e-2) -> Dict[str, float]:
        """Offline calibration of the 16-D router on the module's GPU (foveal_pattention.py:175-255):
        q_proj_16d <- top-16 right singular vectors of the calibration tokens; block_keys_16d <- ridge
        regression of the normalised 16-D projections onto softmax(teacher block energy / T); the
        active set <- base blocks + the top ``remote_blocks`` mean calibrated scores.  Returns the
        reference's dict (explained variance of the 16 directions, initial KL, active blocks, sparsity).

        The teacher energies (the dense SwiGLU of every calibration token over every block) run on the
        gate/up tensor-core kernel for bf16 modules (``fp_block_energy``; the calibration tokens are
        taken in bf16, the module's own precision); the SVD, the 16 x 16 ridge solve and the small
        reductions are cuSOLVER / PyTorch operations on the same GPU."""
        dev = self.k_gate.device
        if dev.type != "cuda":
            raise RuntimeError("calibrate_offline_svd runs on the module's CUDA device; move the module first")
        orig_dtype = self.k_gate.dtype
        X = features.to(device=dev, dtype=torch.float32).reshape(-1, self.hidden_dim)
        _, S, Vh = torch.linalg.svd(X, full_matrices=False)
        if Vh.shape[0] < self.index_dim:
            pad = torch.randn(self.index_dim - Vh.shape[0], self.hidden_dim, device=dev)
            Vh = torch.cat([Vh, pad], dim=0)
        V16 = Vh[: self.index_dim, :].T
        self.q_proj_16d.weight.data.copy_(V16.T.to(dtype=orig_dtype))
        Z = F.rms_norm(X @ V16, (self.index_dim,))
        teacher = self._teacher_block_energy(X)
        target = F.softmax(teacher / self.temperature, dim=-1)
        reg = ridge_lambda * torch.eye(self.index_dim, device=dev)
        block_keys = torch.linalg.solve(Z.T @ Z + reg, Z.T @ target).T
        self.block_keys_16d.data.copy_(block_keys.to(dtype=orig_dtype))
        scores = (Z @ block_keys.T) / math.sqrt(self.index_dim)
        student = F.softmax(scores / self.temperature, dim=-1)
        kl = F.kl_div(student.log(), target, reduction="batchmean").item()
        mean_scores = scores.mean(dim=0)
        _, top_rem = torch.topk(mean_scores[self.base_blocks:], k=self.remote_blocks)
        calib_active = torch.cat([torch.arange(self.base_blocks, device=dev, dtype=torch.int32),
                                  (top_rem + self.base_blocks).to(torch.int32)])
        self.set_active_blocks(calib_active)
        total_var = (S ** 2).sum().item()
        top16_var = (S[: self.index_dim] ** 2).sum().item()
        return {
            "top16_explained_variance": top16_var / max(total_var, 1e-12),
            "initial_kl_divergence": kl,
            "num_blocks": self.num_blocks,
            "active_blocks": self.total_active_blocks,
            "calib_active_blocks": calib_active.tolist(),
            "sparsity_pct": (1.0 - self.total_active_blocks / self.num_blocks) * 100.0,
        }

    def _teacher_block_energy(self, X: Tensor) -> Tensor:
        """E[t, b] = mean_{j in b} |silu(x_t k_gate_j) (x_t k_up_j)| * ||v_b||_F  (foveal_pattention.py:205-216)."""
        vnorm = self.v.detach().float().view(self.num_blocks, self.block_size, self.hidden_dim).norm(dim=(1, 2))
        packed = self._packed()
        if packed is not None:
            return kernels.block_energy(X.to(torch.bfloat16), packed[0], vnorm, self.num_blocks)
        # fp32 modules (and shapes the tensor-core tiles do not cover): the same expression with cuBLAS
        A = F.silu(X @ self.k_gate.detach().float().t()) * (X @ self.k_up.detach().float().t())
        return A.abs().view(X.shape[0], self.num_blocks, self.block_size).mean(dim=-1) * vnorm

    def compute_router_scores(self, x: Tensor) -> Tensor:
        """Per-token 16-D router scores (foveal_pattention.py:257-262), computed in fp32."""
        shape = x.shape
        x2d = x.reshape(-1, shape[-1]).to(self.k_gate.dtype)
        s, _ = kernels.router_scores(x2d, self.q_proj_16d.weight.detach(), self.block_keys_16d.detach())
        return s.reshape(*shape[:-1], self.num_blocks)

    # ------------------------------------------------------------------ helpers
    def _packed(self):
        """Tensor-core weight layouts (packed gate/up rows, V^T), rebuilt whenever k_gate, k_up or v
        is replaced or modified in place; None for fp32 models (CUDA-core path)."""
        if self.v.dtype != torch.bfloat16 or self.hidden_dim % 64:
            return None
        key = tuple((p.data_ptr(), p._version) for p in (self.k_gate, self.k_up, self.v)) + (self.v.device,)
        if self._packed_w is None or self._packed_key != key:
            self._packed_w = kernels.pack_weights(self.k_gate.detach(), self.k_up.detach(), self.v.detach())
            self._packed_key = key
        return self._packed_w

    def _weights(self):
        return (self.k_gate.detach(), self.k_up.detach(), self.v.detach(), self._packed(),
                self.q_proj_16d.weight.detach(), self.block_keys_16d.detach(), self.out_proj_16d.weight.detach())

    def _attach_no_grad(self, y: Tensor, x: Tensor) -> Tensor:
        if torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in self.parameters())):
            params = [p for p in self.parameters() if p.requires_grad]
            return _ForwardOnly.apply(y, x, *params)
        return y

    # ------------------------------------------------------------------ forward
    def forward(self, x: Tensor, return_router_info: bool = False) -> Tensor | Tuple[Tensor, Dict[str, Any]]:
        orig_shape = x.shape
        D = orig_shape[-1]
        if (self.training and self.routing == "pooled" and torch.is_grad_enabled()
                and (x.requires_grad or any(p.requires_grad for p in self.parameters()))):
            return self._forward_pooled_train(x, return_router_info)
        x_in = x
        x2d = x.reshape(-1, D)
        if x2d.dtype != self.k_gate.dtype:
            x2d = x2d.to(self.k_gate.dtype)
        x2d = x2d.detach()
        if self.routing == "token":
            y, info = self._forward_token(x2d, return_router_info)
        else:
            y, info = self._forward_pooled(x2d, orig_shape, return_router_info)
        y = self._attach_no_grad(y.reshape(*orig_shape[:-1], y.shape[-1]), x_in)
        if return_router_info:
            return y, info
        return y

    def _forward_pooled_train(self, x: Tensor, return_router_info: bool):
        D = x.shape[-1]
        x2d = x.reshape(-1, D).to(self.k_gate.dtype).contiguous()
        y, scores, active = _PooledTrain.apply(self, x2d, self.k_gate, self.k_up, self.v, self.q_proj_16d.weight,
                                               self.block_keys_16d, self.out_proj_16d.weight)
        y = y.reshape(*x.shape[:-1], D)
        if return_router_info:
            return y, {"scores": scores, "active_blocks": active,
                       "sparsity": (1.0 - self.total_active_blocks / self.num_blocks) * 100.0}
        return y

    def _forward_pooled(self, x2d: Tensor, orig_shape, return_router_info: bool):
        kg, ku, v, packed, wq, k16, wout = self._weights()
        is_prefill = (len(orig_shape) >= 3 and orig_shape[-2] > 1) or (
            len(orig_shape) == 2 and orig_shape[0] > 1 and self.training)
        if not self.training and self._cached_active_blocks is not None and not is_prefill:
            y = kernels.pooled_forward(x2d, kg, ku, v, packed, self._cached_active_blocks)
            return y, {"active_blocks": self._cached_active_blocks}
        scores = None
        ctx = None
        if self.training:
            scores, _ = kernels.router_scores(x2d, wq, k16)
            active, _ = kernels.pooled_route(None, wq, k16, base_blocks=self.base_blocks,
                                             remote_blocks=self.remote_blocks, mode=1, token_scores=scores,
                                             dtype=x2d.dtype, D=x2d.shape[1])
            _, _, ctx, _ = kernels.select(scores, base_blocks=self.base_blocks, top_p=1.0, min_remote=0,
                                          max_remote=0, capacity=0, temperature=self.temperature,
                                          block_keys=k16, want_routes=False)
        else:
            if self._cached_active_blocks is None:
                active, _ = kernels.pooled_route(x2d, wq, k16, base_blocks=self.base_blocks,
                                                 remote_blocks=self.remote_blocks, mode=0)
                self.set_active_blocks(active)
            active = self._cached_active_blocks
        y = kernels.pooled_forward(x2d, kg, ku, v, packed, active, ctx16=ctx, out_proj=wout if ctx is not None else None)
        info = {}
        if return_router_info:
            if scores is None:
                scores, _ = kernels.router_scores(x2d, wq, k16)
            info = {"scores": scores, "active_blocks": active,
                    "sparsity": (1.0 - self.total_active_blocks / self.num_blocks) * 100.0}
        return y, info

    def forward_host(self, x_host: Tensor, out: Optional[Tensor] = None, chunk_tokens: int = 2048) -> Tensor:
        """Token-routed forward of a batch held in host memory.

        The batch is processed in chunks on CUDA streams of the module's device: one stream copies
        chunks in, one copies results out, and two compute streams take alternate chunks, so that the
        kernels of one chunk overlap the tail of the previous one and both copies overlap compute.  The
        first and last chunks are smaller (``chunk_tokens`` / 4, / 2) to shorten the pipeline fill and
        drain.  Tokens are routed independently, so the result equals ``forward`` on the whole batch.
        ``x_host`` (and ``out``, if given) should be pinned for the copies to overlap.  Returns the output
        in host memory; it is complete once the caller's current stream has been synchronised (the
        current stream is made to wait for the last copy).
        """
        out, done = self.forward_host_async(x_host, out, chunk_tokens)
        torch.cuda.current_stream(self.k_gate.device).wait_event(done)
        return out

    def forward_host_async(self, x_host: Tensor, out: Optional[Tensor] = None,
                           chunk_tokens: int = 2048) -> Tuple[Tensor, "torch.cuda.Event"]:
        """:meth:`forward_host` without joining the caller's stream: returns ``(out, done)`` where
        ``out`` is complete once the CUDA event ``done`` has completed (``done.synchronize()`` or a
        stream's ``wait_event``).  Consecutive calls pipeline: the copy-in of the next batch overlaps the
        last chunks of this one (the device buffers are reused as soon as the chunk that held them is
        done).  Keep ``x_host`` unchanged and do not read ``out`` until ``done``."""
        if self.routing != "token":
            raise ValueError("forward_host needs routing='token' (pooled routing pools over the whole call)")
        if x_host.is_cuda:
            raise ValueError("forward_host takes a host tensor; use forward for device tensors")
        dev = self.k_gate.device
        if dev.type != "cuda":
            raise RuntimeError("the module's parameters must be on a CUDA device")
        D = x_host.shape[-1]
        x2d = x_host.reshape(-1, D)
        M = x2d.shape[0]
        dt = self.k_gate.dtype
        if x2d.dtype != dt:
            raise TypeError(f"x must already have the module dtype {dt} for the streamed copy")
        if out is None:
            out = torch.empty(x_host.shape[:-1] + (D,), dtype=dt, pin_memory=True)
        y2d = out.reshape(-1, D)
        kg, ku, v, packed, wq, k16, wout = self._weights()
        plan = _chunk_plan(M, max(1, int(chunk_tokens)))
        ch = max(plan) if plan else 1
        nslot = max(2, int(getattr(self, "host_slots", 3)))  # device buffer pairs in flight
        hs = getattr(self, "_host_state", None)
        if hs is None or hs["device"] != dev or len(hs["x_free"]) != nslot:
            hs = {"device": dev, "streams": tuple(torch.cuda.Stream(device=dev) for _ in range(4)),
                  "bufs": None, "x_free": [None] * nslot, "y_free": [None] * nslot, "n": 0}
            self._host_state = hs
        s_in, s_out, s_c0, s_c1 = hs["streams"]
        bufs = hs["bufs"]
        if bufs is None or bufs[0].shape[0] < ch or bufs[0].shape[1] != D or bufs[0].dtype != dt:
            for s_ in hs["streams"]:  # earlier calls may still use the old buffers
                s_.synchronize()
            bufs = [torch.empty(ch, D, dtype=dt, device=dev) for _ in range(2 * nslot)]  # x slots, y slots
            hs["bufs"] = bufs
            hs["x_free"] = [None] * nslot
            hs["y_free"] = [None] * nslot
        cur = torch.cuda.current_stream(dev)
        for s_ in hs["streams"]:
            s_.wait_stream(cur)
        x_free, y_free = hs["x_free"], hs["y_free"]  # per slot: compute done / copy-out done
        c0 = 0
        for n in plan:
            i = hs["n"]
            hs["n"] += 1
            slot = i % nslot
            s_cmp = s_c0 if i % 2 == 0 else s_c1
            xb, yb = bufs[slot][:n], bufs[nslot + slot][:n]
            with torch.cuda.stream(s_in):
                if x_free[slot] is not None:
                    s_in.wait_event(x_free[slot])
                xb.copy_(x2d[c0:c0 + n], non_blocking=True)
                e_in = torch.cuda.Event()
                e_in.record(s_in)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(e_in)
                if y_free[slot] is not None:
                    s_cmp.wait_event(y_free[slot])
                kernels.token_forward(xb, kg, ku, v, packed, wq, k16, wout, base_blocks=self.base_blocks,
                                      top_p=self.top_p, min_remote=self.min_remote_blocks,
                                      max_remote=self.max_remote_blocks, temperature=self.temperature,
                                      additive=True, y=yb)
                e_cmp = torch.cuda.Event()
                e_cmp.record(s_cmp)
                x_free[slot] = e_cmp
            with torch.cuda.stream(s_out):
                s_out.wait_event(e_cmp)
                y2d[c0:c0 + n].copy_(yb, non_blocking=True)
                e_out = torch.cuda.Event()
                e_out.record(s_out)
                y_free[slot] = e_out
            c0 += n
        done = torch.cuda.Event()
        done.record(s_out)
        return out, done

    def _forward_token(self, x2d: Tensor, return_router_info: bool):
        kg, ku, v, packed, wq, k16, wout = self._weights()
        if self._shard is not None:
            from .sharding import sharded_token_forward
            y, ridx, cnt, S = sharded_token_forward(self, x2d, want_routes=return_router_info)
        else:
            y, ridx, cnt, S = kernels.token_forward(
                x2d, kg, ku, v, packed, wq, k16, wout, base_blocks=self.base_blocks, top_p=self.top_p,
                min_remote=self.min_remote_blocks, max_remote=self.max_remote_blocks,
                temperature=self.temperature, additive=True, want_routes=return_router_info)
        info = {}
        if return_router_info:
            info = {"scores": S, "remote_indices": ridx, "remote_counts": cnt,
                    "active_blocks": None,
                    "sparsity": (1.0 - (self.base_blocks + cnt.float().mean()) / self.num_blocks) * 100.0}
        return y, info


def sparsify_model_with_foveal_pattention(
    model: nn.Module,
    layers_to_sparsify: Optional[List[int]] = None,
    block_size: int = 64,
    base_blocks: int = 4,
    remote_blocks: int = 20,
    index_dim: int = 16,
    temperature: float = 1.0,
    use_fused_kernel: bool = True,
    **kwargs,
) -> nn.Module:
    """Replaces the MLPs of a causal LM's decoder layers (foveal_pattention.py:355-387)."""
    layers = getattr(model, "model", model).layers
    targets = layers_to_sparsify if layers_to_sparsify is not None else list(range(len(layers)))
    for idx in targets:
        if hasattr(layers[idx], "mlp"):
            dense_mlp = layers[idx].mlp
            layers[idx].mlp = FovealPattentionMLP.from_dense_mlp(
                dense_mlp, block_size=block_size, base_blocks=base_blocks, remote_blocks=remote_blocks,
                index_dim=index_dim, temperature=temperature, use_fused_kernel=use_fused_kernel, **kwargs)
            del dense_mlp
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return model
