"""Functional wrappers of the C-ABI entry points (one call = one ``fp_*`` entry point).

These are the operator layer the module classes are built on.  Each function validates its tensors
(CUDA, dtype, contiguity), allocates its outputs with torch, passes the current stream and raises
``FovealKernelError`` on a non-zero status.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import check, contig, dtype_code, ptr, require_cuda, stream_handle


def router_scores(x2d: torch.Tensor, q_proj: torch.Tensor, block_keys: torch.Tensor,
                  want_q16: bool = False) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """``rms_norm(x W_q^T) K_16^T / 4`` per token (foveal_pattention.py:257-262); fp32 [M, NB]."""
    dev = require_cuda(x2d, q_proj, block_keys)
    dt = dtype_code(x2d.dtype)
    x2d, q_proj, block_keys = contig(x2d), contig(q_proj.to(x2d.dtype)), contig(block_keys.to(x2d.dtype))
    M, D = x2d.shape
    NB = block_keys.shape[0]
    scores = torch.empty(M, NB, dtype=torch.float32, device=dev)
    q16 = torch.empty(M, 16, dtype=torch.float32, device=dev) if want_q16 else None
    rc = _lib.load().fp_router_scores(ptr(x2d), ptr(q_proj), ptr(block_keys), dt, M, D, NB, ptr(scores),
                                      ptr(q16), stream_handle(dev))
    check(rc, "fp_router_scores")
    return scores, q16


def select(scores: torch.Tensor, *, base_blocks: int, top_p: float, min_remote: int, max_remote: int,
           capacity: int, temperature: float = 1.0, block_keys: Optional[torch.Tensor] = None,
           want_stats: bool = False, want_routes: bool = True):
    """Top-p block selection (core.py:46-160, non-causal) and optionally the additive-stream context.

    Returns (remote_indices [M, capacity] int32, remote_counts [M] int32, ctx16 [M, 16] fp32 or None,
    stats [3] fp32 or None)."""
    dev = require_cuda(scores)
    scores = contig(scores.float())
    M, NB = scores.shape
    idx = cnt = None
    if want_routes:
        idx = torch.empty(M, capacity, dtype=torch.int32, device=dev)
        cnt = torch.empty(M, dtype=torch.int32, device=dev)
    k16f = ctx = None
    if block_keys is not None:
        k16f = contig(block_keys.detach().float())
        ctx = torch.empty(M, 16, dtype=torch.float32, device=dev)
    stats = torch.zeros(3, dtype=torch.float32, device=dev) if want_stats else None
    rc = _lib.load().fp_select_blocks(ptr(scores), M, NB, int(base_blocks), float(top_p), int(min_remote),
                                      int(max_remote), int(capacity) if want_routes else 0, float(temperature),
                                      ptr(idx), ptr(cnt), ptr(k16f), ptr(ctx), ptr(stats), stream_handle(dev))
    check(rc, "fp_select_blocks")
    return idx, cnt, ctx, stats


def pooled_route(x2d: Optional[torch.Tensor], q_proj: torch.Tensor, block_keys: torch.Tensor, *,
                 base_blocks: int, remote_blocks: int, mode: int,
                 token_scores: Optional[torch.Tensor] = None, dtype: Optional[torch.dtype] = None,
                 M: Optional[int] = None, D: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Pooled routing (foveal_pattention.py:292-303 train / :310-321 eval): (active int32, pooled scores)."""
    dev = require_cuda(q_proj, block_keys, x2d, token_scores)
    dt_t = dtype or (x2d.dtype if x2d is not None else q_proj.dtype)
    dt = dtype_code(dt_t)
    q_proj, block_keys = contig(q_proj.to(dt_t)), contig(block_keys.to(dt_t))
    NB = block_keys.shape[0]
    if x2d is not None:
        x2d = contig(x2d)
        M, D = x2d.shape
    if token_scores is not None:
        token_scores = contig(token_scores.float())
        M = token_scores.shape[0]
    D = D if D is not None else q_proj.shape[1]
    active = torch.empty(base_blocks + remote_blocks, dtype=torch.int32, device=dev)
    mean_scores = torch.empty(NB, dtype=torch.float32, device=dev)
    lib = _lib.load()
    nbytes = lib.fp_pooled_workspace_size(dt, M, D, NB, 0)
    ws = _lib.workspace(dev, nbytes)
    rc = lib.fp_pooled_route(ptr(x2d), ptr(q_proj), ptr(block_keys), dt, M, D, NB, int(base_blocks),
                             int(remote_blocks), int(mode), ptr(token_scores), ptr(active), ptr(mean_scores),
                             ptr(ws), ws.numel(), stream_handle(dev))
    check(rc, "fp_pooled_route")
    return active, mean_scores


def pack_weights(k_gate: torch.Tensor, k_up: torch.Tensor, v: torch.Tensor):
    """Derived tensor-core layouts (``fp_pack_weights``), both tile-contiguous: packed gate/up rows
    (2 Np x D elements) and V^T (ceil(D / 256) * 256 x Np elements).  bf16 only; opaque buffers for the
    forward entry points."""
    dev = require_cuda(k_gate, k_up, v)
    k_gate, k_up, v = contig(k_gate.detach()), contig(k_up.detach()), contig(v.detach())
    Np, D = v.shape
    w_gu = torch.empty(2 * Np, D, dtype=v.dtype, device=dev)
    vt = torch.empty((D + 255) // 256 * 256, Np, dtype=v.dtype, device=dev)
    rc = _lib.load().fp_pack_weights(ptr(k_gate), ptr(k_up), ptr(v), dtype_code(v.dtype), Np, D, ptr(w_gu),
                                     ptr(vt), stream_handle(dev))
    check(rc, "fp_pack_weights")
    return w_gu, vt


def block_energy(x2d: torch.Tensor, w_gu: torch.Tensor, vnorm: torch.Tensor, num_blocks: int) -> torch.Tensor:
    """Teacher block energies of the offline calibration (``fp_block_energy``): [M, NB] fp32 with
    E[t, b] = mean over block b's channels of |silu(gate) * up| times ``vnorm[b]``.  bf16 x and packed
    weights (:func:`pack_weights`)."""
    dev = require_cuda(x2d, w_gu, vnorm)
    x2d = contig(x2d)
    vnorm = contig(vnorm.float())
    M, D = x2d.shape
    E = torch.empty(M, num_blocks, dtype=torch.float32, device=dev)
    lib = _lib.load()
    ws = _lib.workspace(dev, lib.fp_block_energy_workspace_size(M, num_blocks))
    rc = lib.fp_block_energy(ptr(x2d), M, D, num_blocks, dtype_code(x2d.dtype), ptr(w_gu), ptr(vnorm), ptr(E),
                             ptr(ws), ws.numel(), stream_handle(dev))
    check(rc, "fp_block_energy")
    return E


def swiglu_bwd(dout: torch.Tensor, g: torch.Tensor, u: torch.Tensor, want_h: bool = True):
    """Fused SwiGLU backward (``fp_swiglu_bwd``): returns (dg, du, h or None), same dtype as ``g``."""
    dev = require_cuda(dout, g, u)
    dout, g, u = contig(dout.to(g.dtype)), contig(g), contig(u)
    dg, du = torch.empty_like(g), torch.empty_like(g)
    h = torch.empty_like(g) if want_h else None
    rc = _lib.load().fp_swiglu_bwd(ptr(dout), ptr(g), ptr(u), dtype_code(g.dtype), g.numel(), ptr(dg), ptr(du), ptr(h),
                                   stream_handle(dev))
    check(rc, "fp_swiglu_bwd")
    return dg, du, h


def swiglu_fwd(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """h = silu(g) * u (``fp_swiglu_fwd``), same dtype and shape as ``g``."""
    dev = require_cuda(g, u)
    if g.shape != u.shape:
        raise ValueError(f"g and u must have the same shape, got {tuple(g.shape)} and {tuple(u.shape)}")
    g, u = contig(g), contig(u.to(g.dtype))
    h = torch.empty_like(g)
    check(_lib.load().fp_swiglu_fwd(ptr(g), ptr(u), dtype_code(g.dtype), g.numel(), ptr(h), stream_handle(dev)),
          "fp_swiglu_fwd")
    return h


PATTENTION_ACTIVATIONS = {"swiglu": 0, "silu": 1, "gelu": 2, "relu": 3, "relu2": 4}


def pack_pattention_weights(k_gate: torch.Tensor, k_up: Optional[torch.Tensor], v: torch.Tensor):
    """Tensor-core layouts of a function-level Pattention's weights (``fp_pack_pattention_weights``):
    (w_gu [2 Np, K], v_t [ceil(D_out / 256) * 256, Np]); None when the shape or dtype runs on CUDA cores."""
    Np, K = k_gate.shape
    D_out = v.shape[1]
    if v.dtype != torch.bfloat16 or K % 64 or D_out % 64 or Np % 64:
        return None
    dev = require_cuda(k_gate, k_up, v)
    kg, v = contig(k_gate.detach()), contig(v.detach())
    ku = contig(k_up.detach().to(v.dtype)) if k_up is not None else None
    w_gu = torch.empty(2 * Np, K, dtype=v.dtype, device=dev)
    vt = torch.empty((D_out + 255) // 256 * 256, Np, dtype=v.dtype, device=dev)
    rc = _lib.load().fp_pack_pattention_weights(ptr(kg.to(v.dtype)), ptr(ku), ptr(v), dtype_code(v.dtype), Np, K,
                                                D_out, ptr(w_gu), ptr(vt), stream_handle(dev))
    check(rc, "fp_pack_pattention_weights")
    return w_gu, vt


def pattention_forward(x2d: torch.Tensor, k_gate: torch.Tensor, k_up: Optional[torch.Tensor], v: torch.Tensor,
                       packed, active: Optional[torch.Tensor], activation: str) -> torch.Tensor:
    """Function-level Pattention over one shared active list (``fp_pattention_fwd``): y [M, D_out] in x's
    dtype.  ``packed`` from :func:`pack_pattention_weights` (or None: CUDA cores)."""
    dev = require_cuda(x2d, k_gate, v, k_up, active)
    dtt = x2d.dtype
    x2d = contig(x2d)
    M, K = x2d.shape
    Np, D_out = v.shape
    kg, v = contig(k_gate.detach().to(dtt)), contig(v.detach().to(dtt))
    ku = contig(k_up.detach().to(dtt)) if k_up is not None else None
    act = contig(active.to(torch.int32)) if active is not None else None
    n_active = act.numel() if act is not None else Np // 64
    y = torch.empty(M, D_out, dtype=dtt, device=dev)
    lib = _lib.load()
    code = dtype_code(dtt)
    ws = _lib.workspace(dev, lib.fp_pattention_workspace_size(code, M, K, Np, D_out, n_active))
    w_gu, v_t = packed if packed is not None else (None, None)
    rc = lib.fp_pattention_fwd(ptr(x2d), M, K, Np, D_out, code, ptr(kg), ptr(ku), ptr(v), ptr(w_gu), ptr(v_t),
                               ptr(act), n_active, PATTENTION_ACTIVATIONS[activation], ptr(y), ptr(ws), ws.numel(),
                               stream_handle(dev))
    check(rc, "fp_pattention_fwd")
    return y


def token_forward(x2d, k_gate, k_up, v, packed, q_proj, block_keys, out_proj, *, base_blocks: int,
                  top_p: float, min_remote: int, max_remote: int, temperature: float = 1.0,
                  additive: bool = True, block_stride: int = 1, block_offset: int = 0,
                  out_f32: bool = False, want_routes: bool = False, y: Optional[torch.Tensor] = None):
    """Per-token routed forward, one ``fp_pattention_token_fwd`` call.

    ``packed`` is (w_gu, v_t) from :func:`pack_weights` (bf16) or None (fp32 CUDA-core path).
    Returns (y [M, D], remote_indices or None, remote_counts or None, scores or None)."""
    dev = require_cuda(x2d, k_gate, k_up, v, q_proj, block_keys)
    dtt = x2d.dtype
    dt = dtype_code(dtt)
    x2d = contig(x2d)
    M, D = x2d.shape
    NB = block_keys.shape[0]
    k_gate, k_up, v = contig(k_gate.detach()), contig(k_up.detach()), contig(v.detach())
    q_proj, block_keys = contig(q_proj.detach().to(dtt)), contig(block_keys.detach().to(dtt))
    out_proj = contig(out_proj.detach().to(dtt)) if out_proj is not None else None
    if y is None:
        y = torch.empty(M, D, dtype=torch.float32 if out_f32 else dtt, device=dev)
    cap = max(int(max_remote), 1)
    w_gu, v_t = packed if packed is not None else (None, None)
    ridx = cnt = S = None
    if want_routes:
        ridx = torch.empty(M, cap, dtype=torch.int32, device=dev)
        cnt = torch.empty(M, dtype=torch.int32, device=dev)
        S = torch.empty(M, NB, dtype=torch.float32, device=dev)
    lib = _lib.load()
    nbytes = lib.fp_token_workspace_size(dt, M, D, NB, int(base_blocks), int(max_remote), int(block_stride))
    ws = _lib.workspace(dev, nbytes)
    rc = lib.fp_pattention_token_fwd(
        ptr(x2d), M, D, NB, dt, ptr(k_gate), ptr(k_up), ptr(v), ptr(w_gu), ptr(v_t), ptr(q_proj), ptr(block_keys),
        ptr(out_proj), int(base_blocks), float(top_p), int(min_remote), int(max_remote), float(temperature),
        1 if additive else 0, int(block_stride), int(block_offset), ptr(y), 1 if out_f32 else 0, ptr(ridx),
        ptr(cnt), ptr(S), ptr(ws), ws.numel(), stream_handle(dev))
    check(rc, "fp_pattention_token_fwd")
    return y, ridx, cnt, S


def route_tokens(x2d, q_proj, block_keys, *, base_blocks: int, top_p: float, min_remote: int, max_remote: int,
                 temperature: float = 1.0, want_ctx: bool = True):
    """Routing only (``fp_route_tokens``): (remote_indices [M, max(K_max, 1)] int32, remote_counts [M] int32,
    ctx16 [M, 16] fp32 or None) of the token-routed forward."""
    dev = require_cuda(x2d, q_proj, block_keys)
    dtt = x2d.dtype
    x2d = contig(x2d)
    M, D = x2d.shape
    NB = block_keys.shape[0]
    q_proj, block_keys = contig(q_proj.detach().to(dtt)), contig(block_keys.detach().to(dtt))
    cap = max(int(max_remote), 1)
    ridx = torch.empty(M, cap, dtype=torch.int32, device=dev)
    cnt = torch.empty(M, dtype=torch.int32, device=dev)
    ctx = torch.empty(M, 16, dtype=torch.float32, device=dev) if want_ctx else None
    lib = _lib.load()
    ws = _lib.workspace(dev, lib.fp_route_workspace_size(M))
    rc = lib.fp_route_tokens(ptr(x2d), M, D, NB, dtype_code(dtt), ptr(q_proj), ptr(block_keys), int(base_blocks),
                             float(top_p), int(min_remote), int(max_remote), float(temperature), ptr(ridx), ptr(cnt),
                             ptr(ctx), None, ptr(ws), ws.numel(), stream_handle(dev))
    check(rc, "fp_route_tokens")
    return ridx, cnt, ctx


def routed_forward(x2d, k_gate, k_up, v, packed, out_proj, remote_indices, remote_counts, ctx16, *,
                   base_blocks: int, block_stride: int = 1, block_offset: int = 0, out_f32: bool = False,
                   y: Optional[torch.Tensor] = None):
    """Contraction of the blocks ``b % block_stride == block_offset`` from given routes
    (``fp_pattention_routed_fwd``): y [M, D] (fp32 when ``out_f32``) plus ctx16 . W_out^T where ctx16 is
    given (rows of zeros add nothing)."""
    dev = require_cuda(x2d, k_gate, k_up, v, remote_indices, remote_counts)
    dtt = x2d.dtype
    dt = dtype_code(dtt)
    x2d = contig(x2d)
    M, D = x2d.shape
    NB = k_gate.shape[0] // 64
    k_gate, k_up, v = contig(k_gate.detach()), contig(k_up.detach()), contig(v.detach())
    out_proj = contig(out_proj.detach().to(dtt)) if out_proj is not None else None
    ridx = contig(remote_indices.to(torch.int32))
    cnt = contig(remote_counts.to(torch.int32))
    ctx16 = contig(ctx16.float()) if ctx16 is not None else None
    cap = ridx.shape[1]
    if y is None:
        y = torch.empty(M, D, dtype=torch.float32 if out_f32 else dtt, device=dev)
    w_gu, v_t = packed if packed is not None else (None, None)
    lib = _lib.load()
    ws = _lib.workspace(dev, lib.fp_token_workspace_size(dt, M, D, NB, int(base_blocks), cap, int(block_stride)))
    rc = lib.fp_pattention_routed_fwd(ptr(x2d), M, D, NB, dt, ptr(k_gate), ptr(k_up), ptr(v), ptr(w_gu), ptr(v_t),
                                      ptr(out_proj), int(base_blocks), cap, ptr(ridx), ptr(cnt), ptr(ctx16),
                                      int(block_stride), int(block_offset), ptr(y), 1 if out_f32 else 0, ptr(ws),
                                      ws.numel(), stream_handle(dev))
    check(rc, "fp_pattention_routed_fwd")
    return y


# ---------------------------------------------------------------- peer-memory reduce-scatter
PEER_HANDLE_BYTES = 64
PEER_FLAG_BYTES = 256


def peer_alloc(nbytes: int) -> Tuple[int, bytes]:
    """A zeroed device buffer shared through CUDA IPC (``fp_peer_alloc``): (device address, handle)."""
    p = ctypes.c_void_p()
    h = ctypes.create_string_buffer(PEER_HANDLE_BYTES)
    check(_lib.load().fp_peer_alloc(int(nbytes), ctypes.byref(p), h), "fp_peer_alloc")
    return int(p.value), h.raw


def peer_open(handle: bytes) -> int:
    """Maps another process's :func:`peer_alloc` buffer (``fp_peer_open``): its address in this process."""
    p = ctypes.c_void_p()
    check(_lib.load().fp_peer_open(ctypes.create_string_buffer(bytes(handle), PEER_HANDLE_BYTES), ctypes.byref(p)),
          "fp_peer_open")
    return int(p.value)


def peer_close(addr: int) -> None:
    check(_lib.load().fp_peer_close(ctypes.c_void_p(addr)), "fp_peer_close")


def peer_free(addr: int) -> None:
    check(_lib.load().fp_peer_free(ctypes.c_void_p(addr)), "fp_peer_free")


def routed_peer_forward(x2d, k_gate, k_up, v, packed, out_proj, remote_indices, remote_counts, ctx16, *,
                        base_blocks: int, block_stride: int, block_offset: int, peer_out, peer_flags,
                        rows_per_rank: int, epoch: int, out_f32: bool = False, capacity: int = 0) -> bool:
    """:func:`routed_forward` whose output rows go straight to the ranks that own them
    (``fp_pattention_routed_peer_fwd``): ``peer_out[o]`` / ``peer_flags[o]`` are device addresses (this
    rank's receive slot and flag word on rank o).  ``remote_indices`` / ``remote_counts``: int32 tensors, or
    device addresses of [M, capacity] / [M] int32 tables (the peer route exchange's buffers).  Returns
    False, having launched nothing, for shapes whose contraction is split (small batches): the caller uses
    the collective instead."""
    dev = require_cuda(x2d, k_gate, k_up, v)
    dtt = x2d.dtype
    dt = dtype_code(dtt)
    x2d = contig(x2d)
    M, D = x2d.shape
    NB = k_gate.shape[0] // 64
    world = len(peer_out)
    k_gate, k_up, v = contig(k_gate.detach()), contig(k_up.detach()), contig(v.detach())
    out_proj = contig(out_proj.detach().to(dtt)) if out_proj is not None else None
    if isinstance(remote_indices, int):
        ridx, cnt, cap = ctypes.c_void_p(remote_indices), ctypes.c_void_p(remote_counts), int(capacity)
    else:
        ridx_t = contig(remote_indices.to(torch.int32))
        cnt_t = contig(remote_counts.to(torch.int32))
        ridx, cnt, cap = ptr(ridx_t), ptr(cnt_t), ridx_t.shape[1]
    ctx16 = contig(ctx16.float()) if ctx16 is not None else None
    w_gu, v_t = packed if packed is not None else (None, None)
    outs = (ctypes.c_void_p * world)(*peer_out)
    flags = (ctypes.c_void_p * world)(*peer_flags)
    lib = _lib.load()
    ws = _lib.workspace(dev, lib.fp_token_workspace_size(dt, M, D, NB, int(base_blocks), cap, int(block_stride)))
    rc = lib.fp_pattention_routed_peer_fwd(ptr(x2d), M, D, NB, dt, ptr(k_gate), ptr(k_up), ptr(v), ptr(w_gu),
                                           ptr(v_t), ptr(out_proj), int(base_blocks), cap, ridx, cnt,
                                           ptr(ctx16), int(block_stride), int(block_offset), outs, flags, world,
                                           int(rows_per_rank), int(epoch) & 0xFFFFFFFF, 1 if out_f32 else 0, ptr(ws),
                                           ws.numel(), stream_handle(dev))
    if rc == _lib.FP_ERR_UNSUPPORTED:
        return False
    check(rc, "fp_pattention_routed_peer_fwd")
    return True


def peer_reduce_supported(dtype: torch.dtype, M: int, D: int, NB: int, capacity: int, block_stride: int) -> bool:
    """Whether :func:`routed_peer_forward` takes this shape (``fp_peer_reduce_supported``)."""
    return bool(_lib.load().fp_peer_reduce_supported(dtype_code(dtype), int(M), int(D), int(NB), int(capacity),
                                                      int(block_stride)))


def peer_put(src: torch.Tensor, dst) -> None:
    """The bytes of ``src`` (contiguous, 16-byte multiple) to every device address of ``dst``
    (``fp_peer_put``)."""
    dev = require_cuda(src)
    src = contig(src)
    n = src.numel() * src.element_size()
    arr = (ctypes.c_void_p * len(dst))(*dst)
    check(_lib.load().fp_peer_put(ptr(src), n, arr, len(dst), stream_handle(dev)), "fp_peer_put")


def peer_signal(flags, epoch: int, device) -> None:
    """This rank's flag word on every rank (device addresses) := epoch (``fp_peer_signal``)."""
    arr = (ctypes.c_void_p * len(flags))(*flags)
    check(_lib.load().fp_peer_signal(arr, len(flags), int(epoch) & 0xFFFFFFFF, stream_handle(torch.device(device))),
          "fp_peer_signal")


def peer_wait(flags_addr: int, world: int, epoch: int, err_ws: torch.Tensor) -> None:
    """Orders the stream's later work after every flag of the array at ``flags_addr`` reached ``epoch``
    (``fp_peer_wait``; bounded, its error word in ``err_ws``)."""
    check(_lib.load().fp_peer_wait(ctypes.c_void_p(flags_addr), int(world), int(epoch) & 0xFFFFFFFF, ptr(err_ws),
                                   err_ws.numel(), stream_handle(err_ws.device)), "fp_peer_wait")


def peer_combine(recv_addr: int, flags_addr: int, world: int, rows: int, D: int, *, in_f32: bool, epoch: int,
                 out_dtype: torch.dtype, err_ws: torch.Tensor) -> torch.Tensor:
    """This rank's rows summed over the world slots of its receive buffer once every rank's flag reached
    ``epoch`` (``fp_peer_combine``): y [rows, D].  ``err_ws``: a device buffer of at least 256 bytes of its
    own (the combine's error word; ``_lib.device_error(err_ws)`` reads it)."""
    dev = err_ws.device
    y = torch.empty(rows, D, dtype=out_dtype, device=dev)
    ws = err_ws
    rc = _lib.load().fp_peer_combine(ctypes.c_void_p(recv_addr), ctypes.c_void_p(flags_addr), int(world), int(rows),
                                     int(D), 1 if in_f32 else 0, int(epoch) & 0xFFFFFFFF, ptr(y),
                                     1 if out_dtype == torch.float32 else 0, ptr(ws), ws.numel(), stream_handle(dev))
    check(rc, "fp_peer_combine")
    return y


def pooled_forward(x2d, k_gate, k_up, v, packed, active, *, ctx16=None, out_proj=None, out_f32: bool = False):
    """Forward over one shared active set (``fp_pattention_pooled_fwd``); y [M, D].  ``packed`` as in
    :func:`token_forward`."""
    dev = require_cuda(x2d, k_gate, k_up, v, active)
    dtt = x2d.dtype
    dt = dtype_code(dtt)
    x2d = contig(x2d)
    M, D = x2d.shape
    NB = k_gate.shape[0] // 64
    k_gate, k_up, v = contig(k_gate.detach()), contig(k_up.detach()), contig(v.detach())
    active = contig(active.to(torch.int32))
    out_proj = contig(out_proj.detach().to(dtt)) if out_proj is not None else None
    y = torch.empty(M, D, dtype=torch.float32 if out_f32 else dtt, device=dev)
    lib = _lib.load()
    n_active = active.numel()
    nbytes = lib.fp_pooled_workspace_size(dt, M, D, NB, n_active)
    ws = _lib.workspace(dev, nbytes)
    w_gu, v_t = packed if packed is not None else (None, None)
    rc = lib.fp_pattention_pooled_fwd(ptr(x2d), M, D, NB, dt, ptr(k_gate), ptr(k_up), ptr(v), ptr(w_gu), ptr(v_t),
                                      ptr(active), n_active, ptr(ctx16), ptr(out_proj), ptr(y),
                                      1 if out_f32 else 0, ptr(ws), ws.numel(), stream_handle(dev))
    check(rc, "fp_pattention_pooled_fwd")
    return y


# ---------------------------------------------------------------------------------------------------
# Union-contraction layers (BlockSparseLinear, FovealTokenformerLinear)
# ---------------------------------------------------------------------------------------------------

def param_blocks_16d(P: torch.Tensor, k_proj: torch.Tensor, v_proj: torch.Tensor):
    """Pooled 16-D key (normalised) and value of every 64-row block of ``P`` (``fp_param_blocks_16d``;
    core.py:225-252, block_matmul.py:107-127).  Returns fp32 (k_blocks [N/64, 16], v_blocks [N/64, 16])."""
    dev = require_cuda(P, k_proj, v_proj)
    dtt = P.dtype
    P, k_proj, v_proj = contig(P.detach()), contig(k_proj.detach().to(dtt)), contig(v_proj.detach().to(dtt))
    N, D = P.shape
    kb = torch.empty(N // 64, 16, dtype=torch.float32, device=dev)
    vb = torch.empty(N // 64, 16, dtype=torch.float32, device=dev)
    rc = _lib.load().fp_param_blocks_16d(ptr(P), ptr(k_proj), ptr(v_proj), dtype_code(dtt), N, D, ptr(kb), ptr(vb),
                                         stream_handle(dev))
    check(rc, "fp_param_blocks_16d")
    return kb, vb


def cosine_block_scores(x2d: torch.Tensor, q_proj: torch.Tensor, k_blocks: torch.Tensor,
                        want_q16: bool = False) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """``normalize(rms_norm(x W_q^T)) . normalize(k_blocks)^T / 4`` (``fp_cosine_block_scores``;
    core.py:214-223 then :254-266); fp32 [M, NB]."""
    dev = require_cuda(x2d, q_proj, k_blocks)
    x2d, q_proj = contig(x2d), contig(q_proj.detach().to(x2d.dtype))
    k_blocks = contig(k_blocks.detach().float())
    M, D = x2d.shape
    NB = k_blocks.shape[0]
    scores = torch.empty(M, NB, dtype=torch.float32, device=dev)
    q16 = torch.empty(M, 16, dtype=torch.float32, device=dev) if want_q16 else None
    rc = _lib.load().fp_cosine_block_scores(ptr(x2d), ptr(q_proj), ptr(k_blocks), dtype_code(x2d.dtype), M, D, NB,
                                            ptr(scores), ptr(q16), stream_handle(dev))
    check(rc, "fp_cosine_block_scores")
    return scores, q16


def select_remote_top_p(scores: torch.Tensor, *, base_blocks: int, top_p: float, max_remote: int,
                        want_stats: bool = False):
    """BlockSparseLinear's inference selection (``fp_select_remote_top_p``; block_matmul.py:185-201).
    Returns (remote_indices [M, cap] int32 absolute ids, remote_counts [M] int32, stats [3] or None) with
    cap = min(max_remote, NB - base) (at least 1)."""
    dev = require_cuda(scores)
    scores = contig(scores.float())
    M, NB = scores.shape
    cap = max(1, min(int(max_remote), NB - int(base_blocks)))
    idx = torch.empty(M, cap, dtype=torch.int32, device=dev)
    cnt = torch.empty(M, dtype=torch.int32, device=dev)
    stats = torch.zeros(3, dtype=torch.float32, device=dev) if want_stats else None
    rc = _lib.load().fp_select_remote_top_p(ptr(scores), M, NB, int(base_blocks), float(top_p), int(max_remote), cap,
                                            ptr(idx), ptr(cnt), ptr(stats), stream_handle(dev))
    check(rc, "fp_select_remote_top_p")
    return idx, cnt, stats


def union_blocks(remote_indices: torch.Tensor, remote_counts: torch.Tensor, num_blocks: int, base_blocks: int):
    """Union of the selected blocks (``fp_union_blocks``): (blocks [NB] int32, n_active [1] int32), both on
    the device; blocks[:n] are the selected ids ascending, blocks[n:] the others ascending."""
    dev = require_cuda(remote_indices, remote_counts)
    idx = contig(remote_indices.reshape(-1, remote_indices.shape[-1]).to(torch.int32))
    cnt = contig(remote_counts.reshape(-1).to(torch.int32))
    blocks = torch.empty(num_blocks, dtype=torch.int32, device=dev)
    n_active = torch.empty(1, dtype=torch.int32, device=dev)
    rc = _lib.load().fp_union_blocks(ptr(idx), ptr(cnt), cnt.numel(), idx.shape[1], int(num_blocks), int(base_blocks),
                                     ptr(blocks), ptr(n_active), stream_handle(dev))
    check(rc, "fp_union_blocks")
    return blocks, n_active


def pack_blocked_weight(weight: torch.Tensor) -> torch.Tensor:
    """64 x 64 blocked copy of a bf16 weight [rows, cols] (``fp_pack_blocked_weight``): a flat bf16 tensor
    whose tile (kb, j) (rows j*64.., columns kb*64..) is one contiguous 8 KB run at tile kb * rows/64 + j."""
    dev = require_cuda(weight)
    if weight.dtype != torch.bfloat16 or weight.dim() != 2:
        raise ValueError("pack_blocked_weight: a 2-D bf16 weight")
    w = contig(weight.detach())
    out = torch.empty(w.numel(), dtype=torch.bfloat16, device=dev)
    rc = _lib.load().fp_pack_blocked_weight(ptr(w), w.shape[0], w.shape[1], ptr(out), stream_handle(dev))
    check(rc, "fp_pack_blocked_weight")
    return out


def block_sparse_linear(x2d: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], blocks: torch.Tensor,
                        n_active: torch.Tensor, ctx16: Optional[torch.Tensor] = None,
                        out_proj: Optional[torch.Tensor] = None, max_active: int = 0,
                        weight_blocked: Optional[torch.Tensor] = None) -> torch.Tensor:
    """BlockSparseLinear contraction over the union (``fp_block_sparse_linear_fwd``;
    block_matmul.py:233-254): out [M, out_features] in x's dtype.  ``max_active``: a host-side upper
    bound of the union size (0 = all blocks), which lets small batches split the contraction.
    ``weight_blocked``: the weight's :func:`pack_blocked_weight` copy, read by the tensor cores instead of
    the row-major weight (``fp_block_sparse_linear_blocked_fwd``; bf16 only)."""
    dev = require_cuda(x2d, weight, blocks, n_active)
    dtt = x2d.dtype
    x2d, weight = contig(x2d), contig(weight.detach().to(dtt))
    bias = contig(bias.detach().to(dtt)) if bias is not None else None
    out_proj = contig(out_proj.detach().to(dtt)) if out_proj is not None else None
    ctx16 = contig(ctx16.float()) if ctx16 is not None else None
    M, D_in = x2d.shape
    out_features = weight.shape[0]
    out = torch.empty(M, out_features, dtype=dtt, device=dev)
    lib = _lib.load()
    ws = _lib.workspace(dev, lib.fp_block_sparse_linear_workspace_size(dtype_code(dtt), M, D_in, out_features,
                                                                      int(max_active)))
    if weight_blocked is not None and dtt == torch.bfloat16:
        if weight_blocked.numel() != weight.numel() or weight_blocked.dtype != torch.bfloat16:
            raise ValueError("weight_blocked: the bf16 pack_blocked_weight copy of this weight")
        rc = lib.fp_block_sparse_linear_blocked_fwd(ptr(x2d), M, D_in, ptr(weight), ptr(weight_blocked), ptr(bias),
                                                    out_features, dtype_code(dtt), ptr(blocks), ptr(n_active),
                                                    int(max_active), ptr(ctx16), ptr(out_proj), ptr(out), ptr(ws),
                                                    ws.numel(), stream_handle(dev))
        check(rc, "fp_block_sparse_linear_blocked_fwd")
        return out
    rc = lib.fp_block_sparse_linear_fwd(ptr(x2d), M, D_in, ptr(weight), ptr(bias), out_features, dtype_code(dtt),
                                        ptr(blocks), ptr(n_active), int(max_active), ptr(ctx16), ptr(out_proj),
                                        ptr(out), ptr(ws), ws.numel(), stream_handle(dev))
    check(rc, "fp_block_sparse_linear_fwd")
    return out


ACTIVATIONS = {"softmax": 0, "gelu_l2": 1}


def tokenformer(x2d: torch.Tensor, k_param: torch.Tensor, v_param: torch.Tensor, v_param_t: Optional[torch.Tensor],
                activation: str, blocks: torch.Tensor, n_active: torch.Tensor, ctx16: Optional[torch.Tensor] = None,
                out_proj: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Tokenformer contraction over the active parameter tokens (``fp_tokenformer_fwd``;
    tokenformer.py:183-203): out [M, D_out] in x's dtype."""
    dev = require_cuda(x2d, k_param, v_param, blocks, n_active)
    dtt = x2d.dtype
    x2d, k_param, v_param = contig(x2d), contig(k_param.detach().to(dtt)), contig(v_param.detach().to(dtt))
    v_param_t = contig(v_param_t.detach().to(dtt)) if v_param_t is not None else None
    out_proj = contig(out_proj.detach().to(dtt)) if out_proj is not None else None
    ctx16 = contig(ctx16.float()) if ctx16 is not None else None
    M, D_in = x2d.shape
    Np, D_out = v_param.shape
    out = torch.empty(M, D_out, dtype=dtt, device=dev)
    lib = _lib.load()
    ws = _lib.workspace(dev, lib.fp_tokenformer_workspace_size(dtype_code(dtt), M, Np))
    rc = lib.fp_tokenformer_fwd(ptr(x2d), M, D_in, ptr(k_param), ptr(v_param), ptr(v_param_t), Np, D_out,
                                dtype_code(dtt), ACTIVATIONS[activation], ptr(blocks), ptr(n_active), ptr(ctx16),
                                ptr(out_proj), ptr(out), ptr(ws), ws.numel(), stream_handle(dev))
    check(rc, "fp_tokenformer_fwd")
    return out


def transpose(t: torch.Tensor) -> torch.Tensor:
    """``t.t().contiguous()`` by ``fp_transpose`` (2-D, fp32 or bf16)."""
    dev = require_cuda(t)
    t = contig(t.detach())
    rows, cols = t.shape
    out = torch.empty(cols, rows, dtype=t.dtype, device=dev)
    check(_lib.load().fp_transpose(ptr(t), rows, cols, dtype_code(t.dtype), ptr(out), stream_handle(dev)),
          "fp_transpose")
    return out
