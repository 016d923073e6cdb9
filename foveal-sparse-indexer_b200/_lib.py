"""ctypes binding of libfovealpatt.so (C ABI declared in include/foveal_pattention.h).

Every wrapper takes CUDA tensors, passes raw device pointers, the current CUDA stream and explicit
shapes, and raises on a non-zero status.  There is no CPU fallback: a CPU tensor, a missing library
or a non-sm_100 device raises instead of silently computing elsewhere.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Dict, Optional, Tuple

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libfovealpatt.so")

FP_DTYPE_F32 = 0
FP_DTYPE_BF16 = 1
FP_ERR_UNSUPPORTED = 2

_c_int, _c_i64, _c_f, _c_p, _c_sz = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/foveal_pattention.h
SIGNATURES = {
    "fp_abi_version": (_c_int, []),
    "fp_status_string": (ctypes.c_char_p, [_c_int]),
    "fp_router_scores": (_c_int, [_c_p, _c_p, _c_p, _c_int, _c_i64, _c_int, _c_int, _c_p, _c_p, _c_p]),
    "fp_select_blocks": (_c_int, [_c_p, _c_i64, _c_int, _c_int, _c_f, _c_int, _c_int, _c_int, _c_f, _c_p, _c_p,
                                  _c_p, _c_p, _c_p, _c_p]),
    "fp_pooled_route": (_c_int, [_c_p, _c_p, _c_p, _c_int, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int, _c_p,
                                 _c_p, _c_p, _c_p, _c_sz, _c_p]),
    "fp_pack_weights": (_c_int, [_c_p, _c_p, _c_p, _c_int, _c_int, _c_int, _c_p, _c_p, _c_p]),
    "fp_token_workspace_size": (_c_sz, [_c_int, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int]),
    "fp_pooled_workspace_size": (_c_sz, [_c_int, _c_i64, _c_int, _c_int, _c_int]),
    "fp_pattention_token_fwd": (_c_int, [_c_p, _c_i64, _c_int, _c_int, _c_int, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
                                         _c_p, _c_int, _c_f, _c_int, _c_int, _c_f, _c_int, _c_int, _c_int, _c_p,
                                         _c_int, _c_p, _c_p, _c_p, _c_p, _c_sz, _c_p]),
    "fp_pattention_pooled_fwd": (_c_int, [_c_p, _c_i64, _c_int, _c_int, _c_int, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
                                          _c_int, _c_p, _c_p, _c_p, _c_int, _c_p, _c_sz, _c_p]),
    "fp_pattention_token_fwd_noalloc": (_c_int, [_c_p, _c_i64, _c_int, _c_int, _c_int, _c_p, _c_p, _c_p, _c_p, _c_p,
                                                 _c_p, _c_p, _c_p, _c_int, _c_f, _c_int, _c_int, _c_f, _c_int, _c_int,
                                                 _c_int, _c_p, _c_int, _c_p, _c_p, _c_p, _c_p]),
    "fp_block_energy_workspace_size": (ctypes.c_size_t, [_c_i64, _c_int]),
    "fp_block_energy": (_c_int, [_c_p, _c_i64, _c_int, _c_int, _c_int, _c_p, _c_p, _c_p, _c_p, ctypes.c_size_t,
                                 _c_p]),
    "fp_swiglu_bwd": (_c_int, [_c_p, _c_p, _c_p, _c_int, _c_i64, _c_p, _c_p, _c_p, _c_p]),
    "fp_param_blocks_16d": (_c_int, [_c_p, _c_p, _c_p, _c_int, _c_i64, _c_int, _c_p, _c_p, _c_p]),
    "fp_cosine_block_scores": (_c_int, [_c_p, _c_p, _c_p, _c_int, _c_i64, _c_int, _c_int, _c_p, _c_p, _c_p]),
    "fp_select_remote_top_p": (_c_int, [_c_p, _c_i64, _c_int, _c_int, _c_f, _c_int, _c_int, _c_p, _c_p, _c_p,
                                        _c_p]),
    "fp_union_blocks": (_c_int, [_c_p, _c_p, _c_i64, _c_int, _c_int, _c_int, _c_p, _c_p, _c_p]),
    "fp_block_sparse_linear_workspace_size": (_c_sz, [_c_int, _c_i64, _c_int, _c_int, _c_int]),
    "fp_block_sparse_linear_fwd": (_c_int, [_c_p, _c_i64, _c_int, _c_p, _c_p, _c_int, _c_int, _c_p, _c_p, _c_int,
                                            _c_p, _c_p, _c_p, _c_p, _c_sz, _c_p]),
    "fp_pack_blocked_weight": (_c_int, [_c_p, _c_int, _c_int, _c_p, _c_p]),
    "fp_block_sparse_linear_blocked_fwd": (_c_int, [_c_p, _c_i64, _c_int, _c_p, _c_p, _c_p, _c_int, _c_int, _c_p,
                                                    _c_p, _c_int, _c_p, _c_p, _c_p, _c_p, _c_sz, _c_p]),
    "fp_peer_alloc": (_c_int, [_c_sz, ctypes.POINTER(_c_p), _c_p]),
    "fp_peer_open": (_c_int, [_c_p, ctypes.POINTER(_c_p)]),
    "fp_peer_close": (_c_int, [_c_p]),
    "fp_peer_free": (_c_int, [_c_p]),
    "fp_pattention_routed_peer_fwd": (_c_int, [_c_p, _c_i64, _c_int, _c_int, _c_int, _c_p, _c_p, _c_p, _c_p, _c_p,
                                               _c_p, _c_int, _c_int, _c_p, _c_p, _c_p, _c_int, _c_int, _c_p, _c_p,
                                               _c_int, _c_i64, ctypes.c_uint32, _c_int, _c_p, _c_sz, _c_p]),
    "fp_peer_combine": (_c_int, [_c_p, _c_p, _c_int, _c_i64, _c_int, _c_int, ctypes.c_uint32, _c_p, _c_int, _c_p,
                                 _c_sz, _c_p]),
    "fp_peer_reduce_supported": (_c_int, [_c_int, _c_i64, _c_int, _c_int, _c_int, _c_int]),
    "fp_peer_put": (_c_int, [_c_p, _c_sz, _c_p, _c_int, _c_p]),
    "fp_peer_signal": (_c_int, [_c_p, _c_int, ctypes.c_uint32, _c_p]),
    "fp_peer_wait": (_c_int, [_c_p, _c_int, ctypes.c_uint32, _c_p, _c_sz, _c_p]),
    "fp_tokenformer_workspace_size": (_c_sz, [_c_int, _c_i64, _c_int]),
    "fp_tokenformer_fwd": (_c_int, [_c_p, _c_i64, _c_int, _c_p, _c_p, _c_p, _c_int, _c_int, _c_int, _c_int, _c_p,
                                    _c_p, _c_p, _c_p, _c_p, _c_p, _c_sz, _c_p]),
    "fp_transpose": (_c_int, [_c_p, _c_i64, _c_i64, _c_int, _c_p, _c_p]),
    "fp_set_stage_events": (_c_int, [ctypes.POINTER(_c_p), _c_int]),
    "fp_device_error": (_c_int, [_c_p, _c_p, _c_p]),
    "fp_noalloc_device_error": (_c_int, [_c_p, _c_p]),
    "fp_pack_pattention_weights": (_c_int, [_c_p, _c_p, _c_p, _c_int, _c_int, _c_int, _c_int, _c_p, _c_p, _c_p]),
    "fp_pattention_workspace_size": (_c_sz, [_c_int, _c_i64, _c_int, _c_int, _c_int, _c_int]),
    "fp_pattention_fwd": (_c_int, [_c_p, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_p, _c_p, _c_p, _c_p, _c_p,
                                   _c_p, _c_int, _c_int, _c_p, _c_p, _c_sz, _c_p]),
    "fp_swiglu_fwd": (_c_int, [_c_p, _c_p, _c_int, _c_i64, _c_p, _c_p]),
    "fp_route_workspace_size": (_c_sz, [_c_i64]),
    "fp_route_tokens": (_c_int, [_c_p, _c_i64, _c_int, _c_int, _c_int, _c_p, _c_p, _c_int, _c_f, _c_int, _c_int, _c_f,
                                 _c_p, _c_p, _c_p, _c_p, _c_p, _c_sz, _c_p]),
    "fp_pattention_routed_fwd": (_c_int, [_c_p, _c_i64, _c_int, _c_int, _c_int, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p,
                                          _c_int, _c_int, _c_p, _c_p, _c_p, _c_int, _c_int, _c_p, _c_int, _c_p,
                                          _c_sz, _c_p]),
}

_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None


def load() -> ctypes.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"{LIB_PATH} is missing: build it with "
                                   f"`python {os.path.join(HERE, 'build.py')}` (nvcc, sm_100a)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


class FovealKernelError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().fp_status_string(rc).decode()
        raise FovealKernelError(f"{what} failed: status {rc} ({msg})")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return FP_DTYPE_F32
    if dt == torch.bfloat16:
        return FP_DTYPE_BF16
    raise TypeError(f"unsupported dtype {dt}: the kernels take float32 or bfloat16")


def ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_handle(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("the Foveal Pattention kernels run on CUDA tensors only (no CPU fallback); "
                               f"got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise RuntimeError("no CUDA tensor given")
    return dev


def contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() and t.data_ptr() % 16 == 0 else t.contiguous()


# ------------------------------------------------------------------ workspaces
# One growable byte buffer per (device, stream): calls on one stream are ordered, so they can share it.
_ws: Dict[Tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           torch.cuda.current_stream(device).cuda_stream)
    buf = _ws.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _ws[key] = buf
    return buf


def release_workspaces() -> None:
    _ws.clear()


def device_error(ws: torch.Tensor) -> int:
    """Synchronize the current stream and return (and clear) the workspace's device error code."""
    code = ctypes.c_int(0)
    lib = load()
    rc = lib.fp_device_error(ptr(ws), stream_handle(ws.device), ctypes.byref(code))
    if rc not in (0, 6):
        check(rc, "fp_device_error")
    return code.value


def set_stage_events(events) -> None:
    """Register torch.cuda.Event objects as stage-boundary markers for this thread (None: off)."""
    lib = load()
    if not events:
        check(lib.fp_set_stage_events(None, 0), "fp_set_stage_events")
        return
    handles = []
    for e in events:
        if not e.cuda_event:  # torch creates the CUDA event lazily at its first record
            e.record()
        handles.append(e.cuda_event)
    arr = (_c_p * len(handles))(*handles)
    check(lib.fp_set_stage_events(arr, len(handles)), "fp_set_stage_events")
