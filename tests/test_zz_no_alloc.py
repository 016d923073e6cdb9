"""Allocation-free entry point ``fp_pattention_token_fwd_noalloc`` against the workspace entry point.

Some callers cannot allocate device memory when they run the layer — plugin interfaces that only hand
over input and output pointers, or serving loops whose device-memory budget is fixed at start-up.
The no-alloc entry point serves them from scratch memory the library keeps on each GPU.  This test
drives both entry points through the C ABI on the same decode-step inputs and requires the no-alloc
results of two consecutive calls (which share and reuse that scratch) to match the workspace entry
point within the bf16 tolerance of the other parity tests, each call's device error word (read back
from the scratch with ``fp_noalloc_device_error``) to be clear, and an oversized batch to be refused.
The file is named so that pytest collects it last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import compare_routes, configs, fsi, max_rel, rel_err

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
FP_ERR_WORKSPACE = 3


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def test_noalloc_matches_workspace_entry_point():
    wl = [p for p in configs.decode_points() if p.max_remote_blocks == 16][0]  # 64 tokens, 8B MLP shape
    w = configs.make_weights(wl)
    dev, bf = torch.device("cuda"), torch.bfloat16
    kg, ku, v, wq, k16, wout = (t.to(dev, bf).contiguous() for t in
                                (w.k_gate, w.k_up, w.v, w.q_proj_16d, w.block_keys_16d, w.out_proj_16d))
    x = configs.make_x(wl).reshape(-1, wl.hidden_dim).to(dev, bf).contiguous()
    w_gu, v_t = fsi.kernels.pack_weights(kg, ku, v)
    lib = fsi.load_library()
    M, D, NB, K = x.shape[0], x.shape[1], wl.num_blocks, wl.max_remote_blocks
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = (_p(x), M, D, NB, 1, _p(kg), _p(ku), _p(v), _p(w_gu), _p(v_t), _p(wq), _p(k16), _p(wout),
            wl.base_blocks, wl.top_p, wl.min_remote_blocks, K, wl.temperature, 1, 1, 0)

    # the existing entry point, with a caller-allocated workspace
    ws = torch.empty(lib.fp_token_workspace_size(1, M, D, NB, wl.base_blocks, K, 1), dtype=torch.uint8, device=dev)
    y_ref = torch.empty(M, D, dtype=bf, device=dev)
    idx_ref = torch.empty(M, K, dtype=torch.int32, device=dev)
    cnt_ref = torch.empty(M, dtype=torch.int32, device=dev)
    assert lib.fp_pattention_token_fwd(*args, _p(y_ref), 0, _p(idx_ref), _p(cnt_ref), None, _p(ws), ws.numel(),
                                       stream) == 0
    torch.cuda.synchronize()

    for call in range(2):  # the second call reuses the scratch left behind by the first
        y = torch.full((M, D), float("nan"), dtype=bf, device=dev)
        idx = torch.full((M, K), -1, dtype=torch.int32, device=dev)
        cnt = torch.full((M,), -1, dtype=torch.int32, device=dev)
        assert lib.fp_pattention_token_fwd_noalloc(*args, _p(y), 0, _p(idx), _p(cnt), None, stream) == 0
        torch.cuda.synchronize()
        assert torch.isfinite(y.float()).all(), f"call {call}: output not fully written"
        e1, e2 = rel_err(y.float(), y_ref.float()), max_rel(y.float(), y_ref.float())
        assert e1 < BF16_TOL and e2 < BF16_TOL, f"call {call}: rel_l2 {e1:.3e}, max_rel {e2:.3e}"
        bad, _ = compare_routes(idx.cpu(), cnt.cpu(), idx_ref.cpu(), cnt_ref.cpu())
        assert bad == 0
        # the call's bounded-wait error word, read from the library's scratch array: no wait ran out
        code = ctypes.c_int(-1)
        assert lib.fp_noalloc_device_error(stream, ctypes.byref(code)) == 0 and code.value == 0


def test_noalloc_refuses_batches_beyond_its_scratch():
    wl = configs.CONFIGS["8b"]  # 16384 tokens need ~470 MB of workspace, far above the scratch
    lib = fsi.load_library()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.fp_pattention_token_fwd_noalloc(
        None, wl.tokens, wl.hidden_dim, wl.num_blocks, 1, None, None, None, None, None, None, None, None,
        wl.base_blocks, wl.top_p, wl.min_remote_blocks, wl.max_remote_blocks, 1.0, 1, 1, 0, None, 0, None, None,
        None, stream)
    assert rc == FP_ERR_WORKSPACE
