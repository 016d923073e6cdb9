"""Function-level Pattention (``triton_pattention``, pattention_triton.py:204-311) on the GPU against the
reference's own outputs (``tests/golden/pattention.npz``, written by make_golden.py from
``_pytorch_pattention_fallback``, ``TritonSwiGLUPattentionMLP`` and ``convert_llm_mlp_to_pattention``).

Bars: 1e-4 relative for fp32 (CUDA-core kernel), 2e-2 relative for bf16 (tcgen05 gate/up and down
kernels for widths that are multiples of 64, the CUDA-core kernel otherwise), as ||y - ref|| / ||ref||
and max|y - ref| / max|ref|.
"""

from __future__ import annotations

import pytest
import torch

import oracle
from conftest import configs, fsi, golden, max_rel, rel_err, serve_model

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = {"fp32": 1e-4, "bf16": 2e-2}
CASES = [(n, dt) for n in configs.PATTENTION_CASES for dt in configs.PATTENTION_DTYPES[n]]


def _check(y, ref, dt):
    e1, e2 = rel_err(y.float().cpu(), ref), max_rel(y.float().cpu(), ref)
    assert e1 < TOL[dt] and e2 < TOL[dt], f"rel_l2 {e1:.3e}, max_rel {e2:.3e}"


@pytest.mark.parametrize("name,dt", CASES)
def test_pattention_matches_reference(name, dt):
    g = golden("pattention")
    case = configs.PATTENTION_CASES[name]
    tdt = torch.float32 if dt == "fp32" else torch.bfloat16
    x, kg, ku, v, act = configs.pattention_tensors(case, 0, dt)
    to = lambda t: None if t is None else t.to(DEV, tdt)  # noqa: E731
    with torch.no_grad():
        y = fsi.triton_pattention(to(x), to(kg), to(v), k_up=to(ku),
                                  active_blocks=None if act is None else act.to(DEV), activation=case["activation"])
        y2 = fsi.triton_pattention(to(x), to(kg), to(v), k_up=to(ku),  # packed layouts from the cache
                                   active_blocks=None if act is None else act.to(DEV), activation=case["activation"])
    torch.cuda.synchronize()
    assert y.shape == (case["M"], case["D_out"]) and y.dtype == tdt
    _check(y, torch.from_numpy(g[f"{name}_{dt}_y"]), dt)
    assert torch.equal(y, y2)


def test_pattention_leading_dims_and_list_of_blocks():
    """x [B, T, K] keeps its leading dimensions; active blocks given as a Python list."""
    case = configs.PATTENTION_CASES["swiglu_tc"]
    x, kg, ku, v, act = configs.pattention_tensors(case, 0, "bf16")
    bf = torch.bfloat16
    y = fsi.triton_pattention(x.view(3, 100, -1).to(DEV, bf), kg.to(DEV, bf), v.to(DEV, bf), k_up=ku.to(DEV, bf),
                              active_blocks=case["active"])
    ref = oracle.pattention(x, kg, v, ku, act, "swiglu")
    assert y.shape == (3, 100, case["D_out"])
    _check(y.reshape(300, -1), ref, "bf16")


def test_fused_swiglu_forward_and_backward():
    """triton_fused_swiglu / TritonFusedSwiGLUFunction (pattention_triton.py:30-104) against torch autograd."""
    gen = torch.Generator().manual_seed(5)
    for dt, tol in ((torch.float32, 1e-5), (torch.bfloat16, 1e-2)):
        for n in ((7, 33), (64, 256)):  # odd sizes take the scalar kernel, multiples of 8 the vector one
            g = torch.randn(*n, generator=gen).to(DEV, dt).requires_grad_(True)
            u = torch.randn(*n, generator=gen).to(DEV, dt).requires_grad_(True)
            dh = torch.randn(*n, generator=gen).to(DEV, dt)
            h = fsi.triton_fused_swiglu(g, u)
            h.backward(dh)
            gr, ur = g.detach().float().requires_grad_(True), u.detach().float().requires_grad_(True)
            hr = torch.nn.functional.silu(gr) * ur
            hr.backward(dh.float())
            assert rel_err(h.detach().float().cpu(), hr.detach().cpu()) < tol
            assert rel_err(g.grad.float().cpu(), gr.grad.cpu()) < tol
            assert rel_err(u.grad.float().cpu(), ur.grad.cpu()) < tol


class _Dense(torch.nn.Module):
    def __init__(self, h, i):
        super().__init__()
        self.gate_proj = torch.nn.Linear(h, i, bias=False)
        self.up_proj = torch.nn.Linear(h, i, bias=False)
        self.down_proj = torch.nn.Linear(i, h, bias=False)


@pytest.mark.parametrize("dt", ["fp32", "bf16"])
def test_pattention_mlp_from_dense(dt):
    """TritonSwiGLUPattentionMLP.from_dense_mlp (pattention_triton.py:348-375): sparse and dense forward."""
    g = golden("pattention")
    cfg = configs.PATTENTION_MLP
    wg, wu, wd, x = configs.pattention_mlp_weights(0)
    tdt = torch.float32 if dt == "fp32" else torch.bfloat16
    dense = _Dense(cfg["hidden"], cfg["intermediate"])
    with torch.no_grad():
        for lin, wt in ((dense.gate_proj, wg), (dense.up_proj, wu), (dense.down_proj, wd)):
            lin.weight.copy_(wt.to(tdt).float())
    dense = dense.to(DEV, tdt)
    mlp = fsi.TritonSwiGLUPattentionMLP.from_dense_mlp(dense)
    assert mlp.num_blocks == cfg["intermediate"] // 64 and mlp.k_gate.dtype == tdt
    with torch.no_grad():
        ys = mlp(x.to(DEV, tdt), active_blocks=torch.tensor(cfg["active"], device=DEV))
        yd = mlp(x.to(DEV, tdt))
    # bf16: the reference ran on the unrounded weights, so compare against the oracle on the rounded ones
    if dt == "fp32":
        _check(ys, torch.from_numpy(g["mlp_sparse_y"]), dt)
        _check(yd, torch.from_numpy(g["mlp_dense_y"]), dt)
    else:
        r = lambda t: t.to(tdt).float()  # noqa: E731
        ref_s = oracle.pattention(r(x), r(wg), r(wd).t(), r(wu), torch.tensor(cfg["active"]), "swiglu")
        ref_d = oracle.pattention(r(x), r(wg), r(wd).t(), r(wu), None, "swiglu")
        _check(ys, ref_s, dt)
        _check(yd, ref_d, dt)


def test_convert_llm_mlp_to_pattention():
    """convert_llm_mlp_to_pattention (pattention_triton.py:378-395) on the tiny Llama of the serving
    case: every decoder MLP replaced, logits equal to the reference's converted model (fp32)."""
    g = golden("pattention")
    m = serve_model(g.meta["serve"])
    fsi.convert_llm_mlp_to_pattention(m)
    assert [type(layer.mlp).__name__ for layer in m.model.layers] == list(g["convert_types"])
    m = m.to(DEV).eval()
    with torch.no_grad():
        logits = m(torch.from_numpy(g["convert_prompt"]).to(DEV)).logits[0]
    assert rel_err(logits.float().cpu(), torch.from_numpy(g["convert_logits"])) < 1e-4


def test_pattention_errors_are_loud():
    x = torch.randn(4, 128, device=DEV)
    kg, v = torch.randn(128, 128, device=DEV), torch.randn(128, 64, device=DEV)
    with pytest.raises(ValueError):
        fsi.triton_pattention(x, kg, v, activation="swiglu")  # k_up missing
    with pytest.raises(ValueError):
        fsi.triton_pattention(x, kg, v, activation="tanh")
    with pytest.raises(ValueError):
        fsi.triton_pattention(x, kg, v, activation="relu", block_n=32)
    with pytest.raises(RuntimeError):
        fsi.triton_pattention(x.cpu(), kg.cpu(), v.cpu(), activation="relu")  # no CPU fallback
