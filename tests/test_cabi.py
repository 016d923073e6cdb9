"""CPU checks of the C-ABI library: it builds, loads, exports every declared entry point, answers the
host-only queries, and the Python layer refuses CPU tensors instead of computing elsewhere."""

from __future__ import annotations

import os
import re
import subprocess

import pytest
import torch

from conftest import REPO, configs, fsi

HEADER_DIR = os.path.join(REPO, "include")


def declared_symbols():
    names = []
    for fn in sorted(os.listdir(HEADER_DIR)):
        if fn.endswith(".h"):
            text = open(os.path.join(HEADER_DIR, fn)).read()
            names += re.findall(r"FP_API\s+[\w\s\*]+?\b(fp_\w+)\s*\(", text)
    return names


@pytest.fixture(scope="module")
def lib():
    build = __import__("importlib").import_module("foveal-sparse-indexer_b200.build")
    build.build()
    return fsi.load_library()


def test_header_declares_entry_points():
    names = declared_symbols()
    assert len(names) >= 11
    for must in ("fp_pattention_token_fwd", "fp_pattention_pooled_fwd", "fp_router_scores", "fp_select_blocks",
                 "fp_pooled_route", "fp_token_workspace_size", "fp_device_error"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", fsi.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (fp_\w+)", out))
    missing = [n for n in declared_symbols() if n not in exported]
    assert not missing, missing
    for n in declared_symbols():
        assert hasattr(lib, n)
    # ctypes signatures of the Python layer cover the whole header
    assert set(declared_symbols()) == set(fsi._lib.SIGNATURES)


def test_abi_version_and_status_strings(lib):
    hdr = open(os.path.join(HEADER_DIR, "foveal_pattention.h")).read()
    ver = int(re.search(r"#define FP_ABI_VERSION (\d+)", hdr).group(1))
    assert lib.fp_abi_version() == ver
    for code in range(7):
        assert lib.fp_status_string(code)
    assert lib.fp_status_string(99) == b"unknown status"


def test_workspace_sizes(lib):
    wl = configs.CONFIGS["8b"]
    tok = lib.fp_token_workspace_size(1, wl.tokens, wl.hidden_dim, wl.num_blocks, wl.base_blocks,
                                      wl.max_remote_blocks, 1)
    # dense-masked activations H (M x NB x 64 bf16) dominate
    assert tok >= wl.tokens * wl.num_blocks * 64 * 2
    assert tok < 2 * wl.tokens * wl.num_blocks * 64 * 2
    shard = lib.fp_token_workspace_size(1, wl.tokens, wl.hidden_dim, wl.num_blocks, wl.base_blocks,
                                        wl.max_remote_blocks, 8)
    assert shard < tok / 4
    f32 = lib.fp_token_workspace_size(0, 512, 512, 32, 1, 8, 1)
    assert 0 < f32 < (1 << 24)
    assert lib.fp_pooled_workspace_size(1, 1024, 4096, 224, 24) >= 1024 * 24 * 64 * 2
    assert lib.fp_token_workspace_size(1, 0, 4096, 224, 4, 56, 1) > 0


def test_python_layer_refuses_cpu_tensors():
    wl = configs.CONFIGS["pr1"]
    m = fsi.FovealPattentionMLP(hidden_dim=wl.hidden_dim, intermediate_dim=wl.intermediate_dim,
                                base_blocks=1, remote_blocks=8, dtype=torch.float32, routing="token")
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.zeros(2, 4, wl.hidden_dim))
    with pytest.raises(RuntimeError, match="CUDA"):
        fsi.kernels.router_scores(torch.zeros(2, 64), torch.zeros(16, 64), torch.zeros(4, 16))
    with pytest.raises(RuntimeError):
        fsi.masked_softmax(torch.zeros(2, 3), torch.ones(2, 3, dtype=torch.bool))


def test_module_mirrors_reference_interface():
    """Constructor, parameter names/shapes and state_dict keys of foveal_pattention.py:59-98."""
    m = fsi.FovealPattentionMLP(hidden_dim=256, intermediate_dim=512, base_blocks=2, remote_blocks=4,
                                dtype=torch.float32)
    assert set(m.state_dict()) == {"k_gate", "k_up", "v", "q_proj_16d.weight", "block_keys_16d",
                                   "out_proj_16d.weight", "offsets"}
    assert m.k_gate.shape == (512, 256) and m.v.shape == (512, 256)
    assert m.q_proj_16d.weight.shape == (16, 256) and m.block_keys_16d.shape == (8, 16)
    assert m.out_proj_16d.weight.shape == (256, 16)
    assert m.num_blocks == 8 and m.total_active_blocks == 6 and m.active_channels == 384
    with pytest.raises(ValueError):
        fsi.FovealPattentionMLP(hidden_dim=256, intermediate_dim=512, block_size=32)
    with pytest.raises(ValueError):
        fsi.FovealPattentionMLP(hidden_dim=256, intermediate_dim=512, routing="bogus")


def test_from_dense_mlp_shares_weights():
    """tests/test_foveal_pattention.py:27-44 of the reference (shape/count invariants)."""

    class Dense(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_proj = torch.nn.Linear(256, 512, bias=False)
            self.up_proj = torch.nn.Linear(256, 512, bias=False)
            self.down_proj = torch.nn.Linear(512, 256, bias=False)

    d = Dense()
    p = fsi.FovealPattentionMLP.from_dense_mlp(d, block_size=64, base_blocks=2, remote_blocks=4, index_dim=16)
    assert p.k_gate.shape == (512, 256) and p.k_up.shape == (512, 256) and p.v.shape == (512, 256)
    assert p.num_blocks == 8 and p.total_active_blocks == 6
    assert torch.equal(p.v, d.down_proj.weight.t())
    assert float(p.out_proj_16d.weight.abs().sum()) == 0.0


def test_indexer_interface():
    idx = fsi.FovealIndexer(hidden_size=32, index_dim=16, block_size=16, local_window_blocks=1, top_p=0.9)
    assert idx.q_proj.weight.shape == (16, 32) and idx.out_proj.weight.shape == (32, 16)
    with pytest.raises(NotImplementedError):  # the kernels pool 64-row blocks
        idx.compute_kv_blocks_16d(torch.zeros(32, 32))
    with pytest.raises(RuntimeError):  # no CPU fallback
        idx.distillation_loss(torch.zeros(1, 2, 4), torch.ones(1, 2, 4))
    with pytest.raises(NotImplementedError):
        fsi.select_blocks(torch.zeros(1, 2, 4), causal=True)


def test_variant_layers_interface():
    """BlockSparseLinear / FovealTokenformerLinear / FovealTokenformerFFN: the reference's constructor
    arguments, parameter shapes and init; CPU inputs raise instead of computing on the host."""
    bsl = fsi.BlockSparseLinear(128, 256, base_blocks=2, bias=True)
    assert bsl.weight.shape == (256, 128) and bsl.bias.shape == (256,) and bsl.num_blocks == 4
    assert bsl.indexer.out_proj.weight.shape == (256, 16) and bsl.weight_to_k.weight.shape == (16, 128)
    with pytest.raises(NotImplementedError):
        fsi.BlockSparseLinear(128, 256, block_size=128)
    with pytest.raises(ValueError):
        fsi.BlockSparseLinear(128, 100)
    tf = fsi.FovealTokenformerLinear(64, 96, num_param_tokens=256, activation="gelu_l2")
    assert tf.k_param.shape == (256, 64) and tf.v_param.shape == (256, 96) and tf.num_blocks == 4
    with pytest.raises(ValueError):
        fsi.FovealTokenformerLinear(64, 96, num_param_tokens=100)
    ffn = fsi.FovealTokenformerFFN(64, 128, num_param_tokens=256)
    assert ffn.fc1.activation == "gelu_l2" and ffn.fc2.activation == "softmax"
    with pytest.raises(RuntimeError):
        bsl(torch.zeros(1, 3, 128))
    with pytest.raises(RuntimeError):
        tf(torch.zeros(1, 3, 64))


def test_package_imports_by_plain_name():
    """``import foveal_sparse_indexer_b200`` (repository root on sys.path) binds to the package whose
    directory name contains hyphens."""
    import foveal_sparse_indexer_b200 as alias
    assert alias is fsi
    assert alias.FovealPattentionMLP is fsi.FovealPattentionMLP
