"""Workload configurations and seeded synthetic inputs for the Foveal Pattention MLP forward.

The five configurations are the ones the reference's hot path is measured on (Llama-3-8B / 70B MLP
shapes, a decode step, a CPU-runnable case and a sparsity sweep).  No public dataset is involved:
every tensor is drawn from a seeded normal distribution.

Draw order (fixed, so that a CPU oracle on another machine regenerates identical tensors):
    weights: generator seeded with ``seed``      -> k_gate, k_up, v, q_proj_16d, block_keys_16d, out_proj_16d
    inputs : generator seeded with ``seed + 1``  -> x of shape [B, L, D]
All tensors are drawn in fp32 (x ~ N(0, 1), weights ~ N(0, 0.02)) and, for bf16 configurations,
rounded to bf16 after drawing.  Weights and x use separate generators so that a token subsample of x
does not change the weights.
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace
from typing import Dict, List, Optional

import torch

BLOCK_SIZE = 64
INDEX_DIM = 16
WEIGHT_STD = 0.02


@dataclass(frozen=True)
class Workload:
    """One Pattention-MLP forward configuration.

    Field names follow the reference module (``FovealPattentionMLP`` / ``select_blocks``):
    ``hidden_dim`` = d_model, ``intermediate_dim`` = N_p parameter tokens, ``base_blocks`` = the
    always-active leading blocks, ``top_p`` / ``min_remote_blocks`` / ``max_remote_blocks`` = the
    router's mass target and [K_min, K_max] guardrails.
    """

    name: str
    dtype: str  # "fp32" | "bf16"
    batch: int
    seq_len: int
    hidden_dim: int
    intermediate_dim: int
    base_blocks: int
    top_p: float
    min_remote_blocks: int
    max_remote_blocks: int
    temperature: float = 1.0
    # pooled (reference default) mode active remote-block count; reuses K_max
    note: str = ""

    @property
    def tokens(self) -> int:
        return self.batch * self.seq_len

    @property
    def num_blocks(self) -> int:
        return self.intermediate_dim // BLOCK_SIZE

    @property
    def torch_dtype(self) -> torch.dtype:
        return torch.float32 if self.dtype == "fp32" else torch.bfloat16

    def active_blocks_per_token(self) -> int:
        """A = base + K_max: at the BASELINE weight scale every token selects exactly K_max remote
        blocks (the block softmax is near-uniform, so top-p never binds)."""
        return self.base_blocks + min(self.max_remote_blocks, self.num_blocks - self.base_blocks)

    def flops_per_token(self, active: Optional[int] = None) -> float:
        """Algorithmic FLOPs of the gated contraction per token: 6 * D * 64 * A."""
        a = self.active_blocks_per_token() if active is None else active
        return 6.0 * self.hidden_dim * BLOCK_SIZE * a

    def with_(self, **kw) -> "Workload":
        return replace(self, **kw)


CONFIGS: Dict[str, Workload] = {
    "pr1": Workload("pr1", "fp32", 4, 128, 512, 2048, 1, 0.9, 2, 8,
                    note="CPU-runnable reference case"),
    "8b": Workload("8b", "bf16", 8, 2048, 4096, 14336, 4, 0.8, 8, 56,
                   note="Llama-3-8B MLP shape, 1 GPU"),
    "decode": Workload("decode", "bf16", 64, 1, 4096, 14336, 4, 0.9, 8, 16,
                       note="decode step; K_max swept over 8/16/32"),
    "70b": Workload("70b", "bf16", 4, 4096, 8192, 28672, 8, 0.8, 16, 112,
                    note="Llama-3-70B MLP shape, blocks sharded over GPUs"),
    "sweep": Workload("sweep", "bf16", 4, 4096, 4096, 14336, 4, 0.9, 8, 56,
                      note="sparsity sweep; top_p x K_max grid"),
}

DECODE_KMAX = (8, 16, 32)
SWEEP_TOP_P = (1.0, 0.9, 0.7, 0.5, 0.3)
SWEEP_KMAX = (224, 56, 28, 14)


def sweep_points() -> List[Workload]:
    base = CONFIGS["sweep"]
    pts = []
    for p in SWEEP_TOP_P:
        for k in SWEEP_KMAX:
            pts.append(base.with_(name=f"sweep_p{p}_k{k}", top_p=p, max_remote_blocks=k,
                                  min_remote_blocks=min(8, k)))
    return pts


def decode_points() -> List[Workload]:
    base = CONFIGS["decode"]
    return [base.with_(name=f"decode_k{k}", max_remote_blocks=k, min_remote_blocks=min(8, k))
            for k in DECODE_KMAX]


def calib_workload() -> Workload:
    """Offline router calibration case: the PR1 shape (D 512, 32 blocks) with
    bf16-rounded weights and 512 bf16-rounded calibration tokens, so that the bf16 tensor-core path
    and the fp32 reference see the same values."""
    return CONFIGS["pr1"].with_(name="calib", dtype="bf16")


def train_workload() -> Workload:
    """Training-mode (pooled routing + additive stream) gradient case: 64 tokens, D 256, 16 blocks, base 1
    and 4 pooled remote blocks (``max_remote_blocks`` doubles as the pooled remote count)."""
    return CONFIGS["pr1"].with_(name="train", batch=2, seq_len=32, hidden_dim=256, intermediate_dim=1024,
                                max_remote_blocks=4, min_remote_blocks=1)


@dataclass
class Weights:
    """Parameter tensors with the reference module's names and shapes (fp32 storage, values already
    rounded to the configuration's dtype)."""

    k_gate: torch.Tensor        # [N_p, D]
    k_up: torch.Tensor          # [N_p, D]
    v: torch.Tensor             # [N_p, D]  (= W_down^T)
    q_proj_16d: torch.Tensor    # [16, D]
    block_keys_16d: torch.Tensor  # [NB, 16]
    out_proj_16d: torch.Tensor  # [D, 16]

    def to(self, device=None, dtype=None) -> "Weights":
        f = lambda t: t.to(device=device, dtype=dtype)
        return Weights(f(self.k_gate), f(self.k_up), f(self.v), f(self.q_proj_16d),
                       f(self.block_keys_16d), f(self.out_proj_16d))

    def state_dict(self) -> Dict[str, torch.Tensor]:
        return {
            "k_gate": self.k_gate, "k_up": self.k_up, "v": self.v,
            "q_proj_16d.weight": self.q_proj_16d, "block_keys_16d": self.block_keys_16d,
            "out_proj_16d.weight": self.out_proj_16d,
        }


def _round(t: torch.Tensor, dtype: str) -> torch.Tensor:
    return t if dtype == "fp32" else t.to(torch.bfloat16).to(torch.float32)


def make_weights(w: Workload, seed: int = 0, device=None) -> Weights:
    """Seeded weights.  ``device="cuda"`` draws them on the GPU with a CUDA generator (same distributions
    and draw order, different values than the CPU generator; used by the benchmark for the large shapes,
    where drawing on the host would take most of the run)."""
    g = torch.Generator(device=device or "cpu").manual_seed(seed)
    D, Np, NB = w.hidden_dim, w.intermediate_dim, w.num_blocks

    def draw(*shape):
        return _round(torch.randn(*shape, generator=g, device=device) * WEIGHT_STD, w.dtype)

    return Weights(draw(Np, D), draw(Np, D), draw(Np, D), draw(INDEX_DIM, D),
                   draw(NB, INDEX_DIM), draw(D, INDEX_DIM))


def make_x(w: Workload, seed: int = 0, device=None) -> torch.Tensor:
    g = torch.Generator(device=device or "cpu").manual_seed(seed + 1)
    return _round(torch.randn(w.batch, w.seq_len, w.hidden_dim, generator=g, device=device), w.dtype)


# ---------------------------------------------------------------------------------------------------
# Layers that share the router: BlockSparseLinear ("bsl"), FovealTokenformerLinear ("tf") and
# FovealTokenformerFFN ("ffn").  Parity cases (small, CPU-runnable) and one bench shape each.
# Parameters are drawn in sorted state_dict key order from a generator seeded with ``seed + 11``: matrices
# ~ N(0, fan_in^-0.5), biases and the 16-D output projections ~ N(0, 0.05) (large enough that the
# additive stream is visible in the outputs); x ~ N(0, 1) from ``seed + 12``.
# ---------------------------------------------------------------------------------------------------
VARIANT_CASES: Dict[str, dict] = {
    "bsl_a": dict(kind="bsl", in_features=256, out_features=2048, base_blocks=2, top_p=0.9, min_remote_blocks=0,
                  max_remote_blocks=4, remote_capacity=4, bias=True, use_additive_stream=True, x_shape=(2, 5, 256)),
    "bsl_b": dict(kind="bsl", in_features=512, out_features=1024, base_blocks=1, top_p=0.3, min_remote_blocks=1,
                  max_remote_blocks=6, remote_capacity=6, bias=False, use_additive_stream=False, x_shape=(12, 512)),
    "bsl_c": dict(kind="bsl", in_features=128, out_features=256, base_blocks=2, top_p=0.95, min_remote_blocks=0,
                  max_remote_blocks=8, remote_capacity=8, bias=True, use_additive_stream=True, x_shape=(3, 7, 128)),
    # mass never reaches top_p: the inference rule counts one block past the two available ones
    "bsl_d": dict(kind="bsl", in_features=192, out_features=256, base_blocks=2, top_p=1.5, min_remote_blocks=0,
                  max_remote_blocks=8, remote_capacity=8, bias=False, use_additive_stream=True, x_shape=(2, 3, 192)),
    "tf_softmax": dict(kind="tf", in_features=256, out_features=256, num_param_tokens=2048, base_blocks=2, top_p=0.9,
                       min_remote_blocks=0, max_remote_blocks=4, remote_capacity=4, activation="softmax",
                       x_shape=(2, 6, 256)),
    "tf_gelu": dict(kind="tf", in_features=256, out_features=512, num_param_tokens=1024, base_blocks=2, top_p=0.5,
                    min_remote_blocks=1, max_remote_blocks=3, remote_capacity=4, activation="gelu_l2",
                    x_shape=(1, 9, 256)),
    "ffn": dict(kind="ffn", hidden_size=256, intermediate_size=512, num_param_tokens=512, base_blocks=2, top_p=0.95,
                max_remote_blocks=4, x_shape=(2, 4, 256)),
}

# Bench shapes (bf16): a BlockSparseLinear with the 8B MLP's up-projection shape and a Tokenformer FFN.
VARIANT_BENCH: Dict[str, dict] = {
    "bsl_8b": dict(kind="bsl", in_features=4096, out_features=14336, base_blocks=4, top_p=0.8, min_remote_blocks=0,
                   max_remote_blocks=8, remote_capacity=8, bias=False, use_additive_stream=True, x_shape=(4, 4096, 4096)),
    "tf_ffn": dict(kind="ffn", hidden_size=2048, intermediate_size=2048, num_param_tokens=4096, base_blocks=4,
                   top_p=0.95, max_remote_blocks=8, x_shape=(4, 4096, 2048)),
}

_MODULE_KEYS = {
    "bsl": ("in_features", "out_features", "base_blocks", "top_p", "min_remote_blocks", "max_remote_blocks",
            "remote_capacity", "use_additive_stream", "bias"),
    "tf": ("in_features", "out_features", "num_param_tokens", "base_blocks", "top_p", "min_remote_blocks",
           "max_remote_blocks", "remote_capacity", "activation"),
    "ffn": ("hidden_size", "intermediate_size", "num_param_tokens", "base_blocks", "top_p", "max_remote_blocks"),
}


def variant_kwargs(case: dict) -> dict:
    """Constructor keyword arguments of the case's module (the same for the reference's class)."""
    return {k: case[k] for k in _MODULE_KEYS[case["kind"]]}


def variant_params(module, seed: int = 0, dtype: str = "fp32") -> Dict[str, torch.Tensor]:
    """Seeded values for every tensor of ``module.state_dict()`` (same keys in the reference's class)."""
    g = torch.Generator().manual_seed(seed + 11)
    out = {}
    sd = module.state_dict()
    for k in sorted(sd):  # key order, independent of the class's registration order
        t = sd[k]
        small = k.endswith("bias") or k.endswith("out_proj.weight")
        std = 0.05 if small else (t.shape[-1] ** -0.5)
        out[k] = _round(torch.randn(tuple(t.shape), generator=g) * std, dtype)
    return out


def variant_x(case: dict, seed: int = 0, dtype: str = "fp32") -> torch.Tensor:
    g = torch.Generator().manual_seed(seed + 12)
    return _round(torch.randn(case["x_shape"], generator=g), dtype)


# ---------------------------------------------------------------------------------------------------
# Function-level Pattention (``triton_pattention(x, k_gate, v, k_up, active_blocks, activation)``,
# pattention_triton.py:204-311): one shared active-block list for every token, five activations, the
# gated (SwiGLU, k_up given) and non-gated forms, D_out different from the input width.  Tensors are
# drawn from a generator seeded with ``seed + 21``: x ~ N(0, 1), k_gate / k_up ~ N(0, K^-0.5),
# v ~ N(0, N_p^-0.5); "tc" cases have tensor-core shapes (K, D_out multiples of 64).
# ---------------------------------------------------------------------------------------------------
PATTENTION_CASES: Dict[str, dict] = {
    "swiglu_sparse": dict(M=21, K=256, Np=512, D_out=256, activation="swiglu", gated=True, active=[0, 3, 5]),
    "swiglu_dense": dict(M=21, K=256, Np=512, D_out=256, activation="swiglu", gated=True, active=None),
    "silu": dict(M=33, K=256, Np=512, D_out=192, activation="silu", gated=False, active=[1, 2, 7]),
    "gelu": dict(M=33, K=256, Np=512, D_out=192, activation="gelu", gated=False, active=[6, 0, 4]),
    "relu": dict(M=33, K=256, Np=512, D_out=192, activation="relu", gated=False, active=[2, 3]),
    "relu2": dict(M=33, K=256, Np=512, D_out=192, activation="relu2", gated=False, active=None),
    "gelu_kup_unused": dict(M=9, K=256, Np=512, D_out=256, activation="gelu", gated=True, active=[5, 1]),
    "odd_width": dict(M=17, K=200, Np=256, D_out=136, activation="swiglu", gated=True, active=[3, 1]),
    "swiglu_tc": dict(M=300, K=512, Np=1024, D_out=320, activation="swiglu", gated=True,
                      active=[0, 2, 3, 9, 10, 11, 15]),
    "relu2_tc": dict(M=272, K=512, Np=1024, D_out=192, activation="relu2", gated=False, active=None),
    "silu_tc": dict(M=260, K=384, Np=768, D_out=256, activation="silu", gated=False, active=[11, 4, 7, 0]),
}
# dtypes with golden outputs per case: the tensor-core shapes only in bf16 (fp32 runs on CUDA cores)
PATTENTION_DTYPES = {k: (("bf16",) if k.endswith("_tc") else ("fp32", "bf16")) for k in PATTENTION_CASES}


def pattention_tensors(case: dict, seed: int = 0, dtype: str = "fp32"):
    """(x [M, K], k_gate [Np, K], k_up [Np, K] or None, v [Np, D_out], active int64 or None) of a case."""
    g = torch.Generator().manual_seed(seed + 21)
    M, K, Np, Do = case["M"], case["K"], case["Np"], case["D_out"]
    x = _round(torch.randn(M, K, generator=g), dtype)
    kg = _round(torch.randn(Np, K, generator=g) * K ** -0.5, dtype)
    ku = _round(torch.randn(Np, K, generator=g) * K ** -0.5, dtype)
    v = _round(torch.randn(Np, Do, generator=g) * Np ** -0.5, dtype)
    act = None if case["active"] is None else torch.tensor(case["active"], dtype=torch.int64)
    return x, kg, (ku if case["gated"] else None), v, act


# A dense SwiGLU MLP converted by TritonSwiGLUPattentionMLP.from_dense_mlp (pattention_triton.py:348-368)
PATTENTION_MLP = dict(hidden=256, intermediate=512, x_shape=(2, 5, 256), active=[1, 2, 6])


def pattention_mlp_weights(seed: int = 0):
    """(gate_proj, up_proj, down_proj) weights of the dense MLP (nn.Linear layout) and x."""
    g = torch.Generator().manual_seed(seed + 23)
    h, i = PATTENTION_MLP["hidden"], PATTENTION_MLP["intermediate"]
    wg = torch.randn(i, h, generator=g) * h ** -0.5
    wu = torch.randn(i, h, generator=g) * h ** -0.5
    wd = torch.randn(h, i, generator=g) * i ** -0.5
    x = torch.randn(*PATTENTION_MLP["x_shape"], generator=g)
    return wg, wu, wd, x
