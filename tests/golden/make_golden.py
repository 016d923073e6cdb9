"""Generate golden vectors by running the reference implementation itself.

Run in a container that has the reference checkout (``--ref`` points at the directory holding the
reference's ``foveal_indexer`` package):

    python tests/golden/make_golden.py --ref <path-to-reference-checkout>

It imports the reference's own functions (``FovealPattentionMLP``, ``select_blocks``,
``_pytorch_pattention_fallback``), runs them in fp32 on the seeded synthetic inputs of each
configuration (bf16 configurations use bf16-rounded values in an fp32 module) and writes small
``.npz`` fixtures next to this script.  Weights and inputs are NOT stored: they are regenerated from
the seed by ``configs.make_weights`` / ``configs.make_x``.  The fixtures hold routes, outputs for a
few tokens and the per-token near-tie margins.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
cfgmod = importlib.import_module("foveal-sparse-indexer_b200.configs")
sys.path.insert(0, os.path.dirname(HERE))
from conftest import serve_model  # noqa: E402  (tiny seeded Llama shared with the GPU test)


def load_reference(ref_root: str):
    sys.path.insert(0, ref_root)
    from foveal_indexer.foveal_pattention import FovealPattentionMLP
    from foveal_indexer.core import select_blocks, masked_softmax
    from foveal_indexer.pattention_triton import _pytorch_pattention_fallback
    return FovealPattentionMLP, select_blocks, masked_softmax, _pytorch_pattention_fallback


def build_module(FovealPattentionMLP, wl, w, remote_blocks):
    m = FovealPattentionMLP(hidden_dim=wl.hidden_dim, intermediate_dim=wl.intermediate_dim,
                            block_size=64, base_blocks=wl.base_blocks, remote_blocks=remote_blocks,
                            index_dim=16, temperature=wl.temperature, dtype=torch.float32,
                            use_fused_kernel=False)
    with torch.no_grad():
        sd = m.state_dict()
        for k, t in w.state_dict().items():
            sd[k].copy_(t)
    return m


def margins_from_scores(S, base, counts):
    p = torch.softmax(S.float(), dim=-1)[:, base:]
    sp = p.sort(dim=-1, descending=True, stable=True).values
    c = counts.long().clamp(1, sp.shape[1] - 1)
    ar = torch.arange(S.shape[0])
    return (sp[ar, c - 1] - sp[ar, c]).numpy()


def token_case(ref, wl, x2d, w, n_out):
    FovealPattentionMLP, select_blocks, _, fallback = ref
    m = build_module(FovealPattentionMLP, wl, w, wl.max_remote_blocks)
    with torch.no_grad():
        S = m.compute_router_scores(x2d) / wl.temperature
        r = select_blocks(S[None], causal=False, block_size=64, local_window_blocks=wl.base_blocks,
                          top_p=wl.top_p, min_remote_blocks=wl.min_remote_blocks,
                          max_remote_blocks=wl.max_remote_blocks,
                          remote_capacity=wl.max_remote_blocks)
        idx, cnt = r.remote_indices[0], r.remote_counts[0]
        ys = []
        for t in range(n_out):
            act = torch.cat([torch.arange(wl.base_blocks, dtype=torch.int64),
                             idx[t, :int(cnt[t])].long()])
            y = fallback(x2d[t:t + 1], m.k_gate, m.v, m.k_up, act, "swiglu", 64)
            soft = F.softmax(S[t:t + 1], dim=-1)  # foveal_pattention.py:339 (S already / T)
            y = y + m.out_proj_16d(torch.matmul(soft, m.block_keys_16d))
            ys.append(y[0])
        y = torch.stack(ys) if ys else torch.zeros(0, wl.hidden_dim)
    return {
        "scores": S.numpy().astype(np.float32),
        "remote_indices": idx.numpy().astype(np.int32),
        "remote_counts": cnt.numpy().astype(np.int32),
        "margins": margins_from_scores(S, wl.base_blocks, cnt),
        "cap_rate": np.float32(r.cap_rate), "mean_remote_blocks": np.float32(r.mean_remote_blocks),
        "y": y.numpy().astype(np.float32),
    }


def pooled_case(ref, wl, x, w, remote_blocks, training, n_out):
    FovealPattentionMLP = ref[0]
    m = build_module(FovealPattentionMLP, wl, w, remote_blocks)
    m.train(training)
    with torch.no_grad():
        y, info = m(x, return_router_info=True)
    D = wl.hidden_dim
    y2 = y.reshape(-1, D)[:n_out]
    x2d = x.reshape(-1, D)
    if training:
        ms = info["scores"].mean(dim=0)
    else:
        q = F.rms_norm(m.q_proj_16d(x2d.mean(dim=0, keepdim=True)), (16,))
        ms = torch.matmul(q, m.block_keys_16d.t()).squeeze(0)
    rem = ms[wl.base_blocks:].sort(descending=True).values
    gap = (rem[remote_blocks - 1] - rem[remote_blocks]).item() if remote_blocks < rem.numel() else 1.0
    return {"active_blocks": info["active_blocks"].numpy().astype(np.int32),
            "y": y2.numpy().astype(np.float32), "topk_gap": np.float32(gap)}


def save(name, meta, arrays):
    arrays = {k: np.asarray(v) for k, v in arrays.items()}
    arrays["meta"] = np.array(json.dumps(meta))
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **arrays)
    print(f"wrote {path} ({os.path.getsize(path) / 1024:.0f} KB)")


def flat(prefix, d):
    return {f"{prefix}{k}": v for k, v in d.items()}


CALIB = {"base_blocks": 1, "remote_blocks": 8, "ridge_lambda": 1e-2}


def calib_case(ref, seed):
    """The reference's FovealPattentionMLP.calibrate_offline_svd on bf16-rounded PR1-shape weights and
    512 bf16-rounded calibration tokens (fp32 module).  Stores its returned figures, the calibrated
    router's scores on the calibration tokens (invariant to singular-vector signs) and the teacher block
    energies it fitted (computed with the same expression as foveal_pattention.py:205-216)."""
    FovealPattentionMLP = ref[0]
    wl = cfgmod.calib_workload()
    w, x = cfgmod.make_weights(wl, seed), cfgmod.make_x(wl, seed)
    x2d = x.reshape(-1, wl.hidden_dim)
    m = build_module(FovealPattentionMLP, wl, w, CALIB["remote_blocks"])
    with torch.no_grad():
        A = F.silu(x2d @ m.k_gate.t()) * (x2d @ m.k_up.t())
        teacher = torch.stack([A[:, b * 64:(b + 1) * 64].abs().mean(dim=-1) * m.v[b * 64:(b + 1) * 64].norm()
                               for b in range(m.num_blocks)], dim=-1)
    info = m.calibrate_offline_svd(x2d, ridge_lambda=CALIB["ridge_lambda"])
    with torch.no_grad():
        z = F.rms_norm(x2d @ m.q_proj_16d.weight.t(), (16,))
        scores = z @ m.block_keys_16d.t() / 4.0
    return {"explained": np.float64(info["top16_explained_variance"]),
            "kl": np.float64(info["initial_kl_divergence"]),
            "active": np.array(info["calib_active_blocks"], dtype=np.int32),
            "scores": scores.numpy().astype(np.float32), "teacher": teacher.numpy().astype(np.float32)}


SERVE = {"vocab": 256, "hidden": 512, "intermediate": 2048, "layers": 2, "heads": 8, "prompt": 48, "decode": 8,
         "base_blocks": 2, "remote_blocks": 8, "model_seed": 1234, "prompt_seed": 99}


def serve_case(seed_unused=0):
    """Whole-model surgery and decode serving (foveal_pattention.py:355-387 and the eval cache :278-288,
    :309-325): the reference's sparsify_model_with_foveal_pattention on a tiny Llama, prefill on a
    48-token prompt (routes once, caches the active set), then 8 decode steps fed with the argmax tokens."""
    from foveal_indexer.foveal_pattention import sparsify_model_with_foveal_pattention
    m = serve_model(SERVE)
    sparsify_model_with_foveal_pattention(m, base_blocks=SERVE["base_blocks"], remote_blocks=SERVE["remote_blocks"],
                                          use_fused_kernel=False)
    m.eval()  # the new MLP modules start in training mode; serving runs in eval mode
    g = torch.Generator().manual_seed(SERVE["prompt_seed"])
    ids = torch.randint(0, SERVE["vocab"], (1, SERVE["prompt"]), generator=g)
    with torch.no_grad():
        out = m(ids, use_cache=True)
        prefill = out.logits[0].float()
        past = out.past_key_values
        toks, dec = [], []
        nxt = int(prefill[-1].argmax())
        for _ in range(SERVE["decode"]):
            toks.append(nxt)
            o = m(torch.tensor([[nxt]]), past_key_values=past, use_cache=True)
            past = o.past_key_values
            dec.append(o.logits[0, -1].float())
            nxt = int(dec[-1].argmax())
    active = torch.stack([layer.mlp._cached_active_blocks for layer in m.model.layers])
    return {"prompt": ids.numpy().astype(np.int64), "prefill_logits": prefill.numpy().astype(np.float32),
            "decode_tokens": np.array(toks, dtype=np.int64), "decode_logits": torch.stack(dec).numpy().astype(np.float32),
            "active": active.numpy().astype(np.int32)}


GRAD_NAMES = ("x", "k_gate", "k_up", "v", "q_proj_16d", "block_keys_16d", "out_proj_16d")


def train_case(ref, seed):
    """Training-mode forward and backward of the reference module (pooled routing, additive stream;
    foveal_pattention.py:290-342 under autograd): gradients of x and of every parameter for the loss
    sum(y * dy) with a seeded dy."""
    FovealPattentionMLP = ref[0]
    wl = cfgmod.train_workload()
    w, x = cfgmod.make_weights(wl, seed), cfgmod.make_x(wl, seed)
    m = build_module(FovealPattentionMLP, wl, w, wl.max_remote_blocks)
    m.train()
    x = x.clone().requires_grad_(True)
    dy = torch.randn(x.shape, generator=torch.Generator().manual_seed(seed + 7))
    y, info = m(x, return_router_info=True)
    (y * dy).sum().backward()
    grads = {"x": x.grad, "k_gate": m.k_gate.grad, "k_up": m.k_up.grad, "v": m.v.grad,
             "q_proj_16d": m.q_proj_16d.weight.grad, "block_keys_16d": m.block_keys_16d.grad,
             "out_proj_16d": m.out_proj_16d.weight.grad}
    out = {f"grad_{k}": grads[k].detach().numpy().astype(np.float32) for k in GRAD_NAMES}
    out["y"] = y.detach().numpy().astype(np.float32)
    out["dy"] = dy.numpy().astype(np.float32)
    out["active"] = info["active_blocks"].numpy().astype(np.int32)
    return out


def variants_case(ref_root: str, seed: int):
    """BlockSparseLinear, FovealTokenformerLinear and FovealTokenformerFFN of the reference (fp32 modules;
    the "bf16" entries use bf16-rounded parameters and inputs): outputs in eval without autograd (the
    BlockSparseLinear inference selection) and, for BlockSparseLinear, in training mode under no_grad
    (FovealIndexer.route), with the aux figures, the routes and, for one case each, the distillation
    loss."""
    sys.path.insert(0, ref_root)
    from foveal_indexer.block_matmul import BlockSparseLinear
    from foveal_indexer.tokenformer import FovealTokenformerFFN, FovealTokenformerLinear
    classes = {"bsl": BlockSparseLinear, "tf": FovealTokenformerLinear, "ffn": FovealTokenformerFFN}
    arr = {}
    for name, case in cfgmod.VARIANT_CASES.items():
        for dt in ("fp32", "bf16"):
            pre = f"{name}_{dt}_"
            m = classes[case["kind"]](**cfgmod.variant_kwargs(case))
            m.load_state_dict(cfgmod.variant_params(m, seed, dt))
            x = cfgmod.variant_x(case, seed, dt)
            m.eval()
            with torch.no_grad():
                y, aux = m(x, compute_teacher_loss=(dt == "fp32"))
            arr[pre + "eval_out"] = y.numpy().astype(np.float32)
            if dt == "fp32":
                arr[pre + "distill"] = np.float32(aux["distill_loss"])
            if case["kind"] == "bsl":
                arr[pre + "eval_union"] = np.int32(aux["active_blocks_union"])
                arr[pre + "eval_mean_active"] = np.float64(aux["mean_active_blocks"])
                m.train()
                with torch.no_grad():
                    y, aux = m(x)
                arr[pre + "train_out"] = y.numpy().astype(np.float32)
                arr[pre + "train_union"] = np.int32(aux["active_blocks_union"])
                arr[pre + "train_idx"] = aux["route"].remote_indices.numpy().astype(np.int32)
                arr[pre + "train_cnt"] = aux["route"].remote_counts.numpy().astype(np.int32)
            elif case["kind"] == "tf":
                arr[pre + "eval_union"] = np.int32(aux["active_param_tokens_union"])
                arr[pre + "eval_mean_active"] = np.float64(aux["mean_active_param_tokens"])
                arr[pre + "eval_idx"] = aux["route"].remote_indices.numpy().astype(np.int32)
                arr[pre + "eval_cnt"] = aux["route"].remote_counts.numpy().astype(np.int32)
            else:
                for f in ("fc1", "fc2"):
                    a = aux[f + "_aux"]
                    arr[pre + f + "_union"] = np.int32(a["active_param_tokens_union"])
                    arr[pre + f + "_mean_active"] = np.float64(a["mean_active_param_tokens"])
    return arr


def pattention_case(ref_root: str, seed: int):
    """The reference's function-level Pattention (``_pytorch_pattention_fallback``, the semantics of
    ``triton_pattention``, pattention_triton.py:204-311) on every PATTENTION_CASES entry, fp32 and on
    bf16-rounded values; ``TritonSwiGLUPattentionMLP.from_dense_mlp`` on a seeded dense MLP (sparse and
    dense forward); ``convert_llm_mlp_to_pattention`` on the tiny Llama of the serving case (logits)."""
    sys.path.insert(0, ref_root)
    from foveal_indexer.pattention_triton import (TritonSwiGLUPattentionMLP, _pytorch_pattention_fallback,
                                                  convert_llm_mlp_to_pattention)
    arr = {}
    for name, case in cfgmod.PATTENTION_CASES.items():
        for dt in cfgmod.PATTENTION_DTYPES[name]:
            x, kg, ku, v, act = cfgmod.pattention_tensors(case, seed, dt)
            with torch.no_grad():
                y = _pytorch_pattention_fallback(x, kg, v, ku, act, case["activation"], 64)
            arr[f"{name}_{dt}_y"] = y.numpy().astype(np.float32)

    class Dense(torch.nn.Module):
        def __init__(self, h, i):
            super().__init__()
            self.gate_proj = torch.nn.Linear(h, i, bias=False)
            self.up_proj = torch.nn.Linear(h, i, bias=False)
            self.down_proj = torch.nn.Linear(i, h, bias=False)

    cfg = cfgmod.PATTENTION_MLP
    wg, wu, wd, x = cfgmod.pattention_mlp_weights(seed)
    dense = Dense(cfg["hidden"], cfg["intermediate"])
    with torch.no_grad():
        dense.gate_proj.weight.copy_(wg)
        dense.up_proj.weight.copy_(wu)
        dense.down_proj.weight.copy_(wd)
        mlp = TritonSwiGLUPattentionMLP.from_dense_mlp(dense)
        arr["mlp_sparse_y"] = mlp(x, active_blocks=torch.tensor(cfg["active"])).numpy().astype(np.float32)
        arr["mlp_dense_y"] = mlp(x).numpy().astype(np.float32)
        model = serve_model(SERVE)
        convert_llm_mlp_to_pattention(model)
        ids = torch.randint(0, SERVE["vocab"], (1, 16), generator=torch.Generator().manual_seed(SERVE["prompt_seed"]))
        arr["convert_prompt"] = ids.numpy()
        arr["convert_logits"] = model(ids).logits[0].numpy().astype(np.float32)
        arr["convert_types"] = np.array([type(layer.mlp).__name__ for layer in model.model.layers])
    return arr


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--only", default="", help="comma-separated fixture names to regenerate (default: all)")
    args = ap.parse_args()
    ref = load_reference(args.ref)
    torch.set_num_threads(os.cpu_count())
    C = cfgmod.CONFIGS
    meta_common = {"seed": args.seed, "torch": torch.__version__}
    only = set(filter(None, args.only.split(",")))
    if only and only <= {"calib", "serve", "train", "variants", "pattention"}:
        if "pattention" in only:
            save("pattention", {**meta_common, "config": "pattention", "cases": cfgmod.PATTENTION_CASES,
                                "mlp": cfgmod.PATTENTION_MLP, "serve": SERVE}, pattention_case(args.ref, args.seed))
        if "variants" in only:
            save("variants", {**meta_common, "config": "variants", "cases": cfgmod.VARIANT_CASES},
                 variants_case(args.ref, args.seed))
        if "calib" in only:
            save("calib", {**meta_common, "config": "calib", **CALIB}, calib_case(ref, args.seed))
        if "serve" in only:
            save("serve", {**meta_common, "config": "serve", **SERVE}, serve_case())
        if "train" in only:
            save("train", {**meta_common, "config": "train"}, train_case(ref, args.seed))
        return

    # 1. PR1 (fp32, full size): token mode, pooled eval and pooled train.
    wl = C["pr1"]
    w, x = cfgmod.make_weights(wl, args.seed), cfgmod.make_x(wl, args.seed)
    x2d = x.reshape(-1, wl.hidden_dim)
    arr = flat("tok_", token_case(ref, wl, x2d, w, n_out=x2d.shape[0]))
    arr.update(flat("peval_", pooled_case(ref, wl, x, w, wl.max_remote_blocks, False, 512)))
    arr.update(flat("ptrain_", pooled_case(ref, wl, x, w, wl.max_remote_blocks, True, 512)))
    save("pr1", {**meta_common, "config": "pr1"}, arr)

    # 2. Decode (bf16 values, fp32 math): K_max in {8, 16, 32}, all 64 tokens.
    arr = {}
    for wl in cfgmod.decode_points():
        w, x = cfgmod.make_weights(wl, args.seed), cfgmod.make_x(wl, args.seed)
        x2d = x.reshape(-1, wl.hidden_dim)
        arr.update(flat(f"k{wl.max_remote_blocks}_", token_case(ref, wl, x2d, w, n_out=64)))
        if wl.max_remote_blocks == 16:
            arr.update(flat("peval_", pooled_case(ref, wl, x, w, 16, False, 64)))
    save("decode", {**meta_common, "config": "decode", "kmax": list(cfgmod.DECODE_KMAX)}, arr)

    # 3. 8B slice: first 128 tokens; outputs for 16 of them.
    wl = C["8b"]
    w, x = cfgmod.make_weights(wl, args.seed), cfgmod.make_x(wl, args.seed)
    xs = x.reshape(-1, wl.hidden_dim)[:128].contiguous()
    arr = flat("tok_", token_case(ref, wl, xs, w, n_out=16))
    arr.update(flat("peval_", pooled_case(ref, wl, xs.view(1, 128, -1), w, 20, False, 16)))
    save("8b_slice", {**meta_common, "config": "8b", "tokens": 128}, arr)
    del w, x

    # 4. 70B slice: first 64 tokens; outputs for 4 of them.
    wl = C["70b"]
    w, x = cfgmod.make_weights(wl, args.seed), cfgmod.make_x(wl, args.seed)
    xs = x.reshape(-1, wl.hidden_dim)[:64].contiguous()
    save("70b_slice", {**meta_common, "config": "70b", "tokens": 64},
         flat("tok_", token_case(ref, wl, xs, w, n_out=4)))
    del w, x

    # 5. Sweep: routes for the first 64 tokens at all 20 points, outputs for 4 tokens at two.
    arr = {}
    pts = cfgmod.sweep_points()
    w = cfgmod.make_weights(pts[0], args.seed)
    x = cfgmod.make_x(pts[0], args.seed)
    xs = x.reshape(-1, pts[0].hidden_dim)[:64].contiguous()
    for i, wl in enumerate(pts):
        n_out = 4 if (wl.top_p, wl.max_remote_blocks) in ((0.3, 14), (1.0, 224)) else 0
        d = token_case(ref, wl, xs, w, n_out=n_out)
        d.pop("scores")
        arr.update(flat(f"p{i}_", d))
    save("sweep_slice", {**meta_common, "config": "sweep",
                         "points": [[p.top_p, p.max_remote_blocks, p.min_remote_blocks] for p in pts]},
         arr)

    # 6. Router known-answer cases from the reference's own tests plus a peaked case where top-p
    #    binds (counts vary between K_min and K_max).
    FovealPattentionMLP, select_blocks, masked_softmax, _ = ref
    scores = torch.tensor([[1.0, 2.0, 3.0], [4.0, 5.0, 6.0]])
    mask = torch.tensor([[True, True, False], [False, True, True]])
    arr = {"ms_scores": scores.numpy(), "ms_mask": mask.numpy(),
           "ms_probs": masked_softmax(scores, mask).numpy()}
    g = torch.Generator().manual_seed(1234)
    for name, (B, Q, NB, base, tp, kmin, kmax, cap, scale) in {
        "guard": (2, 8, 8, 2, 0.99, 1, 3, 4, 1.0),      # tests/test_indexer.py:42-61
        "peaked": (1, 256, 32, 1, 0.9, 2, 8, 8, 6.0),
        "wide": (1, 128, 224, 4, 0.5, 0, 56, 56, 20.0),
        "nobase": (1, 64, 40, 0, 0.7, 3, 12, 16, 8.0),
    }.items():
        s = torch.randn(B, Q, NB, generator=g) * scale
        r = select_blocks(s, causal=False, local_window_blocks=base, top_p=tp,
                          min_remote_blocks=kmin, max_remote_blocks=kmax, remote_capacity=cap)
        arr[f"{name}_scores"] = s.numpy()
        arr[f"{name}_params"] = np.array([base, tp, kmin, kmax, cap], dtype=np.float64)
        arr[f"{name}_indices"] = r.remote_indices.numpy()
        arr[f"{name}_counts"] = r.remote_counts.numpy()
        arr[f"{name}_cap_rate"] = np.float32(r.cap_rate)
    save("router_kat", {**meta_common, "config": "router"}, arr)

    # 7. Offline SVD router calibration.
    save("calib", {**meta_common, "config": "calib", **CALIB}, calib_case(ref, args.seed))

    # 8. Whole-model surgery and decode serving with the active-set cache.
    save("serve", {**meta_common, "config": "serve", **SERVE}, serve_case())

    # 9. Training-mode forward and backward (pooled routing, additive stream).
    save("train", {**meta_common, "config": "train"}, train_case(ref, args.seed))

    # 10. Layers that share the router: BlockSparseLinear, FovealTokenformerLinear / FFN.
    save("variants", {**meta_common, "config": "variants", "cases": cfgmod.VARIANT_CASES},
         variants_case(args.ref, args.seed))

    # 11. Function-level Pattention (five activations, gated and non-gated), its MLP module and the model
    #     conversion helper.
    save("pattention", {**meta_common, "config": "pattention", "cases": cfgmod.PATTENTION_CASES,
                        "mlp": cfgmod.PATTENTION_MLP, "serve": SERVE}, pattention_case(args.ref, args.seed))


if __name__ == "__main__":
    main()
