"""Shared test setup.

* ``gpu`` marker: tests that need a B200 (``pytest -m gpu``); everything else runs on the CPU.
* ``fsi``: the package under test (directory ``foveal-sparse-indexer_b200``, imported by path).
* ``golden(name)``: loads a fixture from ``tests/golden`` (written by ``tests/golden/make_golden.py``
  from the reference implementation itself).
"""

from __future__ import annotations

import importlib
import json
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
if REPO not in sys.path:
    sys.path.insert(0, REPO)

fsi = importlib.import_module("foveal-sparse-indexer_b200")
configs = fsi.configs


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200) and the built CUDA library")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


class Golden(dict):
    meta: dict


def golden(name: str) -> Golden:
    path = os.path.join(HERE, "golden", f"{name}.npz")
    z = np.load(path, allow_pickle=False)
    g = Golden({k: z[k] for k in z.files if k != "meta"})
    g.meta = json.loads(str(z["meta"]))
    return g


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """||a - b|| / ||b|| in fp64."""
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def max_rel(a: torch.Tensor, b: torch.Tensor) -> float:
    """max|a - b| / max|b|."""
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def route_sets(idx, cnt):
    idx = np.asarray(idx)
    cnt = np.asarray(cnt)
    return [frozenset(idx[t, :int(cnt[t])].tolist()) for t in range(len(cnt))]


# Probabilities closer than this (fp32, absolute) at the selection boundary are rounding-level near
# ties: p[K-1] - p[K] < TIE_EPS.  Two correct fp32 implementations may order such a pair differently
# (exp, the softmax denominator and the D-long projection round differently on every platform), so a
# differing set there is counted and reported, not failed.  A margin of exactly 0 in the reference's
# fp32 values is a coincidence of that implementation's rounding unless both sides compute the two
# probabilities from identical inputs (repeated block keys, equal scores); there the tie is bit-equal on
# both sides, the lower block id must win, and ``strict_exact=True`` fails any differing set.
TIE_EPS = 2e-8
# Cumulative masses (~0.1-1, fp32 ulp up to 6e-8) closer than this to the top-p target decide the count
# by their last bits: each probability may differ by an ulp between implementations, and the prefix sums
# carry ~150 of them.
COUNT_EPS = 2e-7

# Tie accounting of every route comparison made in this session, printed at the end of the run.
TIE_REPORTS: list = []


class RouteTieReport(dict):
    """Per-comparison route accounting: tokens; mismatches outside the band; tokens in the band
    (reference margin in [0, TIE_EPS)) and how many of them differ; the margin-0 tokens among them and how
    many of those differ; the smallest and largest reference margin among differing tokens (None when
    every set matches)."""


def compare_routes(idx, cnt, ref_idx, ref_cnt, margins=None, tie_eps: float = TIE_EPS, label: str = "",
                   strict_exact: bool = False, count_margins=None):
    """Counts must match exactly; selected sets must match exactly except on tokens whose reference
    boundary margin is below ``tie_eps``.  With ``strict_exact`` (both sides compute bit-equal
    probabilities for tied blocks) margin-0 tokens are not excused: the lower id must win.  Returns
    (n_mismatch_not_excused, n_in_band) and records a :class:`RouteTieReport` in ``TIE_REPORTS`` when
    ``label`` is given.  ``count_margins`` (the oracle's distance of the top-p target from the deciding
    cumulative mass) adds the tokens whose count sits within ``COUNT_EPS`` of flipping to the band."""
    cnt = np.asarray(cnt)
    ref_cnt = np.asarray(ref_cnt)
    a, b = route_sets(idx, cnt), route_sets(ref_idx, ref_cnt)
    m = None if margins is None else np.asarray(margins, dtype=np.float64)
    cm = None if count_margins is None else np.asarray(count_margins, dtype=np.float64).reshape(-1)
    rep = RouteTieReport(label=label, tokens=len(a), differ_outside_band=0, in_band=0, in_band_differ=0,
                         exact_ties=0, exact_tie_differ=0, min_margin_differ=None, max_margin_differ=None,
                         strict_exact=strict_exact, count_band=0, count_band_differ=0)
    for t in range(len(a)):
        mt = None if m is None else float(m[t])
        exact = mt is not None and mt == 0.0
        count_near = cm is not None and float(cm[t]) < COUNT_EPS
        rep["count_band"] += int(count_near)
        near = (mt is not None and mt < tie_eps and not (exact and strict_exact)) or count_near
        rep["exact_ties"] += int(exact)
        rep["in_band"] += int(near)
        if a[t] != b[t] or cnt[t] != ref_cnt[t]:
            if exact:
                rep["exact_tie_differ"] += 1
            if count_near:
                rep["count_band_differ"] += 1
            if near:
                rep["in_band_differ"] += 1
            else:
                rep["differ_outside_band"] += 1
            if mt is not None:
                lo, hi = rep["min_margin_differ"], rep["max_margin_differ"]
                rep["min_margin_differ"] = mt if lo is None else min(lo, mt)
                rep["max_margin_differ"] = mt if hi is None else max(hi, mt)
    if label:
        TIE_REPORTS.append(rep)
        path = os.environ.get("FP_TIE_REPORT")
        if path:
            with open(path, "a") as f:
                f.write(json.dumps(dict(rep)) + "\n")
    return rep["differ_outside_band"], rep["in_band"]


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """One line per route comparison: how many tokens sat in the rounding band and how many of those
    differed (every difference outside the band, or on a bit-equal tie, already failed its test)."""
    if not TIE_REPORTS:
        return
    tr = terminalreporter
    tr.section("route tie accounting (TIE_EPS = %.0e)" % TIE_EPS)
    for r in TIE_REPORTS:
        mg = "-" if r["min_margin_differ"] is None else "%.2e..%.2e" % (r["min_margin_differ"],
                                                                      r["max_margin_differ"])
        eq = "bit-equal on both sides" if r["strict_exact"] else "margin 0 in the reference"
        tr.write_line(f"{r['label']}: tokens {r['tokens']}, in band {r['in_band']} (differ {r['in_band_differ']}), "
                      f"{eq} {r['exact_ties']} (differ {r['exact_tie_differ']}), "
                      f"count band {r['count_band']} (differ {r['count_band_differ']}), "
                      f"differ outside {r['differ_outside_band']}, set margins of differing {mg}")


def active_set_matches(active, gold_scores, base: int, remote: int, rel_tol: float) -> bool:
    """Calibrated active set (base blocks + top ``remote`` mean scores) against the reference's
    calibration scores: blocks may differ only where the reference's mean scores sit within
    ``rel_tol`` (relative to their mean magnitude) of the top-``remote`` boundary."""
    ms = torch.as_tensor(gold_scores).double().mean(dim=0)
    rem = ms[base:]
    order = rem.sort(descending=True).values
    thr = 0.5 * float(order[remote - 1] + order[remote])
    tol = rel_tol * float(rem.abs().mean())
    gold = set(range(base)) | {int(b) + base for b in rem.topk(remote).indices}
    mine = set(int(b) for b in active)
    if len(mine) != base + remote or not set(range(base)) <= mine:
        return False
    return all(abs(float(ms[b]) - thr) <= tol for b in mine ^ gold)


def serve_model(cfgd: dict, dtype=torch.float32):
    """Tiny seeded Llama causal LM for the whole-model serving case (random init from the seed, weights
    rounded to bf16 values), built identically by tests/golden/make_golden.py and the GPU test."""
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=cfgd["vocab"], hidden_size=cfgd["hidden"], intermediate_size=cfgd["intermediate"],
                      num_hidden_layers=cfgd["layers"], num_attention_heads=cfgd["heads"],
                      num_key_value_heads=cfgd["heads"], max_position_embeddings=256)
    torch.manual_seed(cfgd["model_seed"])
    m = LlamaForCausalLM(cfg).eval()
    with torch.no_grad():
        for p_ in m.parameters():
            p_.copy_(p_.to(torch.bfloat16).float())
    return m.to(dtype)


# ---------------------------------------------------------------- layers that share the router
VARIANT_NAMES = list(configs.VARIANT_CASES)


def variant_setup(name: str, dt: str = "fp32"):
    """(case, seeded parameters keyed like the module's state_dict, x) of a parity case; the same values
    the golden generator loaded into the reference's module."""
    case = configs.VARIANT_CASES[name]
    cls = {"bsl": fsi.BlockSparseLinear, "tf": fsi.FovealTokenformerLinear,
           "ffn": fsi.FovealTokenformerFFN}[case["kind"]]
    m = cls(**configs.variant_kwargs(case))
    return case, configs.variant_params(m, 0, dt), configs.variant_x(case, 0, dt)


def tf_kwargs(case: dict, layer: str = ""):
    """Keyword arguments of one Tokenformer layer of a "tf" case or of layer "fc1" / "fc2" of an "ffn" case."""
    if case["kind"] == "tf":
        return {k: case[k] for k in ("in_features", "out_features", "base_blocks", "top_p", "min_remote_blocks",
                                     "max_remote_blocks", "remote_capacity", "activation")}
    h, i = case["hidden_size"], case["intermediate_size"]
    return dict(in_features=h if layer == "fc1" else i, out_features=i if layer == "fc1" else h,
                base_blocks=case["base_blocks"], top_p=case["top_p"], min_remote_blocks=0,
                max_remote_blocks=case["max_remote_blocks"], remote_capacity=4,
                activation="gelu_l2" if layer == "fc1" else "softmax")
