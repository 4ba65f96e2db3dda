"""Precision verification on the dump files (host side).

The reference checks an implementation by dumping logits at chosen decode
steps (``Inference_gpt2/dump_utils.h``) and scoring them against a reference
model with ``verify_precision.py``.  The engine writes the same files
(``Engine.generate_dump`` / ``gpt2b_engine_generate_dump``); this module reads
them and scores two logit vectors with the same metric definitions and
pass/fail tiers (verify_precision.py:37-46 thresholds, :177-223 metrics), so
the reference's validation can run on this engine's output once real weights
are available.

Metrics of reference logits ``a`` against tested logits ``b``:
  cosine        a.b / (|a||b| + 1e-12) in float64, clipped to [-1, 1]
  max_abs, mean_abs of |a - b|
  rel_p50/p95/p99, mean_rel   percentiles / mean of |a - b| / (|a| + 1e-5), in %
  kl            sum p_a log(p_a / (p_b + 1e-12)) with the ratio clipped below at 1e-12
  top1_ok, top5_overlap       stable descending order (ties: lower index first)
"""
from __future__ import annotations

import os

import numpy as np

# pass tiers (verify_precision.py:37-46)
PERFECT_COSINE, PERFECT_MEAN_ABS, PERFECT_KL = 0.99, 0.25, 0.01
BASIC_COSINE, BASIC_MEAN_ABS = 0.95, 2.0
QUANT_COSINE, QUANT_MEAN_ABS, QUANT_KL = 0.99, 3.0, 0.3


def stable_topk(logits, k: int = 5) -> np.ndarray:
    """Indices of the k largest logits, ties broken by the lower index."""
    return np.argsort(-np.asarray(logits), kind="stable")[:k]


def _softmax(x: np.ndarray) -> np.ndarray:
    e = np.exp(x - x.max())
    return e / e.sum()


def compute_metrics(a, b) -> dict:
    """Scores of tested logits ``b`` against reference logits ``a``."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    cosine = float(np.clip(a64 @ b64 / (np.linalg.norm(a64) * np.linalg.norm(b64) + 1e-12), -1.0, 1.0))
    diff = np.abs(a - b)
    rel = diff / (np.abs(a) + 1e-5)
    ta, tb = stable_topk(a), stable_topk(b)
    pa, pb = _softmax(a), _softmax(b)
    kl = float(np.sum(pa * np.log(np.clip(pa / (pb + 1e-12), 1e-12, None))))
    return {
        "top1_ok": bool(ta[0] == tb[0]), "top1_a": int(ta[0]), "top1_b": int(tb[0]),
        "top5_overlap": len(set(ta.tolist()) & set(tb.tolist())),
        "cosine": cosine, "max_abs": float(diff.max()), "mean_abs": float(diff.mean()),
        "rel_p50": float(np.percentile(rel, 50) * 100), "rel_p95": float(np.percentile(rel, 95) * 100),
        "rel_p99": float(np.percentile(rel, 99) * 100), "mean_rel": float(rel.mean() * 100), "kl": kl,
    }


def verdict(m: dict, quant: bool = False) -> tuple[str, bool]:
    """("perfect" | "basic" | "quantised" | "fail", passed) for metrics ``m``;
    8-bit weights are judged on the looser quantised tier."""
    top = m["top1_ok"] and m["top5_overlap"] >= 4
    if quant:
        ok = top and m["cosine"] >= QUANT_COSINE and m["mean_abs"] < QUANT_MEAN_ABS and m["kl"] < QUANT_KL
        return ("quantised", True) if ok else ("fail", False)
    if top and m["cosine"] >= PERFECT_COSINE and m["mean_abs"] < PERFECT_MEAN_ABS and m["kl"] < PERFECT_KL:
        return "perfect", True
    if top and m["cosine"] >= BASIC_COSINE and m["mean_abs"] < BASIC_MEAN_ABS:
        return "basic", True
    return "fail", False


def nll(logits, token: int) -> float:
    """log(sum exp(logits)) - logits[token], max-shifted, summed in float64
    (the engine computes the same quantity on the device)."""
    x = np.asarray(logits, np.float32)
    mx = float(x.max())
    return float(np.float32(mx + np.log(np.sum(np.exp(x.astype(np.float64) - mx))) - float(x[token])))


def ppl_summary(nlls) -> dict:
    """Mean NLL and perplexity exp(mean NLL) of a run."""
    v = np.asarray(nlls, np.float64)
    mean = float(v.mean()) if v.size else float("nan")
    return {"steps": int(v.size), "mean_nll": mean, "ppl": float(np.exp(mean)) if v.size else float("nan")}


# ----------------------------------------------------------------------------
# the dump files
# ----------------------------------------------------------------------------
def read_logits(dump_dir: str, prefix: str, step: int | None = None) -> np.ndarray:
    """<prefix>_logits_step<step>.bin, or <prefix>_logits_t1.bin for step None."""
    name = f"{prefix}_logits_t1.bin" if step is None else f"{prefix}_logits_step{step}.bin"
    return np.fromfile(os.path.join(dump_dir, name), dtype=np.float32)


def read_inputs(dump_dir: str, prefix: str, step: int) -> np.ndarray:
    """<prefix>_inputs_step<step>.bin: the tokens fed before step ``step``."""
    return np.fromfile(os.path.join(dump_dir, f"{prefix}_inputs_step{step}.bin"), dtype=np.int32)


def read_ppl(dump_dir: str, prefix: str) -> tuple[np.ndarray, np.ndarray]:
    """(nll per step, appended token per step) of ppl_<prefix>_*.bin."""
    return (np.fromfile(os.path.join(dump_dir, f"ppl_{prefix}_nll.bin"), dtype=np.float32),
            np.fromfile(os.path.join(dump_dir, f"ppl_{prefix}_tokens.bin"), dtype=np.int32))


def dumped_steps(dump_dir: str, prefix: str) -> list[int]:
    """Steps with a <prefix>_logits_step<t>.bin file, ascending."""
    head, tail = f"{prefix}_logits_step", ".bin"
    out = []
    for f in os.listdir(dump_dir):
        if f.startswith(head) and f.endswith(tail) and f[len(head):-len(tail)].isdigit():
            out.append(int(f[len(head):-len(tail)]))
    return sorted(out)


def compare_dumps(ref_dir: str, ref_prefix: str, test_dir: str, test_prefix: str, quant: bool = False) -> dict:
    """Every step dumped under both prefixes (and step 1): metrics and verdict
    of the tested logits against the reference logits.  The input prefixes
    must agree for a step to be compared."""
    rows = {}
    steps = sorted(set(dumped_steps(ref_dir, ref_prefix)) & set(dumped_steps(test_dir, test_prefix)))
    for t in steps:
        if not np.array_equal(read_inputs(ref_dir, ref_prefix, t), read_inputs(test_dir, test_prefix, t)):
            rows[t] = {"skipped": "different input prefixes"}
            continue
        m = compute_metrics(read_logits(ref_dir, ref_prefix, t), read_logits(test_dir, test_prefix, t))
        m["verdict"], m["passed"] = verdict(m, quant)
        rows[t] = m
    return rows
