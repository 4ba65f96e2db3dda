"""The verification metrics (host side, no GPU): the definitions and pass
tiers of the reference's verify_precision.py (:37-46, :177-223), checked on
hand-built logit vectors, and the dump-file readers on files written in the
reference's layout (Inference_gpt2/dump_utils.h)."""
from __future__ import annotations

import os

import numpy as np
import pytest


def test_identical_logits_are_perfect():
    from cuda_gpt2_inference_b200 import verify
    a = np.random.default_rng(0).standard_normal(1000).astype(np.float32)
    m = verify.compute_metrics(a, a)
    assert m["cosine"] == pytest.approx(1.0, abs=1e-12)
    assert m["max_abs"] == 0.0 and m["mean_abs"] == 0.0 and m["kl"] == pytest.approx(0.0, abs=1e-9)
    assert m["top1_ok"] and m["top5_overlap"] == 5
    assert verify.verdict(m) == ("perfect", True)


def test_metric_values_by_hand():
    from cuda_gpt2_inference_b200 import verify
    a = np.array([3.0, 1.0, 0.0, -1.0, 2.0, 0.5], np.float32)
    b = np.array([2.5, 1.5, 0.0, -1.0, 2.0, 0.5], np.float32)
    m = verify.compute_metrics(a, b)
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    assert m["cosine"] == pytest.approx(float(a64 @ b64 / (np.linalg.norm(a64) * np.linalg.norm(b64))), rel=1e-9)
    assert m["max_abs"] == pytest.approx(0.5) and m["mean_abs"] == pytest.approx(1.0 / 6.0)
    pa = np.exp(a - a.max()); pa /= pa.sum()
    pb = np.exp(b - b.max()); pb /= pb.sum()
    assert m["kl"] == pytest.approx(float(np.sum(pa * np.log(pa / pb))), rel=1e-5)
    rel = np.abs(a - b) / (np.abs(a) + 1e-5)
    assert m["rel_p50"] == pytest.approx(np.percentile(rel, 50) * 100)
    assert m["top1_ok"] and m["top1_a"] == 0


def test_ties_break_to_the_lower_index():
    from cuda_gpt2_inference_b200 import verify
    x = np.array([1.0, 5.0, 5.0, 2.0, 5.0, 0.0], np.float32)
    assert verify.stable_topk(x, 4).tolist() == [1, 2, 4, 3]


def test_verdict_tiers():
    from cuda_gpt2_inference_b200 import verify
    base = {"top1_ok": True, "top5_overlap": 5, "cosine": 0.999, "mean_abs": 0.1, "kl": 0.001}
    assert verify.verdict(base) == ("perfect", True)
    assert verify.verdict(dict(base, kl=0.05)) == ("basic", True)          # KL above the perfect tier
    assert verify.verdict(dict(base, cosine=0.96, mean_abs=1.0)) == ("basic", True)
    assert verify.verdict(dict(base, cosine=0.9)) == ("fail", False)
    assert verify.verdict(dict(base, top5_overlap=3)) == ("fail", False)
    assert verify.verdict(dict(base, mean_abs=2.5, kl=0.2), quant=True) == ("quantised", True)
    assert verify.verdict(dict(base, kl=0.31), quant=True) == ("fail", False)


def test_nll_and_ppl():
    from cuda_gpt2_inference_b200 import verify
    x = np.array([0.0, 0.0, 0.0, 0.0], np.float32)
    assert verify.nll(x, 2) == pytest.approx(np.log(4.0), rel=1e-6)
    big = np.array([1000.0, 0.0], np.float32)  # max-shifted: no overflow
    assert verify.nll(big, 0) == pytest.approx(0.0, abs=1e-6)
    s = verify.ppl_summary([np.log(4.0), np.log(4.0)])
    assert s["steps"] == 2 and s["ppl"] == pytest.approx(4.0)


def test_dump_readers_and_comparison(tmp_path):
    from cuda_gpt2_inference_b200 import verify
    rng = np.random.default_rng(1)
    d = str(tmp_path)
    for prefix, noise in (("ref", 0.0), ("opt_bf16", 1e-3)):
        for t in (1, 5, 9):
            a = rng.standard_normal(50).astype(np.float32) if prefix == "ref" else None
            if prefix == "ref":
                a.tofile(os.path.join(d, f"ref_logits_step{t}.bin"))
            else:
                a = verify.read_logits(d, "ref", t) + np.float32(noise)
                a.astype(np.float32).tofile(os.path.join(d, f"{prefix}_logits_step{t}.bin"))
            np.arange(t, dtype=np.int32).tofile(os.path.join(d, f"{prefix}_inputs_step{t}.bin"))
    np.array([7, 8], np.int32).tofile(os.path.join(d, "opt_bf16_inputs_step9.bin"))  # a different prefix at step 9
    assert verify.dumped_steps(d, "opt_bf16") == [1, 5, 9]
    rows = verify.compare_dumps(d, "ref", d, "opt_bf16")
    assert rows[1]["passed"] and rows[5]["verdict"] == "perfect"
    assert rows[9] == {"skipped": "different input prefixes"}
    np.array([1.5, 2.5], np.float32).tofile(os.path.join(d, "ppl_x_nll.bin"))
    np.array([3, 4], np.int32).tofile(os.path.join(d, "ppl_x_tokens.bin"))
    n, t = verify.read_ppl(d, "x")
    assert n.tolist() == [1.5, 2.5] and t.tolist() == [3, 4]
