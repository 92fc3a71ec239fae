"""Accuracy-gate scorer (TEST INFRASTRUCTURE ONLY -- see oracle/golden.py header).

Restatement of the reference's `compare_gate` (benchmark/gate.py:16-121): a candidate's last-position
top-k log-probabilities are scored against a reference dump, set by set, and the gate verdicts are
taken from the aggregate.  Per sequence (gate.py:33-78):

* cosine of the log-prob vectors over the union of both top-k id sets, an id missing on one side
  taking that side's k-th (smallest) logprob; cosine of the probability vectors with missing = 0;
* top-1 agreement, and the tie-aware top-1 (a flip counts only if the candidate's top-1 sits more
  than 0.1 nats below the reference top-1 under the reference distribution and the candidate does not
  rank the reference top-1 as tied-best within 1e-6);
* the same two top-1 figures for the no-logprobs sampled token when the candidate carries one;
* overlap of the id sets, |Δ logprob| of the reference top-1, mean |Δ logprob| over the reference
  top-k, the fraction of reference top-k ids missing from the candidate, and KL(ref || cand) over the
  reference top-k with both sides renormalised there.

Aggregates and verdicts (gate.py:79-121): means over sets and over all sequences, rounded like the
reference; `gate_quantized_pass` (top-1 >= 0.95, mean cos_logprob >= 0.99), `exact_match_top1_all`,
and `gate_v2` (tie-aware top-1 >= 0.95 and cos_logprob >= 0.99, then PASS if mean |Δ logprob| <= 0.10,
FAIL above 0.15, JUDGE between).

Pinned against the reference's own reports: tests/golden/gate_cases.json (made by
tests/golden/make_golden.py from the reference's gate.py) is checked by tests/test_oracle.py.
"""

from __future__ import annotations

import math
from statistics import mean
from typing import Dict, List, Optional


def _cosine(a: List[float], b: List[float]) -> float:
    na, nb = math.sqrt(sum(x * x for x in a)), math.sqrt(sum(y * y for y in b))
    if na == 0 or nb == 0:
        return 0.0
    return sum(x * y for x, y in zip(a, b)) / (na * nb)


def _seq_metrics(r: Dict, c: Dict) -> Dict[str, Optional[float]]:
    rmap = dict(zip(r["top_ids"], r["top_logprobs"]))
    cmap = dict(zip(c["top_ids"], c["top_logprobs"]))
    r_floor, c_floor = min(r["top_logprobs"]), min(c["top_logprobs"])
    ids = sorted(set(rmap) | set(cmap))
    lr = [rmap.get(t, r_floor) for t in ids]
    lc = [cmap.get(t, c_floor) for t in ids]
    pr = [math.exp(x) if t in rmap else 0.0 for t, x in zip(ids, lr)]
    pc = [math.exp(x) if t in cmap else 0.0 for t, x in zip(ids, lc)]

    ref_top, cand_top = r["top_ids"][0], c["top_ids"][0]
    r1, c1 = r["top_logprobs"][0], c["top_logprobs"][0]
    c_at_ref_top = cmap.get(ref_top, c_floor)
    cand_tied = (c1 - c_at_ref_top) <= 1e-6
    m: Dict[str, Optional[float]] = {
        "cos_lp": _cosine(lr, lc),
        "cos_p": _cosine(pr, pc),
        "top1": float(ref_top == cand_top),
        "overlap": len(set(rmap) & set(cmap)) / max(1, len(rmap)),
        "d_top1": abs(r1 - c_at_ref_top),
        "tie": float((r1 - rmap.get(cand_top, r_floor)) <= 0.1 or cand_tied),
        "nolp": None,
        "tie_nolp": None,
    }
    if "sampled_nolp" in c:
        s = c["sampled_nolp"]
        m["nolp"] = float(s == ref_top)
        m["tie_nolp"] = float((r1 - rmap.get(s, r_floor)) <= 0.1 or (cand_tied and cmap.get(s, c_floor) >= c1 - 1e-6))
    diffs = [abs(lp - cmap.get(t, c_floor)) for t, lp in zip(r["top_ids"], r["top_logprobs"])]
    m["dlp"] = sum(diffs) / len(diffs)
    m["miss"] = sum(t not in cmap for t in r["top_ids"]) / len(r["top_ids"])
    p_ref = [math.exp(x) for x in r["top_logprobs"]]
    q_cand = [math.exp(cmap.get(t, c_floor)) for t in r["top_ids"]]
    zp, zq = sum(p_ref), sum(q_cand)
    m["kl"] = sum((p / zp) * (math.log(p / zp) - math.log(q / zq)) for p, q in zip(p_ref, q_cand))
    return m


def _m(vals, nd):
    return round(mean(vals), nd) if vals else None


def compare_gate(ref_res: List[Dict], cand_res: List[Dict]) -> Dict:
    """Score candidate top-k dumps against reference ones (benchmark/gate.py:16-121)."""
    if len(ref_res) != len(cand_res):
        raise AssertionError(f"gate: {len(ref_res)} reference sets vs {len(cand_res)} candidate sets")
    per_set, every = [], []
    for rs, cs in zip(ref_res, cand_res):
        if (rs["batch_size"], rs["seq_len"]) != (cs["batch_size"], cs["seq_len"]):
            raise AssertionError("gate: set shapes differ")
        if len(rs["seqs"]) != len(cs["seqs"]):
            raise AssertionError(f"gate: set {rs['batch_size']}x{rs['seq_len']} sequence count differs")
        ms = [_seq_metrics(r, c) for r, c in zip(rs["seqs"], cs["seqs"])]
        every += ms
        col = lambda k: [m[k] for m in ms if m[k] is not None]  # noqa: E731
        per_set.append({
            "shape": f"({rs['batch_size']},{rs['seq_len']})", "n": len(ms),
            "top1_agreement": _m(col("top1"), 4),
            "top1_agreement_nolp": _m(col("nolp"), 4),
            "top1_tie_aware": _m(col("tie"), 4),
            "top1_tie_aware_nolp": _m(col("tie_nolp"), 4),
            "mean_abs_dlogprob": _m(col("dlp"), 5), "max_seq_abs_dlogprob": round(max(col("dlp")), 5),
            "kl_top20_mean": _m(col("kl"), 6),
            "ref_top20_missing_frac": _m(col("miss"), 4),
            "cos_logprob_mean": _m(col("cos_lp"), 6), "cos_logprob_min": round(min(col("cos_lp")), 6),
            "cos_prob_mean": _m(col("cos_p"), 6), "cos_prob_min": round(min(col("cos_p")), 6),
            "topk_overlap_mean": _m(col("overlap"), 4),
            "ref_top1_logprob_absdiff_max": round(max(col("d_top1")), 5),
        })
    col = lambda k: [m[k] for m in every if m[k] is not None]  # noqa: E731
    rep = {"sets": per_set,
           "top1_agreement": _m(col("top1"), 4), "top1_agreement_nolp": _m(col("nolp"), 4),
           "top1_tie_aware": _m(col("tie"), 4), "top1_tie_aware_nolp": _m(col("tie_nolp"), 4),
           "mean_abs_dlogprob": _m(col("dlp"), 5), "kl_top20_mean": _m(col("kl"), 6),
           "ref_top20_missing_frac": _m(col("miss"), 4),
           "cos_logprob_mean": _m(col("cos_lp"), 6), "cos_logprob_min": round(min(col("cos_lp")), 6),
           "cos_prob_mean": _m(col("cos_p"), 6), "n_seqs": len(every)}
    nolp_ok = rep["top1_agreement_nolp"] is None or rep["top1_agreement_nolp"] >= 0.95
    rep["gate_quantized_pass"] = bool(rep["top1_agreement"] >= 0.95 and rep["cos_logprob_mean"] >= 0.99 and nolp_ok)
    rep["exact_match_top1_all"] = bool(rep["top1_agreement"] == 1.0 and rep["top1_agreement_nolp"] in (None, 1.0))
    tie_ok = rep["top1_tie_aware"] >= 0.95 and (rep["top1_tie_aware_nolp"] is None
                                                 or rep["top1_tie_aware_nolp"] >= 0.95)
    if not (tie_ok and rep["cos_logprob_mean"] >= 0.99) or rep["mean_abs_dlogprob"] > 0.15:
        rep["gate_v2"] = "FAIL"
    elif rep["mean_abs_dlogprob"] <= 0.10:
        rep["gate_v2"] = "PASS"
    else:
        rep["gate_v2"] = "JUDGE"
    return rep
