"""Comparison of transformer logits against the libtorch-CPU fixture
(tests/golden/transformer_b64_fixture.npz, made by
tests/golden/gen_transformer_fixture.py). Test helper only.

Every measure is an error normalised by the largest |logit| of the
fixture's sequences (max_ref), the form of the logits tolerance:
  rows     max |logit - fixture| over the stored full rows
  row_max  max over positions of |max logit - fixture's|
  row_lse  max over positions of |log-sum-exp - fixture's|
  proj     relative L2 error of the 8 signed projections of every position
           (||delta||_2 / ||fixture||_2, which is not normalised by max_ref)
and argmax: wherever the fixture's margin between the top two logits is
above 2 * tol * max_ref, the argmax must agree (a smaller margin can flip
within the tolerance).
"""
from __future__ import annotations

import importlib.util
import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
FIXTURE = GOLDEN / "transformer_b64_fixture.npz"

_spec = importlib.util.spec_from_file_location("gen_transformer_fixture", GOLDEN / "gen_transformer_fixture.py")
gen = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(gen)


def load() -> dict:
    z = np.load(FIXTURE)
    out = {k: z[k] for k in z.files}
    out["meta"] = json.loads(str(out["meta"]))
    out["weights_sha256"] = str(out["weights_sha256"])
    return out


def errors(fx: dict, logits: np.ndarray) -> dict:
    """logits f32 [len(seqs), S, V] for the fixture's sequences, in order."""
    seqs = fx["meta"]["seqs"]
    assert logits.shape[0] == len(seqs)
    dg = gen.digests(logits, gen.projection_signs(logits.shape[-1], fx["proj"].shape[-1],
                                                  fx["meta"]["projection_seed"]))
    max_ref = float(np.abs(fx["rows"]).max())
    max_ref = max(max_ref, float(np.abs(fx["row_max"]).max()))
    got_rows = np.stack([logits[seqs.index(b), p] for b, p in fx["rows_at"].tolist()]).astype(np.float64)
    e = {
        "max_ref": max_ref,
        "rows": float(np.abs(got_rows - fx["rows"]).max() / max_ref),
        "row_max": float(np.abs(dg["row_max"].astype(np.float64) - fx["row_max"]).max() / max_ref),
        "row_lse": float(np.abs(dg["row_lse"].astype(np.float64) - fx["row_lse"]).max() / max_ref),
        "proj": float(np.linalg.norm(dg["proj"].astype(np.float64) - fx["proj"]) / np.linalg.norm(fx["proj"])),
    }
    margin = fx["row_max"].astype(np.float64) - fx["row_top2"]
    e["argmax_agree"] = float((dg["row_argmax"] == fx["row_argmax"]).mean())
    e["_argmax"] = dg["row_argmax"]
    e["_margin"] = margin
    return e


def check(fx: dict, logits: np.ndarray, tol: float) -> dict:
    e = errors(fx, logits)
    for k in ("rows", "row_max", "row_lse", "proj"):
        assert e[k] <= tol, (k, e[k], tol)
    sure = e["_margin"] > 2.0 * tol * e["max_ref"]
    assert np.array_equal(e["_argmax"][sure], fx["row_argmax"][sure]), "argmax differs where the margin is large"
    return {k: v for k, v in e.items() if not k.startswith("_")}
