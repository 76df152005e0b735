"""The libtorch-CPU fixture of the benchmark transformer (made by
tests/golden/gen_transformer_fixture.py) pins the numpy oracle, on the CPU:
the fixture's tokens and weights are the benchmark's (seeds 5 and 4, same
sha256 as the host generator's buffer), and the numpy restatement, which
rounds to bf16 where the GPU path does, stays within the 2e-2 logits
tolerance of it (measured 3.8e-3). The host generator's own ln/cos series
are checked against libm on a million draws."""
from __future__ import annotations

import hashlib
import math

import numpy as np
import pytest

from fercuda_b200 import synth
from oracle import transformer_ref as ref
from tests import fixture_check

REQUIRED_TOL = 2e-2
TIGHT = 1e-2


@pytest.fixture(scope="module")
def fx():
    return fixture_check.load()


@pytest.fixture(scope="module")
def wbits():
    c = synth.TRANSFORMER
    total = ref.weight_offsets(c["layers"], c["d_model"], c["ffn"], c["vocab"])["total"]
    return synth.normal_bf16(c["weight_seed"], total, 0.0, 0.02)


def test_fixture_inputs_are_the_benchmarks(fx, wbits):
    c = synth.TRANSFORMER
    meta = fx["meta"]
    for k in ("layers", "d_model", "heads", "ffn", "vocab", "seq", "batch", "weight_seed", "token_seed"):
        assert meta[k] == c[k], k
    toks = fixture_check.gen.batch_tokens(c["batch"], c["seq"], c["vocab"], c["token_seed"])
    assert np.array_equal(toks[meta["seqs"]], fx["tokens"])
    assert hashlib.sha256(wbits.astype("<u2").tobytes()).hexdigest() == fx["weights_sha256"]
    assert meta["seqs"] == [0, 21, 42, 63]


def test_numpy_oracle_vs_libtorch_fixture(fx, wbits):
    c = synth.TRANSFORMER
    y = ref.forward(fx["tokens"], wbits, c["layers"], c["d_model"], c["heads"], c["ffn"], c["vocab"], c["eps"])
    e = fixture_check.check(fx, y, REQUIRED_TOL)
    for k in ("rows", "row_max", "row_lse", "proj"):
        assert e[k] <= TIGHT, (k, e)


def test_fixture_check_catches_a_planted_error(fx):
    """A logits array with one full row off by 3% of the largest logit fails."""
    S, V = fx["meta"]["seq"], fx["meta"]["vocab"]
    fake = np.zeros((len(fx["meta"]["seqs"]), S, V), np.float32)
    b, p = fx["rows_at"][0].tolist()
    fake[fx["meta"]["seqs"].index(b), p] = fx["rows"][0] + 0.03 * np.abs(fx["rows"]).max()
    e = fixture_check.errors(fx, fake)
    assert e["rows"] > REQUIRED_TOL


def test_generator_series_track_libm():
    """The portable ln and cos series agree with libm to a few float64 ulps,
    and the f32 normal draws equal the libm-based Box-Muller ones."""
    n = 1 << 20
    d = synth.splitmix64(4, 2 * n)
    k1 = (d[0::2] >> np.uint64(11)) + np.uint64(1)
    k2 = d[1::2] >> np.uint64(11)
    u1 = k1.astype(np.float64) * 2.0 ** -53
    u2 = k2.astype(np.float64) * 2.0 ** -53
    ln = synth.portable_ln(k1)
    assert np.abs(ln - np.log(u1)).max() <= 4e-16 * np.abs(np.log(u1)).max()
    cs = synth.portable_cos_turns(k2)
    assert np.abs(cs - np.cos(2.0 * math.pi * u2)).max() <= 1e-15
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * math.pi * u2)
    assert np.array_equal(synth.normal_f32(4, n), z.astype(np.float32))
    # the end points: u1 = 1 gives +0, every octant boundary is exact
    edge = np.array([1 << 53], np.uint64)
    assert synth.portable_ln(edge)[0] == 0.0
    oct_k = np.arange(8, dtype=np.uint64) << np.uint64(50)
    assert np.allclose(synth.portable_cos_turns(oct_k), np.cos(2 * math.pi * np.arange(8) / 8), atol=1e-15)
