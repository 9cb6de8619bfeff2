"""The oracle itself, pinned against the reference's fixtures (CPU only).

Pins, in order of strength:
  1. the regenerated fixture inputs are byte-identical to the reference's
     tests/fixtures/mm files (sha256 in tests/golden/ref_sha256.json), and the
     expected outputs match them (fp32-rounded digest);
  2. the oracle reproduces the FNV-1a anchors the reference's test_mm prints
     (qwen35-c/tests/test_mm.c:77-81) bit-for-bit;
  3. the oracle passes the reference's own criterion |y-yref| <= tol+tol|yref|
     with tol = 5e-4 on all 8 cases (qwen35-c/tests/test_mm.c:69);
  4. where the reference was compiled (oracle/_ref), oracle == reference
     bit-for-bit on the fixtures and on random shapes.
"""
from __future__ import annotations

import numpy as np
import pytest

import mm_fixtures as M


def test_fixture_pins(golden):
    # the fixture fixture verifies every pin; reaching here means they held
    assert set(golden) == {c[0] for c in M.CASES}


@pytest.mark.parametrize("name", [c[0] for c in M.CASES])
def test_oracle_known_answer(golden, orc, name):
    W, sc, x, yref = golden[name]
    y = orc.mm_fp8(W, sc, x) if sc is not None else orc.mm_bf16(W, x)
    assert np.all(np.abs(y - yref) <= M.TOL + M.TOL * np.abs(yref))


def test_oracle_fnv_anchors(golden, orc):
    anchors = M.pins()["fnv1a_reference_outputs"]
    for name, want in anchors.items():
        W, sc, x, _ = golden[name]
        assert f"{orc.fnv1a(orc.mm_fp8(W, sc, x)):016x}" == want, name


def test_oracle_equals_reference_on_fixtures(golden, orc, ref):
    for name, (W, sc, x, _) in golden.items():
        if sc is None:
            a, b = orc.mm_bf16(W, x), ref.mm_bf16(W, x)
        else:
            a, b = orc.mm_fp8(W, sc, x), ref.mm_fp8(W, sc, x)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), name


@pytest.mark.parametrize("rows,cols", [(1, 1), (7, 33), (130, 257), (256, 1000), (300, 5120)])
def test_oracle_equals_reference_random(orc, ref, rows, cols):
    g = np.random.default_rng(rows * 7919 + cols)
    W = g.integers(0, 256, size=(rows, cols), dtype=np.uint8)
    W[(W & 0x7F) == 0x7F] = 0x3C  # keep NaN codes out of the bit-identity check
    sc = (g.random(((rows + 127) // 128, (cols + 127) // 128)) * 0.5 + 0.5).astype(np.float32)
    import oracle

    sc16 = oracle.bf16_bits(sc)
    X = g.standard_normal((3, cols)).astype(np.float32)
    assert np.array_equal(orc.mm_fp8(W, sc16, X[0]).view(np.uint32), ref.mm_fp8(W, sc16, X[0]).view(np.uint32))
    Yo, Yr = orc.mm_fp8_batch(W, sc16, X), ref.mm_fp8_batch(W, sc16, X)
    assert np.array_equal(Yo.view(np.uint32), Yr.view(np.uint32))
    # batch == n x single (the reference's test_batch_mm contract)
    for t in range(3):
        assert np.array_equal(Yr[t].view(np.uint32), ref.mm_fp8(W, sc16, X[t]).view(np.uint32))
    m4 = ref.mm_fp8_multi4([W, None, W[: rows // 2 + 1]], [sc16, None, sc16[: (rows // 2 + 1 + 127) // 128]], X[0])
    assert np.array_equal(m4[0].view(np.uint32), Yr[0].view(np.uint32))


def test_batch_mm_reference_structure(orc, ref):
    """qwen35-c/tests/test_batch_mm.c: 10240x5120, n=5, zero scales, W[i]=i*7+13."""
    rows, cols, n = 10240, 5120, 5
    W = ((np.arange(rows * cols, dtype=np.uint64) * 7 + 13) & 0xFF).astype(np.uint8).reshape(rows, cols)
    sc = np.zeros(((rows // 128 + 1) * (cols // 128 + 1),), np.uint16)[: 80 * 40].reshape(80, 40)
    X = (((np.arange(n * cols) % 200) - 100) * 0.001).astype(np.float32).reshape(n, cols)
    Y = orc.mm_fp8_batch(W, sc, X)
    for t in range(n):
        assert np.array_equal(Y[t].view(np.uint32), orc.mm_fp8(W, sc, X[t]).view(np.uint32))


def test_e4m3_decode_matches_ml_dtypes(orc):
    import ml_dtypes

    lut = orc.lut()
    want = np.arange(256, dtype=np.uint8).view(ml_dtypes.float8_e4m3fn).astype(np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(lut), nan)
    assert np.array_equal(lut[~nan], want[~nan])
    assert set(np.flatnonzero(nan)) == {0x7F, 0xFF}


def test_e4m3_encode_rne_matches_ml_dtypes(orc):
    import ml_dtypes

    g = np.random.default_rng(3)
    v = np.concatenate([
        g.standard_normal(20000).astype(np.float32) * 50,
        g.standard_normal(5000).astype(np.float32) * 0.01,   # subnormal range
        np.float32([0.0, -0.0, 448.0, -448.0, 464.0, 1e-9, 0.0009765625, 0.00146484375]),
    ])
    # exact midpoints between neighbours must round to the even code
    lut = orc.lut()
    fin = np.sort(lut[np.isfinite(lut) & (lut >= 0)])
    mids = ((fin[1:].astype(np.float64) + fin[:-1]) / 2).astype(np.float32)
    v = np.concatenate([v, mids, -mids])
    v = np.clip(v, -448, 448)
    want = v.astype(ml_dtypes.float8_e4m3fn).view(np.uint8)
    got = np.array([orc.e4m3_rne(t) for t in v], np.uint8)
    # +-0 both decode to 0; compare values, then codes away from zero
    assert np.array_equal(lut[got], lut[want])


def test_synth_recipe(orc):
    """s = bf16(amax/448) per 128x128 block; W = e4m3_rne(W0 / s)."""
    import oracle

    W, sc = orc.synth_fp8(5, 300, 260)
    lut = orc.lut()
    s = (sc.astype(np.uint32) << 16).view(np.float32)
    w0 = np.array([[orc.L.orc_synth_normal(5, r * 260 + c) for c in range(260)] for r in range(0, 300, 37)],
                  np.float32) * np.float32(0.02)
    for i, r in enumerate(range(0, 300, 37)):
        for bj in range(3):
            blk = np.array([[orc.L.orc_synth_normal(5, rr * 260 + c) for c in range(bj * 128, min(260, bj * 128 + 128))]
                            for rr in range((r // 128) * 128, min(300, (r // 128) * 128 + 128))], np.float32)
            amax = np.abs(blk * np.float32(0.02)).max()
            assert s[r // 128, bj] == oracle.bf16_round(np.float32([amax / np.float32(448.0)]))[0]
        srow = np.repeat(s[r // 128], 128)[:260]
        deq = lut[W[r]] * srow
        # nearest e4m3: half a step, |v| * 2^-4 in the normal range, s * 2^-10 below it
        bound = np.maximum(np.abs(w0[i]) / 16, srow * 2.0 ** -10) * (1 + 1e-6)
        assert np.all(np.abs(deq - w0[i]) <= bound)


def test_synth_window_is_a_shard_of_the_whole(orc):
    Wf, sf = orc.synth_fp8(9, 512, 384)
    Ws, ss = orc.synth_fp8(9, 512, 384, row0=128, col0=256, nrows=200, ncols=128)
    assert np.array_equal(Ws, Wf[128:328, 256:384])
    assert np.array_equal(ss, sf[1:3, 2:3])
