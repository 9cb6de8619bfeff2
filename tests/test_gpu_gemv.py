"""Decode GEMV on the GPU through the C-ABI, against the oracle.

Every call here goes through libq35cuda's reference-facing entry points
(q35_mm_fp8 / _batch / _multi4 / q35_mm_bf16) with host buffers, exactly as
the engine calls them, unless a test says it uses the device API.
"""
from __future__ import annotations

import numpy as np
import pytest

import mm_fixtures as M
import q35cu
from parity import GEMV_RTOL, gemv_report

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _fresh_cache(gpu):
    # numpy may hand a new array the address of a freed one; start every test
    # with an empty residency cache (the fingerprint check is tested below)
    gpu.q35cu_release_all()
    yield
    gpu.q35cu_release_all()


def _synth(orc, seed, rows, cols):
    return orc.synth_fp8(seed, rows, cols)


def _check(orc, W, sc, X, Y, Yref, what):
    Y64, A = orc.mm_fp8_f64(W, sc, X)
    rep = gemv_report(Y, Yref, Y64, A)
    assert rep["ok"], (what, rep)
    return rep


@pytest.mark.parametrize("name", [c[0] for c in M.CASES])
def test_known_answer_fixtures(gpu, golden, orc, name):
    """qwen35-c/tests/test_mm.c: every manifest case, tol 5e-4, plus the 1e-5 rule vs the oracle."""
    W, sc, x, yref = golden[name]
    if sc is None:
        y = q35cu.mm_bf16(W, x)
        yo = orc.mm_bf16(W, x)
        assert np.all(np.abs(y - yref) <= M.TOL + M.TOL * np.abs(yref))
        y64 = W.astype(np.uint32) << 16
        A = np.abs(y64.view(np.float32).astype(np.float64) * x).sum(1)
        assert gemv_report(y, yo, yref, A)["ok"]
        return
    y = q35cu.mm_fp8(W, sc, x)
    assert np.all(np.abs(y - yref) <= M.TOL + M.TOL * np.abs(yref)), name
    _check(orc, W, sc, x, y, orc.mm_fp8(W, sc, x), name)


def test_config0_full_size(gpu, orc, ref):
    """C0: N=17408, K=5120, M=1 against the compiled reference q35_mm_fp8."""
    W, sc = _synth(orc, 1001, 17408, 5120)
    x = orc.synth_act(2001, (5120,))
    y = q35cu.mm_fp8(W, sc, x)
    rep = _check(orc, W, sc, x, y, ref.mm_fp8(W, sc, x), "C0")
    # the GPU is no further from the exact product than the reference itself (+1 ulp of sum|.|)
    assert rep["gpu_vs_f64_max_ulps_of_abs"] <= rep["ref_vs_f64_max_ulps_of_abs"] + 1.0


@pytest.mark.parametrize("m", [1, 4, 16, 64])
@pytest.mark.parametrize("shape", [(17408, 5120), (5120, 17408)])
def test_config1_batch_sweep(gpu, orc, ref, shape, m):
    """C1: gate/up [17408x5120] and down [5120x17408] at M in {1,4,16,64} (q35_mm_fp8_batch)."""
    rows, cols = shape
    W, sc = _synth(orc, 3000 + rows, rows, cols)
    X = orc.synth_act(4000 + m, (m, cols))
    Y = q35cu.mm_fp8_batch(W, sc, X)
    _check(orc, W, sc, X, Y, ref.mm_fp8_batch(W, sc, X), f"C1 {shape} m={m}")


@pytest.mark.parametrize("n", [16, 17, 32, 33, 48, 49, 64, 65, 100, 127])
def test_exact_tensor_core_tile_widths(gpu, orc, ref, n):
    """q35_mm_fp8_batch with 16..127 tokens runs the tensor cores on exact
    activations: up to 48 tokens each token as five e4m3 terms (one token
    tile of 16, 32 or 48), above that (or with Q35CU_GEMV_TC_F16) as f16
    hi/lo rows (32-, 64-, 128- or 192-row tiles).  Within the GEMV bound,
    on ragged tile fills too."""
    W, sc = _synth(orc, 70 + n, 1000, 5120)
    X = orc.synth_act(90 + n, (n, 5120))
    Yr = ref.mm_fp8_batch(W, sc, X)
    _check(orc, W, sc, X, q35cu.mm_fp8_batch(W, sc, X), Yr, f"e4m3 terms n={n}")


def _e4m3_values():
    """float value of every e4m3 code (0x7F / 0xFF: NaN)"""
    v = np.empty(256, np.float64)
    for c in range(256):
        sgn = -1.0 if c & 0x80 else 1.0
        e, mt = (c >> 3) & 0xF, c & 7
        v[c] = sgn * (mt / 8.0 * 2.0 ** -6 if e == 0 else (1 + mt / 8.0) * 2.0 ** (e - 7))
    v[0x7F] = v[0xFF] = np.nan
    return v


def test_e4m3_decode_terms_carry_fp32(gpu, orc):
    """The multi-token decode preparation (left in the caller's workspace):
    per token 2^e and five e4m3 rows t0..t4 with x = sum_j t_j 16^-j 2^e to
    within 2^-32 of the row's largest magnitude (fp32 rows spanning 2^40,
    tiny elements beside large ones), the largest in [2^7, 2^8) after
    scaling."""
    import torch

    m, k = 20, 512
    rng = np.random.default_rng(11)
    X = orc.synth_act(111, (m, k)) * np.exp2(rng.integers(-20, 20, (m, 1))).astype(np.float32)
    X[3] = 0.0
    X[4, ::5] *= np.float32(2.0 ** -25)
    w = q35cu.Weight.synth_fp8(112, 256, k)
    try:
        Xd = torch.from_numpy(X).cuda()
        Y = torch.empty((m, 256), device="cuda")
        need = int(q35cu.load().q35cu_gemv_fp8_tc_workspace_bytes(m, k))
        work = torch.zeros(need, dtype=torch.uint8, device="cuda")
        q35cu.gemv_tc(w, Xd, Y, work)
        torch.cuda.synchronize()
        q35cu.check_device_status()
        raw = work.cpu().numpy()
        terms = raw[:5 * m * k].reshape(m, 5, k)
        ts = raw[len(raw) - 4 * m:].view(np.float32).astype(np.float64)
        tab = _e4m3_values()
        rec = sum(tab[terms[:, j]] * 16.0 ** -j for j in range(5)) * ts[:, None]
        x64 = X.astype(np.float64)
        mx = np.abs(x64).max(axis=1, keepdims=True)
        assert np.isfinite(rec).all()
        assert (np.abs(rec - x64) <= mx * 2.0 ** -32).all()
        live = mx[:, 0] > 0
        assert ((mx[live, 0] / ts[live] >= 128) & (mx[live, 0] / ts[live] < 256)).all()
        assert (rec[3] == 0).all()
    finally:
        w.free()


@pytest.mark.parametrize("rows,cols,n", [(17408, 5120, 16), (5120, 17408, 32), (5120, 6144, 48)])
def test_exact_decode_kernels_agree(gpu, orc, ref, monkeypatch, rows, cols, n):
    """The e4m3-term kernel and the f16 hi/lo kernel (Q35CU_GEMV_TC_F16) on
    the same multi-token decode: both within the GEMV bound of the
    reference, runs repeat bit for bit, and their difference is of the order
    of fp32 accumulation (max 2^-16 of sum |w s x|)."""
    W, sc = _synth(orc, 2500 + rows + n, rows, cols)
    X = orc.synth_act(2600 + n, (n, cols))
    Yr = ref.mm_fp8_batch(W, sc, X)
    Ye = q35cu.mm_fp8_batch(W, sc, X)
    assert np.array_equal(Ye.view(np.uint32), q35cu.mm_fp8_batch(W, sc, X).view(np.uint32))
    _check(orc, W, sc, X, Ye, Yr, f"e4m3 terms {rows}x{cols} n={n}")
    monkeypatch.setenv("Q35CU_GEMV_TC_F16", "1")
    Yf = q35cu.mm_fp8_batch(W, sc, X)
    _check(orc, W, sc, X, Yf, Yr, f"hi/lo {rows}x{cols} n={n}")
    _, abs_sum = orc.mm_fp8_f64(W, sc, X)
    assert (np.abs(Ye.astype(np.float64) - Yf) <= 2.0 ** -16 * abs_sum).all()


def test_batch_equals_single_bitwise(gpu, orc):
    """qwen35-c/tests/test_batch_mm.c on the GPU: batch == n x single == multi4."""
    rows, cols, n = 10240, 5120, 5
    W, sc = _synth(orc, 77, rows, cols)
    X = orc.synth_act(78, (n, cols))
    Yb = q35cu.mm_fp8_batch(W, sc, X)
    for t in range(n):
        assert np.array_equal(Yb[t].view(np.uint32), q35cu.mm_fp8(W, sc, X[t]).view(np.uint32))
    m4 = q35cu.mm_fp8_multi4([W], [sc], X[0])
    assert np.array_equal(m4[0].view(np.uint32), Yb[0].view(np.uint32))


def test_batch_mm_reference_inputs(gpu, orc):
    """The exact inputs of test_batch_mm (W[i]=i*7+13, zero scales): all outputs 0, batch == single."""
    rows, cols, n = 10240, 5120, 5
    W = ((np.arange(rows * cols, dtype=np.uint64) * 7 + 13) & 0xFF).astype(np.uint8).reshape(rows, cols)
    sc = np.zeros((80, 40), np.uint16)
    X = (((np.arange(n * cols) % 200) - 100) * 0.001).astype(np.float32).reshape(n, cols)
    Yb = q35cu.mm_fp8_batch(W, sc, X)
    Yo = orc.mm_fp8_batch(W, sc, X)
    # NaN codes (0x7F/0xFF) times a zero scale are NaN on both sides
    assert np.array_equal(np.isnan(Yb), np.isnan(Yo))
    for t in range(n):
        ys = q35cu.mm_fp8(W, sc, X[t])
        assert np.array_equal(Yb[t].view(np.uint32), ys.view(np.uint32))


def test_multi4_deltanet_shapes(gpu, orc, ref):
    """q35_mm_fp8_multi4 as q35_deltanet.c:329 calls it: qkv 10240, z 6144, a 48, b 48 (K=5120)."""
    shapes = [10240, 6144, 48, 48]
    Ws, Ss = zip(*[_synth(orc, 500 + i, r, 5120) for i, r in enumerate(shapes)])
    x = orc.synth_act(600, (5120,))
    ys = q35cu.mm_fp8_multi4(list(Ws), list(Ss), x)
    rs = ref.mm_fp8_multi4(list(Ws), list(Ss), x)
    for W, sc, y, r in zip(Ws, Ss, ys, rs):
        _check(orc, W, sc, x, y, r, f"multi4 {W.shape}")
        assert np.array_equal(y.view(np.uint32), q35cu.mm_fp8(W, sc, x).view(np.uint32))


def test_multi4_skips_zero_rows(gpu, orc):
    W, sc = _synth(orc, 11, 256, 512)
    x = orc.synth_act(12, (512,))
    ys = q35cu.mm_fp8_multi4([None, W, None, W[:100]], [None, sc, None, sc[:1]], x)
    assert ys[0] is None and ys[2] is None
    assert np.array_equal(ys[1].view(np.uint32), q35cu.mm_fp8(W, sc, x).view(np.uint32))
    assert np.array_equal(ys[3], ys[1][:100])


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 5), (7, 33), (129, 129), (130, 4096), (5, 5120), (1023, 1040)])
def test_odd_shapes(gpu, orc, ref, rows, cols):
    """Ragged rows (not a multiple of 4 or 128) and ragged K (not a multiple of 16)."""
    g = np.random.default_rng(rows * 31 + cols)
    W = g.integers(0, 256, size=(rows, cols), dtype=np.uint8)
    W[(W & 0x7F) == 0x7F] = 0x41
    import oracle

    sc = oracle.bf16_bits((g.random(((rows + 127) // 128, (cols + 127) // 128)) + 0.5).astype(np.float32))
    X = g.standard_normal((3, cols)).astype(np.float32)
    _check(orc, W, sc, X[0], q35cu.mm_fp8(W, sc, X[0]), ref.mm_fp8(W, sc, X[0]), "single")
    _check(orc, W, sc, X, q35cu.mm_fp8_batch(W, sc, X), ref.mm_fp8_batch(W, sc, X), "batch")


@pytest.mark.parametrize("rows,cols", [(700, 1040), (4800, 6160), (700, 12304), (400, 18448)])
def test_cuda_core_geometries(gpu, orc, ref, rows, cols):
    """The CUDA-core streaming kernel (cols % 128 != 0) at every register-pass
    count P = 1..4 (1040, 6160, 12304, 18448 fp8 columns), one to four tokens
    (1, 2 or 4 tokens per CTA column block); 4800 rows fill whole 8-row
    stages at P = 2."""
    g = np.random.default_rng(rows + 7 * cols)
    import oracle

    W = g.integers(0, 256, size=(rows, cols), dtype=np.uint8)
    W[(W & 0x7F) == 0x7F] = 0x41
    sc = oracle.bf16_bits((g.random(((rows + 127) // 128, (cols + 127) // 128)) + 0.5).astype(np.float32))
    X = g.standard_normal((4, cols)).astype(np.float32)
    _check(orc, W, sc, X[0], q35cu.mm_fp8(W, sc, X[0]), ref.mm_fp8(W, sc, X[0]), "single")
    for n in (2, 3, 4):
        _check(orc, W, sc, X[:n], q35cu.mm_fp8_batch(W, sc, X[:n]), ref.mm_fp8_batch(W, sc, X[:n]), f"batch {n}")


def test_cuda_core_forced_on_aligned_cols(gpu, orc, ref, monkeypatch):
    """Q35CU_GEMV_SIMT routes a cols % 128 == 0 weight to the CUDA-core kernel
    (6272 columns: two register passes); it agrees with the tensor-core GEMV
    within the GEMV bound."""
    W, sc = _synth(orc, 61, 4800, 6272)
    x = orc.synth_act(62, (6272,))
    y_tc = q35cu.mm_fp8(W, sc, x)
    gpu.q35cu_release_all()
    monkeypatch.setenv("Q35CU_GEMV_SIMT", "1")
    y_cc = q35cu.mm_fp8(W, sc, x)
    yr = ref.mm_fp8(W, sc, x)
    _check(orc, W, sc, x, y_cc, yr, "cuda-core")
    _check(orc, W, sc, x, y_tc, yr, "tensor-core")


@pytest.mark.parametrize("cols", [1024, 8192, 12288])
def test_bf16_geometries(gpu, orc, ref, cols):
    """q35_mm_bf16 at register-pass counts P = 1, 3, 4 (the lm_head's 5120
    columns, P = 2, is test_bf16_lm_head_shape)."""
    g = np.random.default_rng(cols)
    import oracle

    W16 = oracle.bf16_bits(g.standard_normal((5000, cols)).astype(np.float32) * 0.02)
    x = g.standard_normal(cols).astype(np.float32)
    y = q35cu.mm_bf16(W16, x)
    wf = (W16.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    assert gemv_report(y, ref.mm_bf16(W16, x), wf @ x.astype(np.float64), np.abs(wf * x).sum(1))["ok"]


def test_zero_sizes(gpu):
    W = np.zeros((4, 8), np.uint8)
    sc = np.zeros((1, 1), np.uint16)
    y = np.full(4, 7.0, np.float32)
    q35cu.load().q35_mm_fp8(q35cu._p(W, q35cu._u8p), q35cu._p(sc, q35cu._u16p), 0, 8,
                            q35cu._p(np.zeros(8, np.float32), q35cu._f32p), q35cu._p(y, q35cu._f32p))
    assert np.all(y == 7.0)  # rows == 0: nothing written
    q35cu.load().q35_mm_fp8(q35cu._p(W, q35cu._u8p), q35cu._p(sc, q35cu._u16p), 4, 0,
                            q35cu._p(np.zeros(8, np.float32), q35cu._f32p), q35cu._p(y, q35cu._f32p))
    assert np.all(y == 0.0)  # cols == 0: empty sums


def test_nan_codes_propagate(gpu, orc):
    W, sc = _synth(orc, 21, 256, 256)
    W[5, 17] = 0x7F
    W[200, 3] = 0xFF
    x = orc.synth_act(22, (256,))
    y = q35cu.mm_fp8(W, sc, x)
    assert np.isnan(y[5]) and np.isnan(y[200])
    assert np.isfinite(np.delete(y, [5, 200])).all()


def test_repeatable_and_cached(gpu, orc):
    W, sc = _synth(orc, 31, 4096, 5120)
    x = orc.synth_act(32, (5120,))
    a = q35cu.mm_fp8(W, sc, x)
    before = q35cu.load().q35cu_cache_bytes()
    b = q35cu.mm_fp8(W, sc, x)
    assert q35cu.load().q35cu_cache_bytes() == before  # second call hit the cache
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert q35cu.load().q35cu_forget(W.ctypes.data) == 1


def test_bf16_lm_head_shape(gpu, orc, ref):
    """q35_mm_bf16 (the lm_head matvec), a 16384-row slice of 248320x5120."""
    g = np.random.default_rng(41)
    import oracle

    W16 = oracle.bf16_bits(g.standard_normal((16384, 5120)).astype(np.float32) * 0.02)
    x = g.standard_normal(5120).astype(np.float32)
    y = q35cu.mm_bf16(W16, x)
    yr = ref.mm_bf16(W16, x)
    wf = (W16.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    y64 = wf @ x.astype(np.float64)
    A = np.abs(wf * x).sum(1)
    assert gemv_report(y, yr, y64, A)["ok"]


def test_device_api_and_synth(gpu, orc):
    """Device-resident synthetic weight == the host generator; device-pointer gemv == host ABI."""
    import torch

    w = q35cu.Weight.synth_fp8(123, 1024, 5120)
    try:
        Wd, scd = w.download_fp8()
        Wh, sch = orc.synth_fp8(123, 1024, 5120)
        assert np.array_equal(scd, sch)
        assert (Wd != Wh).mean() < 1e-4  # libm vs CUDA logf/cosf may move a rare element by one code
        X = torch.from_numpy(orc.synth_act(124, (4, 5120))).cuda()
        Y = torch.empty((4, 1024), device="cuda")
        q35cu.gemv(w, X, Y)
        torch.cuda.synchronize()
        Yh = q35cu.mm_fp8_batch(Wd, scd, X.cpu().numpy())
        assert np.array_equal(Y.cpu().numpy().view(np.uint32), Yh.view(np.uint32))
    finally:
        w.free()


def test_budget_reports_nomem_and_nan(gpu, orc):
    lib = q35cu.load()
    lib.q35cu_release_all()
    W, sc = _synth(orc, 51, 2048, 2048)
    x = orc.synth_act(52, (2048,))
    lib.q35cu_set_memory_budget(1 << 20)  # smaller than the weight
    try:
        lib.q35cu_clear_error()
        y = q35cu.mm_fp8(W, sc, x)
        code, msg = q35cu.last_error()
        assert code == q35cu.ERR_NOMEM and "budget" in msg
        assert np.isnan(y).all()
    finally:
        lib.q35cu_set_memory_budget(0)
    y = q35cu.mm_fp8(W, sc, x)
    assert np.isfinite(y).all()


def test_bad_arguments_are_recorded(gpu):
    lib = q35cu.load()
    lib.q35cu_clear_error()
    y = np.zeros(8, np.float32)
    lib.q35_mm_fp8(None, None, 8, 16, None, q35cu._p(y, q35cu._f32p))
    assert q35cu.last_error()[0] == q35cu.ERR_ARG
    assert np.isnan(y).all()


def test_cache_detects_reused_address(gpu, orc):
    """Same host address and shape, new contents: the fingerprint forces a re-upload."""
    W, sc = _synth(orc, 61, 512, 1024)
    x = orc.synth_act(62, (1024,))
    a = q35cu.mm_fp8(W, sc, x)
    W2, sc2 = _synth(orc, 63, 512, 1024)
    W[...] = W2          # same buffers, other tensor
    sc[...] = sc2
    b = q35cu.mm_fp8(W, sc, x)
    assert np.array_equal(b.view(np.uint32), q35cu.mm_fp8(W2, sc2, x).view(np.uint32))
    assert not np.array_equal(a, b)


@pytest.mark.parametrize("kernel", ["e4m3", "f16"])
@pytest.mark.parametrize("mode", ["split", "streamk", "whole"])
@pytest.mark.parametrize("rows,cols,n", [(5120, 17408, 16), (5120, 6144, 40), (1024, 5120, 32)])
def test_tensor_core_decode_work_splits(gpu, orc, ref, monkeypatch, kernel, mode, rows, cols, n):
    """Each way of dividing a few-tile decode launch among the CTAs --
    split-K (each tile's blocks cut into equal ranges, one per CTA),
    stream-K (equal unit ranges) and whole tiles -- with either kernel:
    within the GEMV bound and repeating bit for bit."""
    monkeypatch.setenv("Q35CU_GEMM_SPLIT", mode)
    if kernel == "f16":
        monkeypatch.setenv("Q35CU_GEMV_TC_F16", "1")
    W, sc = _synth(orc, 2700 + rows + n, rows, cols)
    X = orc.synth_act(2800 + n, (n, cols))
    Y1 = q35cu.mm_fp8_batch(W, sc, X)
    Y2 = q35cu.mm_fp8_batch(W, sc, X)
    assert np.array_equal(Y1.view(np.uint32), Y2.view(np.uint32))
    _check(orc, W, sc, X, Y1, ref.mm_fp8_batch(W, sc, X), f"{kernel} {mode} {rows}x{cols} n={n}")


@pytest.mark.parametrize("rows,cols,n", [(5120, 17408, 16), (5120, 6144, 33), (5120, 6144, 64), (1024, 5120, 40)])
def test_stream_k_tensor_core_decode(gpu, orc, ref, monkeypatch, rows, cols, n):
    """Multi-token decode on the tensor cores with few row tiles walks equal
    ranges of (tile, 128-column block) units per CTA (stream-K); a tile cut
    by CTA boundaries is finished by adding its segments' accumulators in a
    fixed order.  Runs repeat bit for bit, and both this walk and the
    whole-tile walk (Q35CU_GEMM_NO_STREAMK) meet the GEMV bound."""
    W, sc = _synth(orc, 2100 + rows + n, rows, cols)
    X = orc.synth_act(2200 + n, (n, cols))
    Yr = ref.mm_fp8_batch(W, sc, X)
    Y1 = q35cu.mm_fp8_batch(W, sc, X)
    Y2 = q35cu.mm_fp8_batch(W, sc, X)
    assert np.array_equal(Y1.view(np.uint32), Y2.view(np.uint32))
    _check(orc, W, sc, X, Y1, Yr, f"stream-K {rows}x{cols} n={n}")
    monkeypatch.setenv("Q35CU_GEMM_NO_STREAMK", "1")
    _check(orc, W, sc, X, q35cu.mm_fp8_batch(W, sc, X), Yr, f"whole tiles {rows}x{cols} n={n}")


@pytest.mark.parametrize("rows,cols", [(5120, 17408), (5120, 6144), (1040, 5120)])
def test_gemv_column_split_widths(gpu, orc, ref, monkeypatch, rows, cols):
    """The decode GEMV's column split over a cluster of 1, 2 or 4 CTAs (each
    CTA a contiguous range of the 256-column splits, the partials added in
    column order across the cluster): bit-identical to the unsplit kernel at
    1..8 tokens, including when fewer clusters of 4 fit the device than the
    grid would hold, and within the GEMV bound of the reference."""
    W, sc = _synth(orc, 3100 + rows, rows, cols)
    for n in (1, 2, 4, 8):
        X = orc.synth_act(3200 + n, (n, cols))
        monkeypatch.setenv("Q35CU_GEMV_KSPLIT", "1")
        Y1 = q35cu.mm_fp8_batch(W, sc, X)
        for cs in ("2", "4"):
            monkeypatch.setenv("Q35CU_GEMV_KSPLIT", cs)
            Ys = q35cu.mm_fp8_batch(W, sc, X)
            assert np.array_equal(Ys.view(np.uint32), Y1.view(np.uint32)), (rows, cols, n, cs)
        if n in (1, 4):
            _check(orc, W, sc, X, Y1, ref.mm_fp8_batch(W, sc, X), f"column split {rows}x{cols} n={n}")
