"""Prefill GEMM (tcgen05 tensor cores) on the GPU against the oracle.

Contract (prefill): activations rounded to bf16, relative L2 error of Y
against the reference's own matmul on the same bf16-valued X <= 5e-3.
Two kernels serve it.  The default multiplies e4m3 weights by each
activation carried as two e4m3 terms (block-scaled MMAs); the other
(Q35CU_GEMM_F16) converts the weights to f16 and carries the activations
exactly in f16.  Both promote each 128-column block's fp32 partial with its
scale, so the error is fp32 accumulation order plus, for the terms, at most
2^-21 of a row's largest magnitude on its smallest elements; the tests
also hold both to a tight sanity bound (1e-5) to catch layout or indexing
mistakes that a loose bound would hide.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import q35cu
from parity import GEMM_REL_L2, rel_l2

pytestmark = pytest.mark.gpu
TIGHT = 1e-5


@pytest.fixture(autouse=True)
def _fresh_cache(gpu):
    gpu.q35cu_release_all()
    yield
    gpu.q35cu_release_all()


def _bf16_x(orc, seed, m, k):
    return oracle.bf16_round(orc.synth_act(seed, (m, k)))


@pytest.mark.parametrize("rows,cols,n", [
    (17408, 5120, 128),   # gate / up
    (5120, 17408, 128),   # down
    (5120, 6144, 256),    # out / o
    (1024, 5120, 200),    # k / v, ragged token count
    (300, 512, 130),      # ragged rows (partial 128-row tile), ragged tokens
    (256, 144, 128),      # K not a multiple of 128 (partial last block)
])
def test_batch_abi_takes_tensor_cores(gpu, orc, ref, rows, cols, n):
    """q35_mm_fp8_batch with n >= 128 tokens (host buffers) -> the tcgen05 path."""
    W, sc = orc.synth_fp8(7000 + rows + cols, rows, cols)
    X = _bf16_x(orc, 7100 + n, n, cols)
    before = gpu.q35cu_launch_count()
    Y = q35cu.mm_fp8_batch(W, sc, X)
    assert gpu.q35cu_launch_count() > before
    Yr = ref.mm_fp8_batch(W, sc, X)
    err = rel_l2(Y, Yr)
    assert np.isfinite(Y).all()
    assert err <= GEMM_REL_L2, err
    assert err <= TIGHT, err


@pytest.mark.parametrize("name,rows,cols", [
    ("qkv", 10240, 5120), ("z", 6144, 5120), ("out", 5120, 6144), ("q", 12288, 5120),
    ("k", 1024, 5120), ("v", 1024, 5120), ("o", 5120, 6144), ("gate", 17408, 5120), ("down", 5120, 17408),
])
def test_config2_prefill_shapes(gpu, orc, name, rows, cols):
    """Configuration 2 (M=2048) through the device API, checked against fp64 on 48 sampled tokens."""
    import torch

    m = 2048
    w = q35cu.Weight.synth_fp8(8000 + rows * 3 + cols, rows, cols)
    try:
        Wh, sch = w.download_fp8()
        X = _bf16_x(orc, 8100 + rows, m, cols)
        Xb = torch.from_numpy(X).to(torch.bfloat16).cuda()
        assert torch.equal(Xb.float().cpu(), torch.from_numpy(X))  # X already bf16-valued
        Y = torch.empty((m, rows), device="cuda")
        q35cu.gemm(w, Xb.view(torch.int16), Y)
        torch.cuda.synchronize()
        q35cu.check_device_status()
        Yh = Y.cpu().numpy()
        pick = np.random.default_rng(rows).choice(m, 48, replace=False)
        Y64, _ = orc.mm_fp8_f64(Wh, sch, np.ascontiguousarray(X[pick]))
        err = rel_l2(Yh[pick], Y64)
        assert np.isfinite(Yh).all()
        assert err <= GEMM_REL_L2, (name, err)
        assert err <= TIGHT, (name, err)
    finally:
        w.free()


def test_gemm_deterministic(gpu, orc):
    import torch

    w = q35cu.Weight.synth_fp8(91, 2048, 1024)
    try:
        X = torch.from_numpy(_bf16_x(orc, 92, 384, 1024)).to(torch.bfloat16).cuda()
        Y1 = torch.empty((384, 2048), device="cuda")
        Y2 = torch.empty_like(Y1)
        q35cu.gemm(w, X.view(torch.int16), Y1)
        q35cu.gemm(w, X.view(torch.int16), Y2)
        torch.cuda.synchronize()
        q35cu.check_device_status()
        assert torch.equal(Y1, Y2)
    finally:
        w.free()


def _e4m3_table():
    """float value of every e4m3 code (0x7F / 0xFF: NaN)"""
    v = np.empty(256, np.float64)
    for c in range(256):
        sgn = -1.0 if c & 0x80 else 1.0
        e, mt = (c >> 3) & 0xF, c & 7
        v[c] = sgn * (mt / 8.0 * 2.0 ** -6 if e == 0 else (1 + mt / 8.0) * 2.0 ** (e - 7))
    v[0x7F] = v[0xFF] = np.nan
    return v


def test_e4m3_activation_terms_carry_bf16(gpu, orc):
    """The fp8-operand GEMM's prepared activations (left in the caller's
    workspace): per token a power of two 2^e and two e4m3 rows t0, t1 (two
    planes [m, K]) with
    x = (t0 + t1 / 16) 2^e exactly for every element down to 2^-13 of the
    row's largest, and within 2^-21 of it below; the largest lies in
    [2^7, 2^8) after scaling.  Rows span magnitudes over 2^40."""
    import torch

    m, k = 130, 512
    rng = np.random.default_rng(7)
    X = orc.synth_act(77, (m, k)) * np.exp2(rng.integers(-20, 20, (m, 1))).astype(np.float32)
    X[5] = 0.0
    X[6, ::3] *= 2.0 ** -30  # tiny elements beside normal ones
    X = oracle.bf16_round(X)
    w = q35cu.Weight.synth_fp8(78, 256, k)
    try:
        Xb = torch.from_numpy(X).to(torch.bfloat16).cuda()
        Y = torch.empty((m, 256), device="cuda")
        work = torch.zeros(q35cu.gemm_workspace_bytes(m, k), dtype=torch.uint8, device="cuda")
        q35cu.gemm(w, Xb.view(torch.int16), Y, work)
        torch.cuda.synchronize()
        q35cu.check_device_status()
        raw = work.cpu().numpy()
        terms = raw[:2 * m * k].reshape(2, m, k)  # plane 0: t0 [m, k], plane 1: t1 [m, k]
        ts = raw[len(raw) - 4 * m:].view(np.float32).astype(np.float64)
        tab = _e4m3_table()
        rec = (tab[terms[0]] + tab[terms[1]] / 16.0) * ts[:, None]
        x64 = X.astype(np.float64)
        mx = np.abs(x64).max(axis=1, keepdims=True)
        assert np.isfinite(rec).all()
        err = np.abs(rec - x64)
        big = np.abs(x64) >= mx * 2.0 ** -13
        assert (err[big] == 0).all()
        assert (err <= mx * 2.0 ** -21).all()
        live = mx[:, 0] > 0
        assert ((mx[live, 0] / ts[live] >= 128) & (mx[live, 0] / ts[live] < 256)).all()
        assert (rec[5] == 0).all()
    finally:
        w.free()


@pytest.mark.parametrize("rows,cols,n", [(17408, 5120, 300), (5120, 17408, 256), (300, 512, 130), (256, 144, 128)])
def test_fp8_and_f16_kernels_agree(gpu, orc, monkeypatch, rows, cols, n):
    """The fp8-operand kernel (default) and the f16-operand one
    (Q35CU_GEMM_F16) both meet the tight bound against fp64 on the same
    bf16 activations."""
    import torch

    w = q35cu.Weight.synth_fp8(9000 + rows + cols, rows, cols)
    try:
        Wh, sch = w.download_fp8()
        X = _bf16_x(orc, 9100 + n, n, cols)
        Xb = torch.from_numpy(X).to(torch.bfloat16).cuda()
        outs = {}
        for kern in ("fp8", "f16"):
            if kern == "f16":
                monkeypatch.setenv("Q35CU_GEMM_F16", "1")
            Y = torch.full((n, rows), float("nan"), device="cuda")
            q35cu.gemm(w, Xb.view(torch.int16), Y)
            torch.cuda.synchronize()
            q35cu.check_device_status()
            outs[kern] = Y.cpu().numpy()
        pick = np.unique(np.concatenate([np.random.default_rng(rows).choice(n, 24, replace=False), [0, n - 1]]))
        Y64, _ = orc.mm_fp8_f64(Wh, sch, np.ascontiguousarray(X[pick]))
        for kern, Y in outs.items():
            assert np.isfinite(Y).all(), kern
            err = rel_l2(Y[pick], Y64)
            assert err <= TIGHT, (kern, err)
    finally:
        w.free()


@pytest.mark.parametrize("kernel", ["e4m3", "f16"])
def test_gemm_f32_input_equals_bf16_input(gpu, orc, monkeypatch, kernel):
    """q35cu_gemm_fp8_f32 rounds fp32 activations to bf16 while preparing
    them: the same bits as converting to bf16 first and calling
    q35cu_gemm_fp8, with either kernel."""
    import torch

    if kernel == "f16":
        monkeypatch.setenv("Q35CU_GEMM_F16", "1")
    w = q35cu.Weight.synth_fp8(97, 1024, 2048)
    try:
        X = torch.from_numpy(orc.synth_act(98, (300, 2048))).cuda()
        Y1 = torch.empty((300, 1024), device="cuda")
        Y2 = torch.empty_like(Y1)
        q35cu.gemm_f32(w, X, Y1)
        q35cu.gemm(w, X.to(torch.bfloat16).view(torch.int16), Y2)
        torch.cuda.synchronize()
        q35cu.check_device_status()
        assert torch.equal(Y1, Y2)
    finally:
        w.free()


@pytest.mark.parametrize("kernel", ["e4m3", "f16"])
@pytest.mark.parametrize("rows,m", [
    ((1024, 300, 1000, 128), 300),        # ragged last row blocks between segments
    ((2048, 256), 1),                     # one token: one token tile
    ((640,), 420),                        # one weight: the single-GEMM path
])
def test_gemm_multi_equals_single(gpu, orc, monkeypatch, kernel, rows, m):
    """q35cu_gemm_fp8_multi: weights sharing one input in one launch (their
    row blocks concatenated, a row block of each segment partial) give the
    bits of one q35cu_gemm_fp8 call per weight, on bf16 and fp32 inputs."""
    import torch

    if kernel == "f16":
        monkeypatch.setenv("Q35CU_GEMM_F16", "1")
    K = 1536
    ws = [q35cu.Weight.synth_fp8(700 + i, r, K) for i, r in enumerate(rows)]
    try:
        X = torch.from_numpy(orc.synth_act(720, (m, K))).cuda()
        Xb = X.to(torch.bfloat16).view(torch.int16)
        for x in (Xb, X):
            Ym = [torch.full((m, w.rows), 7.0, device="cuda") for w in ws]
            q35cu.gemm_multi(ws, x, Ym)
            for w, y in zip(ws, Ym):
                ys = torch.empty((m, w.rows), device="cuda")
                q35cu.gemm(w, Xb, ys)
                torch.cuda.synchronize()
                assert torch.equal(y, ys), (w.rows, x.dtype)
        q35cu.check_device_status()
    finally:
        for w in ws:
            w.free()


def test_gemm_multi_rejects_mixed_columns(gpu):
    """Weights of different cols cannot share one activation matrix."""
    import torch

    a = q35cu.Weight.synth_fp8(730, 256, 512)
    b = q35cu.Weight.synth_fp8(731, 256, 1024)
    try:
        X = torch.zeros((128, 512), dtype=torch.int16, device="cuda")
        Y = [torch.empty((128, 256), device="cuda") for _ in range(2)]
        with pytest.raises(q35cu.Q35Error):
            q35cu.gemm_multi([a, b], X, Y)
    finally:
        a.free()
        b.free()


def test_gemm_nonfinite_activation(gpu, orc, monkeypatch):
    """A token holding an infinity or a NaN gets non-finite outputs (the fp8
    kernel: NaN); every other token is unchanged."""
    W, sc = orc.synth_fp8(95, 256, 256)
    X = _bf16_x(orc, 96, 140, 256)
    base = q35cu.mm_fp8_batch(W, sc, X)
    X2 = X.copy()
    X2[3, 10] = np.inf
    X2[7, 0] = np.nan
    Y = q35cu.mm_fp8_batch(W, sc, X2)
    assert not np.isfinite(Y[3]).any() and not np.isfinite(Y[7]).any()
    keep = np.ones(140, bool)
    keep[[3, 7]] = False
    assert np.array_equal(Y[keep], base[keep])


def test_gemm_nan_code_propagates(gpu, orc, ref):
    W, sc = orc.synth_fp8(93, 256, 256)
    W[17, 40] = 0x7F
    X = _bf16_x(orc, 94, 128, 256)
    Y = q35cu.mm_fp8_batch(W, sc, X)
    assert np.isnan(Y[:, 17]).all()
    keep = np.ones(256, bool)
    keep[17] = False
    assert rel_l2(Y[:, keep], ref.mm_fp8_batch(W, sc, X)[:, keep]) <= TIGHT
