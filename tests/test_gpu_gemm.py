"""Prefill GEMM (tcgen05 tensor cores) on the GPU against the oracle.

Contract (prefill): activations rounded to bf16, relative L2 error of Y
against the reference's own matmul on the same bf16-valued X <= 5e-3.
The kernel converts e4m3 -> bf16 exactly and promotes each 128-column
block's fp32 partial with its scale, so the error is fp32 accumulation
order only; the tests also hold it to a tight sanity bound (1e-5) to catch
layout or indexing mistakes that a loose bound would hide.
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


def test_gemm_nan_code_propagates(gpu, orc, ref):
    W, sc = orc.synth_fp8(93, 256, 256)
    W[17, 40] = 0x7F
    X = _bf16_x(orc, 94, 128, 256)
    Y = q35cu.mm_fp8_batch(W, sc, X)
    assert np.isnan(Y[:, 17]).all()
    keep = np.ones(256, bool)
    keep[17] = False
    assert rel_l2(Y[:, keep], ref.mm_fp8_batch(W, sc, X)[:, keep]) <= TIGHT
