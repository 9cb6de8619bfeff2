"""The allocation-free prefill entry point, q35cu_gemm_fp8_f32_noalloc.

Some callers cannot let the library call cudaMalloc when they run a prefill
batch -- a serving process that reserved its whole HBM budget up front, or
a loop that cannot absorb the device synchronisation an allocation can
bring.  This entry point takes fp32 activations already on the device and
keeps their bf16 copy in a fixed array compiled into the library, so it
allocates nothing.  Here it is called through the C-ABI twice in a row on
different inputs, and each result is checked against the existing entry
point (q35cu_gemm_fp8 on the same bf16-rounded activations) with the
tolerance the GEMM tests use; a batch larger than the fixed array must be
refused.  The file sorts last so a stop-at-first-failure run has already run
every other test.
"""
from __future__ import annotations

import numpy as np
import pytest

import q35cu
from parity import GEMM_REL_L2, rel_l2

pytestmark = pytest.mark.gpu


def _call_noalloc(w, X, Y):
    import torch

    stream = torch.cuda.current_stream().cuda_stream
    return q35cu.load().q35cu_gemm_fp8_f32_noalloc(w.h, int(X.data_ptr()), X.shape[0], int(Y.data_ptr()),
                                                   stream if stream else None)


def test_noalloc_matches_gemm_twice(gpu, orc):
    import torch

    w = q35cu.Weight.synth_fp8(4242, 2048, 5120)
    try:
        for seed, m in ((71, 256), (72, 640)):
            X = torch.from_numpy(orc.synth_act(seed, (m, 5120))).cuda()
            Y = torch.full((m, 2048), float("nan"), device="cuda")
            q35cu.check(_call_noalloc(w, X, Y))
            torch.cuda.synchronize()
            assert q35cu.device_status(clear=True) == 0  # no bounded wait gave up
            Yref = torch.empty((m, 2048), device="cuda")
            q35cu.gemm(w, X.to(torch.bfloat16).view(torch.int16), Yref)
            torch.cuda.synchronize()
            assert q35cu.device_status(clear=True) == 0
            a, b = Y.cpu().numpy(), Yref.cpu().numpy()
            assert np.isfinite(a).all()
            err = rel_l2(a, b)
            assert err <= GEMM_REL_L2, err
            assert err <= 1e-5, err
    finally:
        w.free()


def test_noalloc_rejects_oversized_batch(gpu):
    import torch

    w = q35cu.Weight.synth_fp8(4243, 256, 4096)
    try:
        m = (8 << 20) // 4096 + 1  # one token more than the fixed array holds
        X = torch.zeros((m, 4096), device="cuda")
        Y = torch.zeros((m, 256), device="cuda")
        gpu.q35cu_clear_error()
        rc = _call_noalloc(w, X, Y)
        assert rc == q35cu.ERR_ARG
        assert "exceed" in q35cu.last_error()[1]
        assert bool((Y == 0).all())  # nothing was launched
    finally:
        w.free()
