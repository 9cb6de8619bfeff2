"""The decode chain (q35cu_chain_*): the 64-layer step's projections as one
cooperative launch must give exactly the per-projection launches' results
(each output depends only on its row and K, not on how rows meet CTAs), run
after run, and inside a CUDA graph replay too."""
from __future__ import annotations

import pytest


@pytest.mark.gpu
def test_chain_matches_step(gpu):
    import torch

    import stack

    st = stack.Stack(0, 1, n_layers=4)
    try:
        st.x.copy_(torch.randn(st.x.shape, generator=torch.Generator().manual_seed(3)).cuda())
        st.step()
        torch.cuda.synchronize()
        ref = (st.y.clone(), st.o_buf.clone(), st.col_local.clone(), st.gu_local.clone())
        for buf in (st.y, st.o_buf, st.col_local, st.gu_local):
            buf.fill_(float("nan"))
        for _ in range(3):  # repeat: the grid barrier's counters are reset between launches
            st.step_chain()
            torch.cuda.synchronize()
            got = (st.y, st.o_buf, st.col_local, st.gu_local)
            for a, b in zip(ref, got):
                assert torch.equal(a, b)
        # a captured replay of the chain
        st.y.zero_()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                st.step_chain(s)
        torch.cuda.current_stream().wait_stream(s)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(ref[0], st.y)
        del g
        import ctypes as C

        import q35cu

        status = C.c_uint32(0)
        q35cu.check(q35cu.load().q35cu_device_status(C.byref(status), 1))
        assert status.value == 0
    finally:
        st.free()


@pytest.mark.gpu
def test_chain_rejects_bad_ops(gpu):
    import torch

    import q35cu

    w = q35cu.Weight.synth_fp8(5, 256, 200)  # cols not a multiple of 128
    ch = q35cu.Chain()
    try:
        x = torch.zeros(200, device="cuda")
        y = torch.empty(256, device="cuda")
        with pytest.raises(q35cu.Q35Error):
            ch.add([w], x, [y])
        with pytest.raises(q35cu.Q35Error):
            ch.add([w], x, [y], mode=7)
    finally:
        ch.free()
        w.free()
