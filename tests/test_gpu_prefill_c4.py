"""Benchmark configuration 4 on the GPU: the long prefill (M = 8192 tokens).

The engine's batch prefill (qwen35-c/src/q35_model.c:980-1104) hands every
projection of a layer to q35_mm_fp8_batch (qwen35-c/src/q35_mm.c:158-172)
with all M tokens.  At M = 8192 the tensor-core GEMM walks 43 token tiles per
weight row block (the last one partial) and its prepared activations no
longer fit in L2 (285 MB for `down`); these tests pin that shape:

* the `down` (5120 x 17408) and `gate` (17408 x 5120) projections alone,
  sampled tokens against fp64 and against the compiled reference's own
  batch matmul (relative L2 <= 5e-3, the prefill contract, and <= 1e-5 as a
  sanity bound), the whole output finite, the device status word clean;
* the back-to-back layer sequence the benchmark times (qkv / z or q / k / v,
  bf16 conversion, out / o, gate, up, down, every GEMM sharing one
  workspace), each projection checked on sampled tokens against fp64 on the
  very bf16 input the GPU consumed.
"""
from __future__ import annotations

import numpy as np
import pytest

import q35cu
from parity import GEMM_REL_L2, rel_l2

pytestmark = pytest.mark.gpu
TIGHT = 1e-5
M = 8192


def _tokens(m, seed, n=40):
    """Sampled token rows: random ones plus the first and the last (the last
    token tile is partial at M = 8192: 43 x 192 = 8256)."""
    pick = np.random.default_rng(seed).choice(m, n, replace=False)
    return np.unique(np.concatenate([pick, [0, m - 1, 8064]]))


@pytest.mark.parametrize("name,rows,cols", [("down", 5120, 17408), ("gate", 17408, 5120)])
def test_gemm_m8192(gpu, orc, ref, name, rows, cols):
    import torch

    w = q35cu.Weight.synth_fp8(61000 + rows, rows, cols)
    try:
        Wh, sch = w.download_fp8()
        g = torch.Generator(device="cuda").manual_seed(rows + cols)
        X = torch.randn((M, cols), device="cuda", generator=g).to(torch.bfloat16)
        Y = torch.full((M, rows), float("nan"), device="cuda")
        work = torch.empty(q35cu.gemm_workspace_bytes(M, cols), dtype=torch.uint8, device="cuda")
        for _ in range(2):  # the second call reuses the workspace, as the benchmark does
            q35cu.gemm(w, X, Y, work)
        torch.cuda.synchronize()
        q35cu.check_device_status()
        assert bool(torch.isfinite(Y).all())
        pick = _tokens(M, rows)
        Xp = np.ascontiguousarray(X[torch.from_numpy(pick).cuda()].float().cpu().numpy())
        Yp = Y[torch.from_numpy(pick).cuda()].cpu().numpy()
        Y64, _ = orc.mm_fp8_f64(Wh, sch, Xp)
        err = rel_l2(Yp, Y64)
        assert err <= GEMM_REL_L2, (name, err)
        assert err <= TIGHT, (name, err)
        Yr = ref.mm_fp8_batch(Wh, sch, Xp[:6])
        err_ref = rel_l2(Yp[:6], Yr)
        assert err_ref <= GEMM_REL_L2 and err_ref <= TIGHT, (name, err_ref)
    finally:
        w.free()


@pytest.fixture(scope="module")
def small_stack(gpu):
    import stack

    st = stack.Stack(0, 1, n_layers=4)  # layers 0-2 DeltaNet, layer 3 GQA
    yield st
    st.free()


@pytest.mark.parametrize("kind", ["dn", "gqa"])
def test_config4_layer_sequence(small_stack, orc, kind):
    """One layer of the benchmark's configuration-4 sequence, run twice back
    to back; every GEMM of the second run checked on sampled tokens."""
    import torch

    import prefill

    pf = prefill.PrefillLayers(small_stack, m=M)
    L = pf.dn if kind == "dn" else pf.gqa
    pf.layer(L)
    kept = {}
    pf.layer(L, keep=kept)
    torch.cuda.synchronize()
    q35cu.check_device_status()
    pick = torch.from_numpy(_tokens(M, 7 if kind == "dn" else 8, n=12)).cuda()
    outs = {p.name: pf.col[p.name] for p in L.col_in}
    outs.update({L.attn_out.name: pf.o, "gate": pf.gu["gate"], "up": pf.gu["up"], "down": pf.y})
    projs = {p.name: p for p in L.col_in + [L.attn_out, L.gate, L.up, L.down]}
    for name, out in outs.items():
        assert bool(torch.isfinite(out).all()), name
        Wh, sch = projs[name].w.download_fp8()
        Xp = np.ascontiguousarray(kept[name][pick].float().cpu().numpy())
        Y64, _ = orc.mm_fp8_f64(Wh, sch, Xp)
        err = rel_l2(out[pick].cpu().numpy(), Y64)
        assert err <= GEMM_REL_L2, (kind, name, err)
        assert err <= TIGHT, (kind, name, err)
