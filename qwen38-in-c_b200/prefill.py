"""Long prefill through the projection set (benchmark configuration 4) -- a
harness over libq35cuda's C-ABI, shared by bench.py and the GPU tests.

The engine's batch prefill (qwen35-c/src/q35_model.c:980-1104) runs every
projection of a layer on all M tokens at once through q35_mm_fp8_batch
(q35_deltanet.c:387-390, q35_attn.c:305-307, q35_model.c:972-975).  One
layer here issues the same projections, in the same order, on the weights of
a ``stack.Stack`` (this rank's tensor-parallel shards):

  DeltaNet: qkv, z = GEMM(x)           column-parallel
            o = GEMM_out(bf16(z))       row-parallel (the caller-batched out)
  GQA:      q, k, v = GEMM(x)           column-parallel
            o = GEMM_o(bf16(attn))      row-parallel (attn: the local heads'
                                        attention output, a stand-in)
  MLP:      gate, up = GEMM(bf16(o))    column-parallel
            y = GEMM_down(bf16(gate))   row-parallel

Every GEMM is ``q35cu_gemm_fp8`` (the tcgen05 kernel, bf16 activations, one
caller workspace).  The recurrence, attention and swiglu arithmetic between
projections is not part of the matmul path and is not run.

Tensor parallelism (world > 1): "literal" all-gathers each column-parallel
output ([M, N/p] fp32 per rank) and all-reduces each row-parallel partial
([M, 5120] fp32) with NCCL; "paired" (Megatron) drops the all-gathers -- the
row-parallel projection consumes the local shard.
"""
from __future__ import annotations

import q35cu
import stack


class PrefillLayers:
    """Device buffers for M tokens through one layer of each kind of `st`."""

    def __init__(self, st: "stack.Stack", m: int = 8192, scheme: str = "literal", seed: int = 4321):
        import torch

        assert scheme in ("literal", "paired")
        self.st, self.m, self.scheme = st, m, scheme
        self.world = st.world
        self.dn = next(L for L in st.layers if L.kind == "dn")
        self.gqa = next(L for L in st.layers if L.kind == "gqa")
        dev = st.dev
        f32 = dict(dtype=torch.float32, device=dev)
        g = torch.Generator(device=dev).manual_seed(seed)
        # bf16-rounded N(0, 1) activations (the configuration's input)
        self.x = torch.randn((m, stack.HIDDEN), device=dev, generator=g).to(torch.bfloat16)
        layers = (self.dn, self.gqa)
        kmax = max(max(p.w.cols for p in L.col_in + [L.attn_out, L.gate, L.up, L.down]) for L in layers)
        self.work = torch.empty(q35cu.gemm_workspace_bytes(m, kmax), dtype=torch.uint8, device=dev)
        self.xb = torch.empty((m * kmax,), dtype=torch.bfloat16, device=dev)
        self.o = torch.empty((m, stack.HIDDEN), **f32)
        self.y = torch.empty((m, stack.HIDDEN), **f32)
        self.col = {p.name: torch.empty((m, p.window[1]), **f32) for L in layers for p in L.col_in}
        literal = scheme == "literal" and self.world > 1
        self.gath = {k: torch.empty((self.world * v.numel(),), **f32) for k, v in self.col.items()} if literal else {}
        g_n = self.dn.gate.window[1]
        self.gu = {n: torch.empty((m, g_n), **f32) for n in ("gate", "up")}
        self.gu_g = {n: torch.empty((self.world * m * g_n,), **f32) for n in self.gu} if literal else {}
        # stands in for the local heads' attention output
        self.attn = torch.randn((m, self.gqa.attn_out.window[3]), device=dev, generator=g)

    def bf16(self, src, stream=None):
        """bf16(src) into the shared conversion buffer, as [rows, cols]."""
        n = src.numel()
        q35cu.f32_to_bf16(src, self.xb[:n], stream)
        return self.xb[:n].view(src.shape[0], -1)

    def layer(self, L, stream=None, keep=None) -> None:
        """Issue one layer's projections (asynchronous on `stream`).  `keep`, a
        dict, receives clones of every GEMM's bf16 input (for checks)."""
        literal = self.scheme == "literal" and self.world > 1

        def run(w, xin, yout, name):
            if keep is not None:
                keep[name] = xin.clone()
            q35cu.gemm(w, xin, yout, self.work, stream)

        for p in L.col_in:
            run(p.w, self.x, self.col[p.name], p.name)
            if literal:
                q35cu.allgather(self.col[p.name], self.gath[p.name], stream)
        src = self.col["z"] if L.kind == "dn" else self.attn
        run(L.attn_out.w, self.bf16(src, stream), self.o, L.attn_out.name)
        if self.world > 1:
            q35cu.allreduce(self.o, stream)
        xo = self.bf16(self.o, stream)
        run(L.gate.w, xo, self.gu["gate"], "gate")
        run(L.up.w, xo, self.gu["up"], "up")
        if literal:
            for n in ("gate", "up"):
                q35cu.allgather(self.gu[n], self.gu_g[n], stream)
        run(L.down.w, self.bf16(self.gu["gate"], stream), self.y, "down")
        if self.world > 1:
            q35cu.allreduce(self.y, stream)

    def flops(self, L) -> float:
        """This rank's GEMM flops for one layer of L's kind."""
        return 2.0 * self.m * sum(p.window[1] * p.window[3] for p in L.col_in + [L.attn_out, L.gate, L.up, L.down])
